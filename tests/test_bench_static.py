"""bench.py on CPU, without running it (the multi-GPU paths need several
GPUs): every module a function imports stays bound to that module for the
whole function, so no later assignment can shadow it. A prefill stopwatch
once reused the name `tp` of the tensor-parallel module, and the
tensor-parallel leg of multi-GPU runs failed on it."""
import ast
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BENCH = os.path.join(ROOT, "bench.py")


def _assigned_names(fn: ast.AST):
    for node in ast.walk(fn):
        if isinstance(node, ast.Name) and isinstance(node.ctx, ast.Store):
            yield node.id, node.lineno
        elif isinstance(node, (ast.FunctionDef, ast.AsyncFunctionDef)) and node is not fn:
            yield node.name, node.lineno


def test_imported_modules_are_not_rebound():
    tree = ast.parse(open(BENCH).read())
    problems = []
    for fn in [n for n in ast.walk(tree) if isinstance(n, ast.FunctionDef)]:
        imported = set()
        for node in ast.walk(fn):
            if isinstance(node, (ast.Import, ast.ImportFrom)):
                for a in node.names:
                    imported.add(a.asname or a.name.split(".")[0])
        for name, line in _assigned_names(fn):
            if name in imported:
                problems.append(f"{fn.name}: line {line} rebinds imported name {name!r}")
    assert not problems, problems


def test_help_runs_without_a_gpu():
    r = subprocess.run([sys.executable, BENCH, "--help"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and "--gpus" in r.stdout and "--impl" in r.stdout
