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


def test_prompts_match_the_product_generator():
    import numpy as np

    sys.path.insert(0, ROOT)
    import bench
    from inferox_b200 import synth
    for v, n, s in ((128256, 1024, 0), (32000, 17, 3)):
        assert np.array_equal(bench.prompt_ids(v, n, s), synth.prompt_ids(v, n, seq_index=s))


def test_reference_arm_loads_only_the_oracle():
    """`--impl reference` on a 1-layer, 4096-token-vocabulary cut of the 8B
    shape: it prints its line
    with the requested steps and warm-up, the same config the GPU arm reports,
    and neither imports the product package nor maps its library."""
    code = (
        "import json, runpy, sys\n"
        f"sys.argv = ['bench.py', '--impl', 'reference', '--layers', '1', '--vocab', '4096', '--steps', '2', '--warmup', '3']\n"
        f"runpy.run_path({BENCH!r}, run_name='__main__')\n"
        "maps = open('/proc/self/maps').read()\n"
        "print(json.dumps({'pkg': 'inferox_b200' in sys.modules, 'so': 'libinferox_b200' in maps,"
        " 'oracle': 'librefcpu' in maps}))\n")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=900, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    import json
    lines = [json.loads(x) for x in r.stdout.splitlines() if x.startswith("{")]
    line, seen = lines[0], lines[-1]
    assert seen == {"pkg": False, "so": False, "oracle": True}
    assert line["impl"] == "reference" and line["steps"] == 2 and line["warmup"] == 3
    assert line["config"]["decode_context"] == [1027, 1029]
    assert line["cpu_baseline"]["cores"] >= 1 and line["value"] > 0
