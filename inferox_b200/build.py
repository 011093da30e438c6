"""Builds libinferox_b200.so in-tree with nvcc for sm_100a.

    python inferox_b200/build.py          # incremental
    python inferox_b200/build.py --clean  # from scratch

(Run it as a script: importing the package loads the library it builds.)

Objects go to inferox_b200/_build/ (git-ignored); the shared library lands
next to this file so it travels with the repository snapshot.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libinferox_b200.so")
CLI_SRC = os.path.join(HERE, "cli", "ifx.cpp")
CLI = os.path.join(HERE, "ifx")  # the command-line program (src/main.rs)
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]


def sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def headers_mtime():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs.append(os.path.join(HERE, "..", "include", "inferox.h"))
    return max(os.path.getmtime(h) for h in hs)


def compile_one(src: str, verbose: bool) -> str:
    obj = os.path.join(BUILD, src + ".o")
    path = os.path.join(CSRC, src)
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(path), headers_mtime()):
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, "-c", path, "-o", obj]
    if src.endswith(".cpp"):
        cmd = [NVCC, "-O3", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "-c", path, "-o", obj]
    if verbose:
        cmd += ["-Xptxas", "-v"] if src.endswith(".cu") else []
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stderr}\n{r.stdout}")
    if verbose and r.stderr:
        sys.stderr.write(f"--- {src}\n{r.stderr}")
    return obj


def build(clean: bool = False, verbose: bool = False) -> str:
    if clean and os.path.isdir(BUILD):
        shutil.rmtree(BUILD)
    os.makedirs(BUILD, exist_ok=True)
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: compile_one(s, verbose), srcs))
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-lcudart", "-lpthread", "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
    build_cli()
    return LIB


def build_cli() -> str:
    """The `ifx` program: host C++ over the library (rpath: its own folder)."""
    deps = [CLI_SRC, LIB, os.path.join(CSRC, "gguf.h")]
    if os.path.exists(CLI) and os.path.getmtime(CLI) >= max(os.path.getmtime(d) for d in deps):
        return CLI
    cmd = ["g++", "-O2", "-std=c++17", "-Wall", CLI_SRC, "-o", CLI, f"-L{HERE}", "-linferox_b200",
           "-Wl,-rpath,$ORIGIN"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"ifx build failed:\n{r.stderr}")
    return CLI


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.clean, a.verbose))
