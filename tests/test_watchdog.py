"""Failure detection for tensor-parallel calls, on CPU: the bounded wait
behind every tensor-parallel step (inferox_b200/csrc/watchdog.h, used by
tp_wait in tp.cu) against fake streams and communicators: a step that
finishes, a device error, an asynchronous NCCL error (abort once, report
Nccl) and a peer rank that never reaches the collective (abort at the
deadline, report Timeout). No GPU is touched and nothing is made to hang:
the fakes count polls on a fake clock."""
import os
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_bounded_wait_outcomes(tmp_path):
    exe = tmp_path / "watchdog_test"
    src = os.path.join(ROOT, "tests", "cpp", "watchdog_test.cpp")
    subprocess.run(["g++", "-O1", "-std=c++17", "-Wall", "-Werror", src, "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.count("ok  ") == 6, r.stdout


def test_timeout_option_round_trips():
    from inferox_b200 import load_opts
    assert load_opts().tp_timeout_ms == 0  # 0: the library's default (300 s)
    assert load_opts(tp_timeout_ms=1500).tp_timeout_ms == 1500
