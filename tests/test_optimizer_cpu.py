"""Runs the CPU test of the runtime's program optimiser
(tests/cpp/test_optimizer.cpp): fusion rewrites on hand-built programs in
the shapes the reference's typed executor records, including the cases
that must not fuse.  No GPU needed."""
import os
import subprocess

from templit_b200 import BUILD_DIR


def test_program_optimizer_rewrites():
    path = os.path.join(BUILD_DIR, "tests", "test_optimizer")
    assert os.path.exists(path), "make -C templit_b200 tests"
    proc = subprocess.run([path], capture_output=True, text=True, timeout=120)
    out = proc.stdout + proc.stderr
    assert proc.returncode == 0, out
    assert "FAIL" not in out and out.count("PASS") >= 10, out
