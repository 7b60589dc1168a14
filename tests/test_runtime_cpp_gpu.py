"""Runs the C++ test programs built against the TempLit headers
(tests/cpp/*.cpp -> templit_b200/_build/tests/*): the reference's runtime
known-answer suite and compiled-graph cases on cuda::Runtime, through the
real passes::Compiled executor."""
import os
import subprocess

import pytest

from templit_b200 import BUILD_DIR

pytestmark = pytest.mark.gpu

PROGRAMS = ["test_cuda_runtime", "test_cuda_compiled"]


@pytest.mark.parametrize("program", PROGRAMS)
def test_cpp_program(program):
    path = os.path.join(BUILD_DIR, "tests", program)
    if not os.path.exists(path):
        pytest.fail(f"{path} not built (make -C templit_b200 tests)")
    proc = subprocess.run([path], capture_output=True, text=True, timeout=600)
    out = proc.stdout + proc.stderr
    assert proc.returncode == 0, out
    assert "FAIL" not in out, out
    assert out.count("PASS") >= 3, out
