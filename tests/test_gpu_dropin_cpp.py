"""The C++ operator API (llama2_b200/cpp: the reference's include/kernel/*.h
signatures over the C ABI) exercised by its C++ test program, which follows
the reference's own test pattern (Tensor<T> on the GPU, launch_*, compare with
the CPU expectation)."""
import os
import subprocess

import pytest

from llama2_b200 import build

pytestmark = pytest.mark.gpu


def test_cpp_dropin_program(cuda_lib):
    exe = build.DROPIN_TEST if os.path.exists(build.DROPIN_TEST) else build.build_dropin_test()
    res = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    print(res.stdout)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "0 failed" in res.stdout
