"""The reference's own unit tests, run unchanged against this repository's
drop-in operator API on the GPU.

oracle/Makefile (target ref-tests, run by build() where the reference
sources are present) compiles every test program of the reference —
test/kernel/test_*.cu and test/core/test_tensor.cu, e.g.
test/kernel/test_embedding.cu:21 and test/kernel/test_linear.cu:289-406 —
against llama2_b200/cpp/include (the reference's header paths, template
parameters and argument order) with a runnable GoogleTest stand-in, and
links them to llama2_b200/libllama2_b200.so. Each program runs its TESTs
with the reference's own expectations and tolerances; this test requires
every one of them to pass.
"""
import glob
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN_DIR = os.path.join(ROOT, "oracle", "_ref", "tests")
PROGRAMS = sorted(os.path.basename(p) for p in glob.glob(os.path.join(BIN_DIR, "test_*"))
                  if os.access(p, os.X_OK) and not p.endswith(".o"))

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _lib(cuda_lib):
    yield


def test_programs_were_built():
    if not PROGRAMS:
        pytest.skip("the reference's test programs were not built here (no reference sources at build time)")
    assert len(PROGRAMS) == 15, PROGRAMS


@pytest.mark.parametrize("program", PROGRAMS or ["(none)"])
def test_reference_test_program(program):
    if program == "(none)":
        pytest.skip("the reference's test programs were not built here")
    res = subprocess.run([os.path.join(BIN_DIR, program)], capture_output=True, text=True, timeout=600)
    out = res.stdout + res.stderr
    ran = re.search(r"\[==========\] (\d+) tests ran", out)
    failed = re.findall(r"^\[  FAILED  \] (\S+)$", out, re.M)
    assert res.returncode == 0 and ran and int(ran.group(1)) > 0 and not failed, \
        f"{program}: rc={res.returncode}, failed={sorted(set(failed))}\n{out[-4000:]}"
