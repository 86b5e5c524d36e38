"""The reference's own doctest unit tests (toolchain/frontend/dev/unittest)
compiled unchanged against this build's C++ step API (include/heteromm/dev)
and linked to libheteromm_steps.so: the drop-in check of the step
signatures and of the functional-test contract of execute().

Runs where the reference checkout is present (this CPU-only check copies the
test sources and doctest.h to a scratch directory; nothing is copied into
the repository); skipped elsewhere."""
import os
import shutil
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
from conftest import REFERENCE  # noqa: E402

REF_UNITTEST = os.path.join(REFERENCE, "toolchain", "frontend", "dev", "unittest")
TESTS = ["test_innerproduct", "test_topk_retrieval", "test_threshold_retrieval",
         "test_paged_kv_index_builder", "test_block_sparse_attention"]


@pytest.fixture(scope="module")
def steps_lib():
    from heteromm_b200 import build
    build.build_cuda()
    lib = build.build_steps()
    assert lib and os.path.exists(lib)
    return lib


@pytest.mark.skipif(not os.path.isdir(REF_UNITTEST), reason="reference checkout not present")
@pytest.mark.parametrize("name", TESTS)
def test_reference_unittest_passes_against_this_api(steps_lib, name):
    dev = os.path.join(ROOT, "include", "heteromm", "dev")
    with tempfile.TemporaryDirectory() as tmp:
        os.makedirs(os.path.join(tmp, "unittest"))
        for f in (f"{name}.cpp", "doctest.h"):
            shutil.copy(os.path.join(REF_UNITTEST, f), os.path.join(tmp, "unittest", f))
        os.symlink(os.path.join(dev, "steps"), os.path.join(tmp, "steps"))
        os.symlink(os.path.join(dev, "types"), os.path.join(tmp, "types"))
        exe = os.path.join(tmp, name)
        libdir = os.path.dirname(steps_lib)
        cc = subprocess.run(
            ["g++", "-std=c++17", "-O1", "-o", exe, os.path.join(tmp, "unittest", f"{name}.cpp"),
             f"-L{libdir}", "-lheteromm_steps", f"-Wl,-rpath,{libdir}"],
            stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
        assert cc.returncode == 0, cc.stdout[-4000:]
        run = subprocess.run([exe], stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True,
                             timeout=120)
        assert run.returncode == 0, run.stdout[-4000:]
        assert "Status: SUCCESS" in run.stdout
