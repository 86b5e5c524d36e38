"""GPU arms of the C++ step API (libheteromm_steps.so) against their CPU
arms: tests/cpp/test_steps_gpu.cpp compiled with g++ and run."""
import os
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

pytestmark = pytest.mark.gpu


def test_step_gpu_arms_match_cpu_arms(cuda):
    from heteromm_b200 import build
    build.build_cuda()
    lib = build.build_steps()
    libdir = os.path.dirname(lib)
    with tempfile.TemporaryDirectory() as tmp:
        exe = os.path.join(tmp, "test_steps_gpu")
        cc = subprocess.run(
            ["g++", "-std=c++17", "-O1", "-o", exe,
             os.path.join(ROOT, "tests", "cpp", "test_steps_gpu.cpp"),
             f"-I{os.path.join(ROOT, 'include')}", f"-L{libdir}", "-lheteromm_steps",
             f"-Wl,-rpath,{libdir}"],
            stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
        assert cc.returncode == 0, cc.stdout[-4000:]
        run = subprocess.run([exe], stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True,
                             timeout=300)
        assert run.returncode == 0, run.stdout[-6000:]
