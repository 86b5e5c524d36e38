"""The deploy layer (include/heteromm/deploy: MemoryManager, ScheduleConfig,
PagedAttention; the interfaces of the reference's toolchain/frontend/deploy)
through tests/cpp/test_deploy.cpp, compiled with g++ against the headers and
linked to libheteromm_steps.so.

CPU: the schedule reader and rule matching, the pipeline on CPU kernels
against the steps composed by hand, functional tests, FPGA stubs, the
projection-weight generator.  GPU (`--gpu`): the pipeline scheduled on the
GPU, the device-resident pass against the step-by-step GPU route (bit-exact)
and the CPU pipeline (rtol 2e-5, atol 2e-6), and its host->device traffic."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def exe(tmp_path_factory):
    from heteromm_b200 import build
    build.build_cuda()
    lib = build.build_steps()
    libdir = os.path.dirname(lib)
    out = str(tmp_path_factory.mktemp("deploy") / "test_deploy")
    cc = subprocess.run(
        ["g++", "-std=c++17", "-O1", "-Wall", "-Wextra", "-o", out,
         os.path.join(ROOT, "tests", "cpp", "test_deploy.cpp"),
         f"-I{os.path.join(ROOT, 'include')}", f"-L{libdir}", "-lheteromm_steps",
         f"-Wl,-rpath,{libdir}"],
        stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    assert cc.returncode == 0, cc.stdout[-4000:]
    assert "warning" not in cc.stdout, cc.stdout[-4000:]
    return out


def test_deploy_layer_cpu(exe):
    run = subprocess.run([exe], stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True,
                         timeout=300)
    assert run.returncode == 0, run.stdout[-6000:]
    assert "PASSED: 0 failure(s)" in run.stdout


@pytest.mark.gpu
def test_deploy_layer_gpu(cuda, exe):
    run = subprocess.run([exe, "--gpu"], stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                         text=True, timeout=600)
    print(run.stdout[-3000:])
    assert run.returncode == 0, run.stdout[-6000:]
    assert "PASSED: 0 failure(s)" in run.stdout
