"""Ingest and device residency of the step API (FlatIndexMemory's row log,
include/heteromm/residency.h) through tests/cpp/test_residency.cpp, compiled
with g++ and linked to libheteromm_steps.so.

CPU: the row log's entries, generation chain, bound, and that set_data and
copies break the chain.  GPU (`--gpu`): GPU steps after inserts, pops and
erases agree with the CPU arm while uploading only appended rows and queries;
logs past their bound, copies and set_data fall back to full uploads;
make_resident / release / is_resident; held copies of GPU_MEM-tagged memories;
a resident KV cache."""
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
    out = str(tmp_path_factory.mktemp("residency") / "test_residency")
    cc = subprocess.run(
        ["g++", "-std=c++17", "-O1", "-Wall", "-Wextra", "-o", out,
         os.path.join(ROOT, "tests", "cpp", "test_residency.cpp"),
         f"-I{os.path.join(ROOT, 'include')}", f"-L{libdir}", "-lheteromm_steps",
         f"-Wl,-rpath,{libdir}"],
        stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    assert cc.returncode == 0, cc.stdout[-4000:]
    assert "warning" not in cc.stdout, cc.stdout[-4000:]
    return out


def test_row_log_cpu(exe):
    run = subprocess.run([exe], stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True,
                         timeout=300)
    assert run.returncode == 0, run.stdout[-6000:]
    assert "PASSED: 0 failure(s)" in run.stdout


@pytest.mark.gpu
def test_ingest_and_residency_gpu(cuda, exe):
    run = subprocess.run([exe, "--gpu"], stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                         text=True, timeout=600)
    print(run.stdout[-3000:])
    assert run.returncode == 0, run.stdout[-6000:]
    assert "PASSED: 0 failure(s)" in run.stdout
