"""Builds the native libraries of heteromm_b200 in-tree.

  lib/libheteromm_cuda.so   the C ABI (include/heteromm_cuda.h) and its sm_100a
                            kernels, compiled by nvcc from csrc/*.cu
  lib/libheteromm_steps.so  the C++17 heteromm step API (include/heteromm/dev),
                            CPU bodies and GPU adapters (src/*.cpp), linked
                            to the former
  lib/heteromm_cpp_kernels<ext>  Python bindings of the steps under the names the
                            reference's pipeline generator calls
                            (src/py/heteromm_cpp_kernels.cpp, pybind11)

nvcc cross-compiles for sm_100a without a GPU; the built .so files travel with
the repository snapshot to the GPU machine.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
INC = os.path.join(ROOT, "include")
LIB_DIR = os.path.join(PKG, "lib")
CUDA_LIB = os.path.join(LIB_DIR, "libheteromm_cuda.so")
STEPS_LIB = os.path.join(LIB_DIR, "libheteromm_steps.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _newer(target: str, sources: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout)
        raise RuntimeError(f"build failed: {' '.join(cmd[:3])} ... (exit {r.returncode})")


def build_cuda(force: bool = False, verbose: bool = False) -> str:
    srcs = sorted(glob.glob(os.path.join(PKG, "csrc", "*.cu")))
    deps = srcs + glob.glob(os.path.join(PKG, "csrc", "*.cuh")) + [os.path.join(INC, "heteromm_cuda.h")]
    if force or _newer(CUDA_LIB, deps):
        os.makedirs(LIB_DIR, exist_ok=True)
        cmd = [NVCC, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
               f"-I{INC}", "-o", CUDA_LIB, *srcs]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        _run(cmd)
    return CUDA_LIB


def build_steps(force: bool = False) -> str:
    srcs = sorted(glob.glob(os.path.join(PKG, "src", "*.cpp")))
    if not srcs:
        return ""
    deps = srcs + glob.glob(os.path.join(PKG, "src", "*.h")) + \
        glob.glob(os.path.join(INC, "heteromm", "**", "*.h"), recursive=True) + [CUDA_LIB]
    if force or _newer(STEPS_LIB, deps):
        cmd = ["g++", "-std=c++17", "-O2", "-ffp-contract=off", "-fPIC", "-shared", "-Wall",
               "-Wextra", f"-I{INC}",
               "-I/usr/local/cuda/include", "-o", STEPS_LIB, *srcs, f"-L{LIB_DIR}",
               "-lheteromm_cuda", "-Wl,-rpath,$ORIGIN", "-L/usr/local/cuda/lib64", "-lcudart"]
        _run(cmd)
    return STEPS_LIB


def py_kernels_path() -> str:
    import sysconfig
    return os.path.join(LIB_DIR, "heteromm_cpp_kernels" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_py_kernels(force: bool = False) -> str:
    """The pybind11 module heteromm_cpp_kernels, linked to the step library."""
    import sysconfig
    try:
        import pybind11
    except ImportError:   # bindings are optional; the C ABI and step API stand alone
        return ""
    src = os.path.join(PKG, "src", "py", "heteromm_cpp_kernels.cpp")
    out = py_kernels_path()
    deps = [src, STEPS_LIB, os.path.join(PKG, "src", "packed.h")] + \
        glob.glob(os.path.join(INC, "heteromm", "**", "*.h"), recursive=True)
    if force or _newer(out, deps):
        cmd = ["g++", "-std=c++17", "-O2", "-fPIC", "-shared", "-fvisibility=hidden",
               f"-I{pybind11.get_include()}", f"-I{sysconfig.get_paths()['include']}",
               f"-I{INC}", f"-I{os.path.join(PKG, 'src')}", "-o", out, src, f"-L{LIB_DIR}",
               "-lheteromm_steps", "-Wl,-rpath,$ORIGIN"]
        _run(cmd)
    return out


def build(force: bool = False) -> None:
    build_cuda(force)
    build_steps(force)
    build_py_kernels(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
    print(CUDA_LIB)
