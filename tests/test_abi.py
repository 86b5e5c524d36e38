"""CPU checks of the C ABI: the library builds, loads, exports every entry
point that include/*.h declares, and rejects bad arguments before touching
the device."""
import ctypes as C
import glob
import os
import re
import subprocess

import pytest

import heteromm_b200 as hmm
from heteromm_b200 import _abi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b(hmm_[a-z0-9_]+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    lib = hmm.load()
    nm = subprocess.run(["nm", "-D", "--defined-only", hmm.lib_path()], capture_output=True,
                        text=True, check=True).stdout
    exported = set(re.findall(r" T (hmm_[a-z0-9_]+)", nm))
    decl = declared_symbols()
    assert decl, "no declarations found"
    missing = decl - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"
    for name in decl:
        assert getattr(lib, name) is not None
    # the ctypes table covers every declaration
    assert decl <= set(_abi.SIGNATURES), sorted(decl - set(_abi.SIGNATURES))


def test_version_and_last_error():
    lib = hmm.load()
    assert lib.hmm_version().startswith(b"heteromm-b200")
    assert isinstance(lib.hmm_last_error(), bytes)


def test_invalid_arguments_rejected_without_device():
    lib = hmm.load()
    P = C.c_void_p(0x1000)  # never dereferenced: validation fails first
    # dim out of range
    st = lib.hmm_ip_topk_f32(P, 10, 0, P, 1, 4, P, None, 0.0, None, P, 1 << 20, None)
    assert st == 1 and "dim" in hmm.last_error()
    # k = 0
    st = lib.hmm_ip_topk_f32(P, 10, 8, P, 1, 0, P, None, 0.0, None, P, 1 << 20, None)
    assert st == 1 and "k must be" in hmm.last_error()
    # k too large for the fused kernel
    st = lib.hmm_ip_topk_f32(P, 10, 8, P, 1, 100000, P, None, 0.0, None, P, 1 << 20, None)
    assert st == 1
    # null memory
    st = lib.hmm_ip_topk_f32(None, 10, 8, P, 1, 4, P, None, 0.0, None, P, 1 << 20, None)
    assert st == 1 and "null" in hmm.last_error()
    # negative sizes
    assert lib.hmm_threshold_bitmap_f32(P, -1, 1, 0.0, P, None) == 1
    assert lib.hmm_topk_f32(P, 10, 1, 0, P, None, P, 1 << 20, None) == 1
    assert lib.hmm_shard_merge_topk(P, P, 0, 1, 4, P, P, None, 0, None) == 1


def test_workspace_sizes_are_positive():
    lib = hmm.load()
    assert lib.hmm_ip_topk_f32_workspace_size(65536, 128, 64, 64) > 64 * 64 * 8
    assert lib.hmm_topk_f32_workspace_size(1000, 3, 10) >= 3 * 10 * 8
    assert lib.hmm_ip_topk_bf16_workspace_size(1 << 26, 128, 256, 100) > 0
    assert lib.hmm_topk_f32_workspace_size(-1, 1, 1) == 0
