"""ctypes binding of the C ABI in include/heteromm_cuda.h.

The library is built in-tree (heteromm_b200/lib/libheteromm_cuda.so) by
heteromm_b200.build.  Loading fails loudly when it is missing: there is no
fallback implementation behind these entry points.
"""
from __future__ import annotations

import ctypes as C
import os

from . import build as _build

HMM_OK = 0
HMM_ERR_INVALID, HMM_ERR_CUDA, HMM_ERR_OOM = 1, 2, 3
HMM_ERR_BOUNDS, HMM_ERR_TIMEOUT, HMM_ERR_UNSUPPORTED = 4, 5, 6
STATUS_NAMES = {
    0: "HMM_OK", 1: "HMM_ERR_INVALID", 2: "HMM_ERR_CUDA", 3: "HMM_ERR_OOM",
    4: "HMM_ERR_BOUNDS", 5: "HMM_ERR_TIMEOUT", 6: "HMM_ERR_UNSUPPORTED",
}

_P = C.c_void_p
_I = C.c_int64
_F = C.c_float
_S = C.c_size_t

# name -> (restype, argtypes); mirrors include/heteromm_cuda.h
SIGNATURES = {
    "hmm_last_error": (C.c_char_p, []),
    "hmm_version": (C.c_char_p, []),
    "hmm_ip_score_f32": (C.c_int, [_P, _I, _I, _P, _I, _P, _P]),
    "hmm_topk_f32_workspace_size": (_S, [_I, _I, _I]),
    "hmm_topk_f32": (C.c_int, [_P, _I, _I, _I, _P, _P, _P, _S, _P]),
    "hmm_threshold_bitmap_f32": (C.c_int, [_P, _I, _I, _F, _P, _P]),
    "hmm_ip_topk_f32_workspace_size": (_S, [_I, _I, _I, _I]),
    "hmm_ip_topk_f32": (C.c_int, [_P, _I, _I, _P, _I, _I, _P, _P, _F, _P, _P, _S, _P]),
    "hmm_ip_topk_bf16_workspace_size": (_S, [_I, _I, _I, _I]),
    "hmm_ip_topk_bf16": (C.c_int, [_P, _I, _I, _P, _I, _I, _I, _P, _P, _P, _S, _P]),
    "hmm_ip_topk_bf16_async": (C.c_int, [_P, _I, _I, _P, _I, _I, _I, _P, _P, _P, _P, _S, _P]),
    "hmm_ip_topk_f32_noalloc": (C.c_int, [_P, _I, _I, _P, _I, _I, _P, _P, _F, _P, _P]),
    "hmm_shard_merge_topk_workspace_size": (_S, [_I, _I, _I]),
    "hmm_shard_merge_topk": (C.c_int, [_P, _P, _I, _I, _I, _P, _P, _P, _S, _P]),
    "hmm_paged_kv_summary_f32": (C.c_int, [_P, _I, _I, _I, _P, _I, _I, _P, _P]),
    "hmm_paged_workspace_size": (_S, [_I, _I, _I, _I]),
    "hmm_paged_kv_summary_bf16": (C.c_int, [_P, _I, _P, _I, _I, _I, _I, _I, _I, _P, _P, _S,
                                            _P]),
    "hmm_paged_kv_minmax_bf16": (C.c_int, [_P, _I, _P, _I, _I, _I, _I, _I, _I, _P, _P, _S,
                                           _P]),
    "hmm_block_select_minmax": (C.c_int, [_P, _P, _I, _I, _I, _I, _P, _P]),
    "hmm_block_pages": (C.c_int, [_P, _I, _I, _P, _I, _I, _P, _P, _P]),
    "hmm_block_sparse_attention_bf16": (C.c_int, [_P, _P, _P, _I, _P, _I, _I, _I, _I, _I, _I,
                                                  _P, _I, _P, _P, _S, _P]),
    "hmm_block_sparse_attention_f32": (C.c_int, [_P, _P, _P, _I, _I, _I, _I, _P, _I, _P, _P,
                                                 _S, _P]),
    "hmm_block_sparse_decode_bf16_async": (C.c_int, [_P, _P, _P, _P, _I, _P, _I, _I, _I, _I,
                                                     _I, _I, _I, _P, _P, _P, _P, _S, _P]),
    "hmm_status_read": (C.c_int, [_P, _P]),
    "hmm_block_sparse_decode_bf16": (C.c_int, [_P, _P, _P, _P, _I, _P, _I, _I, _I, _I, _I, _I,
                                               _I, _P, _P, _P, _S, _P]),
    "hmm_bm25_stats_host": (C.c_int, [_P, _I, _P, _I, _P, _P]),
    "hmm_bm25_skips_count": (_S, [_I, _I]),
    "hmm_bm25_prepare": (C.c_int, [_P, _P, _P, _I, _P, _I, _P, C.c_double, _P, _P, _P, _S,
                                   _P]),
    "hmm_bm25_topk_workspace_size": (_S, [_I, _I, _I]),
    "hmm_bm25_csr_workspace_size": (_S, [_I, _I]),
    "hmm_bm25_csr_from_docs": (C.c_int, [_P, _P, _P, _I, _I, _P, _P, _P, _P, _P, _S, _P]),
    "hmm_bm25_topk_csr": (C.c_int, [_P, _P, _I, _I, _I, _P, _P, _I, _I, _I, _P, _P, _P, _S,
                                    _P]),
    "hmm_indexer_workspace_size": (_S, [_I, _I]),
    "hmm_lserve_topk_i16": (C.c_int, [_P, _I, _P, _P, _I, _I, _I, _I, _P, _P, _S, _P]),
    "hmm_seer_budget_i16": (C.c_int, [_P, _I, _P, _P, _I, _I, _I, _P, _P, _S, _P]),
    "hmm_seer_words_per_query": (_I, [_I, _I]),
    "hmm_seer_threshold_i16": (C.c_int, [_P, _I, _P, _P, _I, _I, _I, _P, _P]),
    "hmm_dsa_indexer_fp8_workspace_size": (_S, [_I, _I, _I, _I]),
    "hmm_dsa_indexer_fp8": (C.c_int, [_P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _S,
                                      _P]),
    "hmm_kernel_launches": (_I, []),
    "hmm_profile_enable": (C.c_int, [C.c_int]),
    "hmm_profile_read": (C.c_int, [_P, _P]),
    "hmm_debug_set_wait_limit_ns": (C.c_int, [_I]),
}


class HmmError(RuntimeError):
    def __init__(self, status: int, where: str, msg: str):
        super().__init__(f"{where}: {STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


_lib = None


def lib_path() -> str:
    return _build.CUDA_LIB


def load(build_if_missing: bool = True) -> C.CDLL:
    """Loads libheteromm_cuda.so (building it first if it is absent)."""
    global _lib
    if _lib is None:
        path = lib_path()
        if not os.path.exists(path):
            if not build_if_missing:
                raise FileNotFoundError(f"{path} is not built")
            _build.build_cuda()
        lib = C.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def call(name: str, *args) -> int:
    lib = load()
    st = getattr(lib, name)(*args)
    if st != HMM_OK:
        raise HmmError(st, name, lib.hmm_last_error().decode())
    return st


def last_error() -> str:
    return load().hmm_last_error().decode()


def kernel_launches() -> int:
    """Kernels the CUDA library has launched since it was loaded."""
    return int(load().hmm_kernel_launches())


def profile_enable(on: bool) -> None:
    """Starts / stops CUDA-event timing of the dominant scoring kernel."""
    call("hmm_profile_enable", 1 if on else 0)


def set_wait_limit_ns(ns: int) -> None:
    """Test hook: limit of the tensor-core kernels' bounded waits for the
    calls that follow (ns; negative restores the 2 s default)."""
    call("hmm_debug_set_wait_limit_ns", int(ns))


def profile_read() -> tuple:
    """(summed ms, launches) of the scoring-kernel launches timed since the last read."""
    ms = C.c_double(0.0)
    n = C.c_int64(0)
    call("hmm_profile_read", C.byref(ms), C.byref(n))
    return ms.value, n.value
