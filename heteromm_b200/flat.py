"""Torch-facing wrappers of the flat score / select entry points.

Device memory, streams and workspaces come from PyTorch (caching allocator,
current stream); the work itself runs in libheteromm_cuda.so through its C ABI.
"""
from __future__ import annotations

import torch

from ._abi import call, load

_ws_cache: dict = {}


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t):
    return None if t is None else t.data_ptr()


def workspace(nbytes: int, device) -> torch.Tensor:
    """A reusable per-device scratch buffer of at least nbytes."""
    key = torch.device(device).index
    buf = _ws_cache.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _ws_cache[key] = buf
    return buf


def _check(t: torch.Tensor, dtype, name: str):
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def ip_score_f32(mem: torch.Tensor, queries: torch.Tensor) -> torch.Tensor:
    """scores [nq, n] = exact fp32 inner products (reference order)."""
    _check(mem, torch.float32, "mem"); _check(queries, torch.float32, "queries")
    q2 = queries.reshape(-1, queries.shape[-1])
    n, d = mem.shape
    out = torch.empty((q2.shape[0], n), dtype=torch.float32, device=mem.device)
    call("hmm_ip_score_f32", mem.data_ptr(), n, d, q2.data_ptr(), q2.shape[0], out.data_ptr(),
         _stream())
    return out


def topk_f32(scores: torch.Tensor, k: int, want_scores: bool = True):
    _check(scores, torch.float32, "scores")
    s2 = scores.reshape(-1, scores.shape[-1])
    nq, n = s2.shape
    idx = torch.empty((nq, k), dtype=torch.int32, device=scores.device)
    sc = torch.empty((nq, k), dtype=torch.float32, device=scores.device) if want_scores else None
    need = load().hmm_topk_f32_workspace_size(n, nq, k)
    ws = workspace(need, scores.device)
    call("hmm_topk_f32", s2.data_ptr(), n, nq, k, idx.data_ptr(), _ptr(sc), ws.data_ptr(),
         ws.numel(), _stream())
    return idx, sc


def threshold_bitmap_f32(scores: torch.Tensor, threshold: float) -> torch.Tensor:
    _check(scores, torch.float32, "scores")
    s2 = scores.reshape(-1, scores.shape[-1])
    nq, n = s2.shape
    out = torch.empty((nq, (n + 63) // 64), dtype=torch.int64, device=scores.device)
    call("hmm_threshold_bitmap_f32", s2.data_ptr(), n, nq, float(threshold), out.data_ptr(),
         _stream())
    return out


def ip_topk_f32(mem: torch.Tensor, queries: torch.Tensor, k: int, threshold: float | None = None,
                want_scores: bool = True):
    """Fused score + top-k (+ threshold bitmap).  Returns (idx int32 [nq,k],
    scores fp32 [nq,k] or None, bitmap int64 [nq, ceil(n/64)] or None)."""
    _check(mem, torch.float32, "mem"); _check(queries, torch.float32, "queries")
    q2 = queries.reshape(-1, queries.shape[-1])
    n, d = mem.shape
    nq = q2.shape[0]
    idx = torch.empty((nq, k), dtype=torch.int32, device=mem.device)
    sc = torch.empty((nq, k), dtype=torch.float32, device=mem.device) if want_scores else None
    bm = (torch.empty((nq, (n + 63) // 64), dtype=torch.int64, device=mem.device)
          if threshold is not None else None)
    need = load().hmm_ip_topk_f32_workspace_size(n, d, nq, k)
    ws = workspace(need, mem.device)
    call("hmm_ip_topk_f32", mem.data_ptr(), n, d, q2.data_ptr(), nq, k, idx.data_ptr(), _ptr(sc),
         float(threshold if threshold is not None else 0.0), _ptr(bm), ws.data_ptr(), ws.numel(),
         _stream())
    return idx, sc, bm


def ip_topk_bf16(mem: torch.Tensor, queries: torch.Tensor, k: int, row_offset: int = 0,
                 status: torch.Tensor | None = None):
    """One shard of a bf16 memory: returns (global idx int64 [nq,k], scores fp32 [nq,k]).
    With `status` (int32 device word, zeroed by the caller) the call never
    waits for the stream (hmm_ip_topk_bf16_async); check_status(status) later
    raises HmmError for a timeout or a pool overflow."""
    if mem.dtype == torch.bfloat16:
        mem = mem.view(torch.int16)
    if queries.dtype == torch.bfloat16:
        queries = queries.view(torch.int16)
    _check(mem, torch.int16, "mem"); _check(queries, torch.int16, "queries")
    q2 = queries.reshape(-1, queries.shape[-1])
    n, d = mem.shape
    nq = q2.shape[0]
    idx = torch.empty((nq, k), dtype=torch.int64, device=mem.device)
    sc = torch.empty((nq, k), dtype=torch.float32, device=mem.device)
    need = load().hmm_ip_topk_bf16_workspace_size(n, d, nq, k)
    ws = workspace(need, mem.device)
    if status is None:
        call("hmm_ip_topk_bf16", mem.data_ptr(), n, d, q2.data_ptr(), nq, k, int(row_offset),
             idx.data_ptr(), sc.data_ptr(), ws.data_ptr(), ws.numel(), _stream())
    else:
        _check(status, torch.int32, "status")
        call("hmm_ip_topk_bf16_async", mem.data_ptr(), n, d, q2.data_ptr(), nq, k,
             int(row_offset), idx.data_ptr(), sc.data_ptr(), status.data_ptr(), ws.data_ptr(),
             ws.numel(), _stream())
    return idx, sc


def check_status(status: torch.Tensor) -> None:
    """Waits for the stream and raises HmmError if the device status word has
    bits set (HMM_ERR_TIMEOUT, HMM_ERR_UNSUPPORTED for a pool overflow,
    HMM_ERR_BOUNDS for the paged kernels' bounds flags)."""
    call("hmm_status_read", status.data_ptr(), _stream())


def shard_merge_topk(cand_scores: torch.Tensor, cand_idx: torch.Tensor, k: int):
    """cand_* [n_shards, nq, k] -> (scores [nq,k], idx int64 [nq,k])."""
    _check(cand_scores, torch.float32, "cand_scores"); _check(cand_idx, torch.int64, "cand_idx")
    n_shards, nq, kk = cand_scores.shape
    if kk != k:
        raise ValueError("candidate lists must hold k entries")
    out_s = torch.empty((nq, k), dtype=torch.float32, device=cand_scores.device)
    out_i = torch.empty((nq, k), dtype=torch.int64, device=cand_scores.device)
    call("hmm_shard_merge_topk", cand_scores.data_ptr(), cand_idx.data_ptr(), n_shards, nq, k,
         out_s.data_ptr(), out_i.data_ptr(), None, 0, _stream())
    return out_s, out_i
