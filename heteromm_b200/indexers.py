"""Torch-facing wrappers of the int16 sparse-attention indexers (LServe block
top-k, SeerAttention token budget and threshold bitmap).  Arrays are int16
tensors on the device: past [L, D], queries [nq, D], new_keys [nq, D]."""
from __future__ import annotations

import torch

from ._abi import call, load
from .flat import _check, _stream, workspace


def _common(past, queries, new_keys):
    for t, n in ((past, "past"), (queries, "queries"), (new_keys, "new_keys")):
        _check(t, torch.int16, n)
    return past.shape[0], queries.shape[0], queries.shape[1]


def lserve_topk_i16(past, queries, new_keys, topk: int = 64, block: int = 16):
    L, nq, D = _common(past, queries, new_keys)
    out = torch.empty((nq, topk), dtype=torch.int32, device=queries.device)
    ws = workspace(load().hmm_indexer_workspace_size(L, nq), queries.device)
    call("hmm_lserve_topk_i16", past.data_ptr(), L, queries.data_ptr(), new_keys.data_ptr(), nq,
         D, topk, block, out.data_ptr(), ws.data_ptr(), ws.numel(), _stream())
    return out


def seer_budget_i16(past, queries, new_keys, topk: int = 64):
    L, nq, D = _common(past, queries, new_keys)
    out = torch.empty((nq, topk), dtype=torch.int32, device=queries.device)
    ws = workspace(load().hmm_indexer_workspace_size(L, nq), queries.device)
    call("hmm_seer_budget_i16", past.data_ptr(), L, queries.data_ptr(), new_keys.data_ptr(), nq,
         D, topk, out.data_ptr(), ws.data_ptr(), ws.numel(), _stream())
    return out


def seer_threshold_i16(past, queries, new_keys, threshold: int = 100000):
    L, nq, D = _common(past, queries, new_keys)
    wpq = load().hmm_seer_words_per_query(L, nq)
    out = torch.empty((nq, wpq), dtype=torch.int64, device=queries.device)
    call("hmm_seer_threshold_i16", past.data_ptr(), L, queries.data_ptr(), new_keys.data_ptr(),
         nq, D, threshold, out.data_ptr(), _stream())
    return out


def dsa_indexer_fp8(q, keys, w, pos0: int, topk: int, want_all_scores: bool = False):
    """DSA lightning indexer on FP8 tensor cores.  q [T, H, 128] and keys
    [L, 128] as uint8 e4m3 bit patterns, w [T, H] fp32.  Returns (idx [T, topk]
    int32, scores [T, topk] fp32) and, if asked, every score [T, L]."""
    _check(q, torch.uint8, "q")
    _check(keys, torch.uint8, "keys")
    _check(w, torch.float32, "w")
    T, H, D = q.shape
    L = keys.shape[0]
    idx = torch.empty((T, topk), dtype=torch.int32, device=q.device)
    sc = torch.empty((T, topk), dtype=torch.float32, device=q.device)
    full = torch.empty((T, L), dtype=torch.float32, device=q.device) if want_all_scores else None
    ws = workspace(load().hmm_dsa_indexer_fp8_workspace_size(T, H, L, topk), q.device)
    call("hmm_dsa_indexer_fp8", q.data_ptr(), keys.data_ptr(), w.data_ptr(), T, H, L, D, pos0,
         topk, idx.data_ptr(), sc.data_ptr(), None if full is None else full.data_ptr(),
         ws.data_ptr(), ws.numel(), _stream())
    return (idx, sc, full) if want_all_scores else (idx, sc)
