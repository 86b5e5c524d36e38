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


_copy_streams: dict = {}


def _streams(device):
    """This device's (upload, read-back) copy streams, made once."""
    key = torch.device(device).index
    if key not in _copy_streams:
        _copy_streams[key] = (torch.cuda.Stream(device), torch.cuda.Stream(device))
    return _copy_streams[key]


def dsa_indexer_fp8_host(q_host, keys, w_host, pos0: int, topk: int, chunks=None,
                         sync: bool = True):
    """The DSA indexer from host inputs to host outputs, with the transfers
    hidden behind the work: q_host [T, H, 128] uint8 (e4m3 bits) and w_host
    [T, H] fp32 in host memory (pinned, for the copies to overlap), keys
    [L, 128] already on the device.  Returns pinned host (idx [T, topk] int32,
    scores [T, topk] fp32), equal to dsa_indexer_fp8 on the same inputs.

    The tokens go in slices.  The upload of every slice is queued at once on an
    upload stream; the indexer runs slice after slice on the current stream,
    each as soon as its slice has arrived; each slice's results are read back
    on a third stream as soon as they are done.  So the transfers of slices
    c + 1 and c - 1 overlap the indexer on slice c, and the indexer calls share
    the library workspace in stream order.

    Slices (chunks=None): the scoring kernel runs one block per SM over the
    query-token groups (256 / H tokens each), so a slice costs whole "waves" of
    SM-count groups.  The first slice is one wave (a short exposed upload), the
    last is the ragged remainder (a short exposed read-back), the middle holds
    the rest; the three take as many waves as one call over all tokens.  An
    integer `chunks` cuts that many equal slices of whole 256-token blocks
    instead (each slice then rounds up to whole waves on its own).
    With sync=False the call returns once the current stream has been made to
    wait for the last read-back: the outputs are valid after that stream has
    been synchronised."""
    if q_host.is_cuda or w_host.is_cuda:
        raise ValueError("q_host and w_host must be host tensors")
    _check(keys, torch.uint8, "keys")
    if q_host.dtype != torch.uint8 or w_host.dtype != torch.float32:
        raise ValueError("q_host must be uint8 (e4m3 bits) and w_host float32")
    T, H, D = q_host.shape
    if tuple(w_host.shape) != (T, H):
        raise ValueError("w_host must be [T, H]")
    dev = keys.device
    cur = torch.cuda.current_stream(dev)
    up, down = _streams(dev)
    q_dev = torch.empty((T, H, D), dtype=torch.uint8, device=dev)
    w_dev = torch.empty((T, H), dtype=torch.float32, device=dev)
    idx_h = torch.empty((T, topk), dtype=torch.int32, pin_memory=True)
    sc_h = torch.empty((T, topk), dtype=torch.float32, pin_memory=True)
    if chunks is None:
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        wave = sms * max(1, 256 // H)             # tokens of one wave of the scoring kernel
        n_w = -(-T // wave)
        cuts = [0, wave, (n_w - 1) * wave, T] if n_w >= 3 else [0, wave, T] if n_w == 2 else [0, T]
        bounds = [(a, b) for a, b in zip(cuts, cuts[1:]) if b > a]
    else:
        per = -(-T // max(1, int(chunks)))        # ceil(T / chunks) tokens per slice,
        per = max(256, -(-per // 256) * 256)      # rounded up to whole 256-token blocks
        bounds = [(t0, min(T, t0 + per)) for t0 in range(0, T, per)]
    up.wait_stream(cur)   # buffers allocated on the current stream
    arrived = []
    with torch.cuda.stream(up):
        for t0, t1 in bounds:
            q_dev[t0:t1].copy_(q_host[t0:t1], non_blocking=True)
            w_dev[t0:t1].copy_(w_host[t0:t1], non_blocking=True)
            e = torch.cuda.Event()
            e.record(up)
            arrived.append(e)
    q_dev.record_stream(up)
    w_dev.record_stream(up)
    for (t0, t1), e in zip(bounds, arrived):
        cur.wait_event(e)
        i, s = dsa_indexer_fp8(q_dev[t0:t1], keys, w_dev[t0:t1], pos0 + t0, topk)
        done = torch.cuda.Event()
        done.record(cur)
        with torch.cuda.stream(down):
            down.wait_event(done)
            idx_h[t0:t1].copy_(i, non_blocking=True)
            sc_h[t0:t1].copy_(s, non_blocking=True)
        i.record_stream(down)
        s.record_stream(down)
    cur.wait_stream(down)
    if sync:
        cur.synchronize()
    return idx_h, sc_h
