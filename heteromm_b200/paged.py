"""Torch-facing wrappers of the paged-KV entry points: block summaries,
block -> page expansion, block-sparse decode attention and the fused decode
step (select the top blocks by summary score, then attend over them).

A paged cache is `pages` [n_pages, page_tokens, D] bf16 (as int16 bit
patterns) plus `page_table` [n_seq, pages_per_seq] int32.
"""
from __future__ import annotations

import torch

from ._abi import call, load
from .flat import _check, _stream, workspace


def paged_kv_summary_f32(keys: torch.Tensor, page_size: int,
                         weight: torch.Tensor | None = None) -> torch.Tensor:
    """PagedKVIndexBuilder on contiguous fp32 keys [n_seq, L, D] (or [L, D]):
    [n_seq, ceil(L/page_size), out_dim] page summaries, bit-exact."""
    _check(keys, torch.float32, "keys")
    k3 = keys if keys.dim() == 3 else keys.unsqueeze(0)
    n_seq, L, D = k3.shape
    out_dim = D
    if weight is not None:
        _check(weight, torch.float32, "weight")
        out_dim = weight.shape[0]
        if weight.shape[1] != D:
            raise ValueError("weight must be [out_dim, D]")
    pages = (L + page_size - 1) // page_size if L > 0 else 0
    out = torch.empty((n_seq, pages, out_dim), dtype=torch.float32, device=keys.device)
    call("hmm_paged_kv_summary_f32", k3.data_ptr(), n_seq, L, D,
         None if weight is None else weight.data_ptr(), out_dim, page_size, out.data_ptr(),
         _stream())
    return out if keys.dim() == 3 else out[0]


def _cache_dims(pages: torch.Tensor, page_table: torch.Tensor):
    _check(pages, torch.int16, "pages")
    _check(page_table, torch.int32, "page_table")
    n_pages, page_tokens, D = pages.shape
    n_seq, pps = page_table.shape
    return n_pages, page_tokens, D, n_seq, pps


def paged_kv_summary_bf16(k_pages: torch.Tensor, page_table: torch.Tensor, seq_len: int,
                          block_tokens: int) -> torch.Tensor:
    """[n_seq, ceil(seq_len/block_tokens), D] fp32 block means of the paged keys."""
    n_pages, pt, D, n_seq, pps = _cache_dims(k_pages, page_table)
    nb = (seq_len + block_tokens - 1) // block_tokens
    out = torch.empty((n_seq, nb, D), dtype=torch.float32, device=k_pages.device)
    ws = workspace(load().hmm_paged_workspace_size(n_seq, 0, block_tokens, D), k_pages.device)
    call("hmm_paged_kv_summary_bf16", k_pages.data_ptr(), n_pages, page_table.data_ptr(), n_seq,
         pps, seq_len, pt, block_tokens, D, out.data_ptr(), ws.data_ptr(), ws.numel(), _stream())
    return out


def paged_kv_minmax_bf16(k_pages: torch.Tensor, page_table: torch.Tensor, seq_len: int,
                         block_tokens: int) -> torch.Tensor:
    """[n_seq, n_blocks, 2, D] fp32 per-block min and max keys (MinMaxIndexMemory:
    for every block its min vector, then its max vector)."""
    n_pages, pt, D, n_seq, pps = _cache_dims(k_pages, page_table)
    nb = (seq_len + block_tokens - 1) // block_tokens
    out = torch.empty((n_seq, nb, 2, D), dtype=torch.float32, device=k_pages.device)
    ws = workspace(load().hmm_paged_workspace_size(n_seq, 0, block_tokens, D), k_pages.device)
    call("hmm_paged_kv_minmax_bf16", k_pages.data_ptr(), n_pages, page_table.data_ptr(), n_seq,
         pps, seq_len, pt, block_tokens, D, out.data_ptr(), ws.data_ptr(), ws.numel(), _stream())
    return out


def block_select_minmax(q: torch.Tensor, minmax: torch.Tensor, top: int) -> torch.Tensor:
    """[n_seq, top] int32: the blocks with the largest upper bound of q.k over their
    keys, sum_j max(q_j min_j, q_j max_j); best first, ties to the lower block, -1
    past the block count.  q [n_seq, D] bf16 bits (int16), minmax
    [n_seq, n_blocks, 2, D] fp32."""
    _check(q, torch.int16, "q")
    _check(minmax, torch.float32, "minmax")
    n_seq, nb, _, D = minmax.shape
    out = torch.empty((n_seq, top), dtype=torch.int32, device=q.device)
    call("hmm_block_select_minmax", q.data_ptr(), minmax.data_ptr(), n_seq, nb, D, top,
         out.data_ptr(), _stream())
    return out


def block_pages(page_table: torch.Tensor, blocks: torch.Tensor, pages_per_block: int):
    """(pages [n_seq, n_sel*ppb] int32, -1 padded; counts [n_seq] int32)."""
    _check(page_table, torch.int32, "page_table")
    _check(blocks, torch.int32, "blocks")
    n_seq, pps = page_table.shape
    n_sel = blocks.shape[1]
    out = torch.empty((n_seq, n_sel * pages_per_block), dtype=torch.int32,
                      device=page_table.device)
    cnt = torch.empty((n_seq,), dtype=torch.int32, device=page_table.device)
    call("hmm_block_pages", page_table.data_ptr(), n_seq, pps, blocks.data_ptr(), n_sel,
         pages_per_block, out.data_ptr(), cnt.data_ptr(), _stream())
    return out, cnt


def block_sparse_attention_bf16(q: torch.Tensor, k_pages: torch.Tensor, v_pages: torch.Tensor,
                                page_table: torch.Tensor, seq_len: int, block_tokens: int,
                                blocks: torch.Tensor) -> torch.Tensor:
    """[n_seq, D] fp32 softmax attention of q over the selected blocks' tokens."""
    n_pages, pt, D, n_seq, pps = _cache_dims(k_pages, page_table)
    _check(v_pages, torch.int16, "v_pages")
    _check(q, torch.int16, "q")
    _check(blocks, torch.int32, "blocks")
    n_sel = blocks.shape[1]
    out = torch.empty((n_seq, D), dtype=torch.float32, device=q.device)
    ws = workspace(load().hmm_paged_workspace_size(n_seq, n_sel, block_tokens, D), q.device)
    call("hmm_block_sparse_attention_bf16", q.data_ptr(), k_pages.data_ptr(), v_pages.data_ptr(),
         n_pages, page_table.data_ptr(), n_seq, pps, seq_len, pt, block_tokens, D,
         blocks.data_ptr(), n_sel, out.data_ptr(), ws.data_ptr(), ws.numel(), _stream())
    return out


def block_sparse_decode_bf16(q: torch.Tensor, summaries: torch.Tensor, k_pages: torch.Tensor,
                             v_pages: torch.Tensor, page_table: torch.Tensor, seq_len: int,
                             block_tokens: int, top_blocks: int,
                             status: torch.Tensor | None = None):
    """One decode step: (selected blocks [n_seq, top_blocks] int32, out [n_seq, D] fp32).

    With `status` (an int32 device tensor the caller zeroes) the call does not
    wait for the stream: bad page-table entries / block ids set its bits, and
    check_status(status) raises for them later."""
    n_pages, pt, D, n_seq, pps = _cache_dims(k_pages, page_table)
    _check(v_pages, torch.int16, "v_pages")
    _check(q, torch.int16, "q")
    _check(summaries, torch.float32, "summaries")
    blocks = torch.empty((n_seq, top_blocks), dtype=torch.int32, device=q.device)
    out = torch.empty((n_seq, D), dtype=torch.float32, device=q.device)
    ws = workspace(load().hmm_paged_workspace_size(n_seq, top_blocks, block_tokens, D),
                   q.device)
    if status is None:
        call("hmm_block_sparse_decode_bf16", q.data_ptr(), summaries.data_ptr(),
             k_pages.data_ptr(), v_pages.data_ptr(), n_pages, page_table.data_ptr(), n_seq, pps,
             seq_len, pt, block_tokens, D, top_blocks, blocks.data_ptr(), out.data_ptr(),
             ws.data_ptr(), ws.numel(), _stream())
    else:
        _check(status, torch.int32, "status")
        call("hmm_block_sparse_decode_bf16_async", q.data_ptr(), summaries.data_ptr(),
             k_pages.data_ptr(), v_pages.data_ptr(), n_pages, page_table.data_ptr(), n_seq, pps,
             seq_len, pt, block_tokens, D, top_blocks, blocks.data_ptr(), out.data_ptr(),
             status.data_ptr(), ws.data_ptr(), ws.numel(), _stream())
    return blocks, out


def check_status(status: torch.Tensor) -> None:
    """Waits for the stream and raises HmmError(HMM_ERR_BOUNDS) if `status` has bits set."""
    call("hmm_status_read", status.data_ptr(), _stream())


def block_sparse_attention_f32(q: torch.Tensor, keys: torch.Tensor, values: torch.Tensor,
                               block_tokens: int, blocks: torch.Tensor) -> torch.Tensor:
    """Attention over contiguous fp32 K/V [n_seq, L, D] (or [L, D]): [n_seq, D] fp32."""
    for t, n in ((q, "q"), (keys, "keys"), (values, "values")):
        _check(t, torch.float32, n)
    _check(blocks, torch.int32, "blocks")
    k3 = keys if keys.dim() == 3 else keys.unsqueeze(0)
    v3 = values if values.dim() == 3 else values.unsqueeze(0)
    q2 = q if q.dim() == 2 else q.unsqueeze(0)
    b2 = blocks if blocks.dim() == 2 else blocks.unsqueeze(0)
    n_seq, L, D = k3.shape
    n_sel = b2.shape[1]
    out = torch.empty((n_seq, D), dtype=torch.float32, device=q.device)
    ws = workspace(load().hmm_paged_workspace_size(n_seq, n_sel, block_tokens, D), q.device)
    call("hmm_block_sparse_attention_f32", q2.data_ptr(), k3.data_ptr(), v3.data_ptr(), n_seq, L,
         D, block_tokens, b2.data_ptr(), n_sel, out.data_ptr(), ws.data_ptr(), ws.numel(),
         _stream())
    return out if q.dim() == 2 else out[0]
