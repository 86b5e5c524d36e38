"""Row-sharded retrieval over the ranks of one torch.distributed group.

Rank r of P owns the contiguous rows [r*N/P, (r+1)*N/P) (the last rank takes
the remainder), scores them locally with global row indices, and one
all-gather of the (score, index) candidates (packed into one byte buffer per
rank, so one collective carries both) lets every rank merge the same
global top-k (score desc, global index asc).  The reference has no
multi-device path; this is the exchange its single-device top-k implies.

The local top-k and the merge are parameters, so the exchange itself runs
unchanged with NCCL on GPUs (ip_topk_bf16 + shard_merge_topk) and with gloo
on CPU ranks in the tests.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist


def shard_range(n_rows: int, rank: int, world: int) -> tuple[int, int]:
    """[r0, r1) of the rows rank `rank` owns."""
    per = n_rows // world
    r0 = rank * per
    r1 = n_rows if rank == world - 1 else r0 + per
    return r0, r1


def gather_merge(scores: torch.Tensor, idx: torch.Tensor, k: int,
                 merge: Callable[[torch.Tensor, torch.Tensor, int], tuple],
                 group=None) -> tuple[torch.Tensor, torch.Tensor]:
    """All-gathers every rank's [nq, k] (scores, global indices) and merges
    them with `merge(scores [P, nq, k], idx [P, nq, k], k) -> (scores, idx)`.
    With one rank the local result is returned as is."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1:
        return scores, idx
    # one collective: each rank's scores and indices packed as bytes, side by side
    ns = scores.numel() * scores.element_size()
    mine = torch.cat([scores.contiguous().reshape(-1).view(torch.uint8),
                      idx.contiguous().reshape(-1).view(torch.uint8)])
    g = torch.empty((world, mine.numel()), dtype=torch.uint8, device=mine.device)
    if mine.is_cuda:
        dist.all_gather_into_tensor(g, mine, group=group)
    else:   # gloo: list form
        dist.all_gather(list(g.unbind(0)), mine, group=group)
    gs = g[:, :ns].contiguous().view(scores.dtype).reshape((world,) + tuple(scores.shape))
    gi = g[:, ns:].contiguous().view(idx.dtype).reshape((world,) + tuple(idx.shape))
    return merge(gs, gi, k)


def sharded_ip_topk_bf16(shard: torch.Tensor, queries: torch.Tensor, k: int, row_offset: int,
                         group=None) -> tuple[torch.Tensor, torch.Tensor]:
    """Global (idx [nq, k] int64, scores [nq, k] fp32) of a row-sharded bf16
    memory: the local tensor-core top-k of this rank's shard, then the
    candidate exchange and merge."""
    from .flat import ip_topk_bf16, shard_merge_topk
    idx, sc = ip_topk_bf16(shard, queries, k, row_offset)
    sc, idx = gather_merge(sc, idx, k, shard_merge_topk, group)
    return idx, sc
