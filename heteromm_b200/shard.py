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

Failure handling.  The reference's only multi-device code exits the process
on any error (toolchain/backend/p2p_handler/gpu_mem_control.h:9-17).  Here a
rank that never contributes must not hang the others: with a deadline the
exchange is issued asynchronously and polled on the host; when the deadline
passes, the group's communicator is aborted (NCCL: ncclCommAbort through
the process group; created non-blocking by `nccl_options`) and
ExchangeTimeout (status HMM_ERR_TIMEOUT) is raised.
"""
from __future__ import annotations

import time
from typing import Callable

import torch
import torch.distributed as dist

from ._abi import HMM_ERR_TIMEOUT, HmmError


class ExchangeTimeout(HmmError):
    """The candidate exchange did not complete before its host deadline.
    `work` is the abandoned collective (already aborted for NCCL groups)."""

    def __init__(self, msg: str, work=None):
        super().__init__(HMM_ERR_TIMEOUT, "gather_merge", msg)
        self.work = work


def nccl_options(nonblocking: bool = True):
    """ProcessGroupNCCL options whose communicators are created non-blocking
    (ncclConfig_t.blocking = 0): NCCL calls return at once and report their
    state through the communicator's asynchronous error, so a stalled peer
    can be abandoned by ncclCommAbort instead of blocking this host thread."""
    from torch._C._distributed_c10d import ProcessGroupNCCL
    opts = ProcessGroupNCCL.Options()
    opts.config.blocking = 0 if nonblocking else 1
    return opts


def abort_group(group=None) -> bool:
    """Aborts the group's communicators (NCCL only: ncclCommAbort on every
    communicator of the group).  Returns False for backends without abort
    (gloo), whose pending collectives end at the group's own timeout."""
    backend = dist.get_backend(group)
    if backend != "nccl":
        return False
    from torch.distributed import distributed_c10d as c10d
    c10d._abort_process_group(group)
    return True


def wait_with_deadline(work, deadline_s: float, group=None, poll_s: float = 50e-6) -> None:
    """Waits on the host for an asynchronous collective until `deadline_s`
    seconds have passed; then aborts the group and raises ExchangeTimeout."""
    t_end = time.monotonic() + deadline_s
    while not work.is_completed():
        if time.monotonic() > t_end:
            aborted = abort_group(group)
            raise ExchangeTimeout(
                f"the candidate all-gather did not complete within {deadline_s:g} s "
                f"(a rank did not contribute); "
                + ("communicator aborted" if aborted else "abandoned until the group timeout"),
                work)
        time.sleep(poll_s)
    work.wait()


def shard_range(n_rows: int, rank: int, world: int) -> tuple[int, int]:
    """[r0, r1) of the rows rank `rank` owns."""
    per = n_rows // world
    r0 = rank * per
    r1 = n_rows if rank == world - 1 else r0 + per
    return r0, r1


def gather_merge(scores: torch.Tensor, idx: torch.Tensor, k: int,
                 merge: Callable[[torch.Tensor, torch.Tensor, int], tuple],
                 group=None, deadline_s: float | None = None
                 ) -> tuple[torch.Tensor, torch.Tensor]:
    """All-gathers every rank's [nq, k] (scores, global indices) and merges
    them with `merge(scores [P, nq, k], idx [P, nq, k], k) -> (scores, idx)`.
    With one rank the local result is returned as is.  With `deadline_s` the
    host waits for the exchange at most that long (wait_with_deadline); without
    it the collective is queued on the stream and the process group's own
    timeout is the only bound."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1:
        return scores, idx
    # one collective: each rank's scores and indices packed as bytes, side by side
    ns = scores.numel() * scores.element_size()
    mine = torch.cat([scores.contiguous().reshape(-1).view(torch.uint8),
                      idx.contiguous().reshape(-1).view(torch.uint8)])
    g = torch.empty((world, mine.numel()), dtype=torch.uint8, device=mine.device)
    asy = deadline_s is not None
    if mine.is_cuda:
        work = dist.all_gather_into_tensor(g, mine, group=group, async_op=asy)
    else:   # gloo: list form
        work = dist.all_gather(list(g.unbind(0)), mine, group=group, async_op=asy)
    if asy:
        wait_with_deadline(work, deadline_s, group)
    gs = g[:, :ns].contiguous().view(scores.dtype).reshape((world,) + tuple(scores.shape))
    gi = g[:, ns:].contiguous().view(idx.dtype).reshape((world,) + tuple(idx.shape))
    return merge(gs, gi, k)


def sharded_ip_topk_bf16(shard: torch.Tensor, queries: torch.Tensor, k: int, row_offset: int,
                         group=None, status: torch.Tensor | None = None,
                         deadline_s: float | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Global (idx [nq, k] int64, scores [nq, k] fp32) of a row-sharded bf16
    memory: the local tensor-core top-k of this rank's shard, then the
    candidate exchange and merge.  With `status` (an int32 device word the
    caller zeroes) the local step does not wait for its stream: its timeout
    and pool-overflow flags go into `status`, which the caller checks once
    per many steps (heteromm_b200.flat.check_status)."""
    from .flat import ip_topk_bf16, shard_merge_topk
    idx, sc = ip_topk_bf16(shard, queries, k, row_offset, status=status)
    sc, idx = gather_merge(sc, idx, k, shard_merge_topk, group, deadline_s)
    return idx, sc
