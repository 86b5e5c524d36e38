"""The multi-rank exchange of the sharded flat retrieval (heteromm_b200.shard)
on gloo CPU ranks (world sizes 2 and 4): each rank takes its row range, computes its
local top-k with global indices (the oracle stands in for the GPU kernel),
all-gathers and merges (the oracle's merge); every rank must hold the
unsharded top-k."""
import os
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _rank_main(rank, world, port, n, nq, k, out_dir):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import gen
    from heteromm_b200 import shard
    from oracle import oracle as O
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rows = gen.bf16_bits(gen.normal_f32(1201, (n, 128)))
        qry = gen.bf16_bits(gen.normal_f32(1202, (nq, 128)))
        r0, r1 = shard.shard_range(n, rank, world)
        li, ls = O.ip_topk_bf16(rows[r0:r1], qry, k, r0)

        def merge(gs, gi, kk):
            s, i = O.shard_merge_topk(gs.numpy(), gi.numpy(), kk)
            return torch.from_numpy(s), torch.from_numpy(i)

        sc, idx = shard.gather_merge(torch.from_numpy(ls), torch.from_numpy(li), k, merge)
        np.save(os.path.join(out_dir, f"idx{rank}.npy"), idx.numpy())
        np.save(os.path.join(out_dir, f"sc{rank}.npy"), sc.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n,nq,k", [(2, 20011, 8, 50), (2, 300, 3, 100), (4, 9001, 5, 64)])
def test_sharded_topk_equals_unsharded(tmp_path, world, n, nq, k):
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import gen
    from oracle import oracle as O
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_rank_main, args=(world, port, n, nq, k, str(tmp_path)), nprocs=world, join=True)
    rows = gen.bf16_bits(gen.normal_f32(1201, (n, 128)))
    qry = gen.bf16_bits(gen.normal_f32(1202, (nq, 128)))
    oi, os_ = O.ip_topk_bf16(rows, qry, k)
    for r in range(world):
        assert np.array_equal(np.load(tmp_path / f"idx{r}.npy"), oi)
        assert np.array_equal(np.load(tmp_path / f"sc{r}.npy").view(np.uint32), os_.view(np.uint32))


def test_shard_ranges_cover_rows_once():
    from heteromm_b200 import shard
    for n, w in ((10, 3), (64 << 20, 8), (7, 7), (100, 1)):
        rs = [shard.shard_range(n, r, w) for r in range(w)]
        assert rs[0][0] == 0 and rs[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(rs, rs[1:]))
