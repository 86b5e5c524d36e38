"""The multi-rank exchange of the sharded flat retrieval (heteromm_b200.shard)
on gloo CPU ranks (world sizes 2, 4 and 8): each rank takes its row range, computes its
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


@pytest.mark.parametrize("world,n,nq,k", [(2, 20011, 8, 50), (2, 300, 3, 100), (4, 9001, 5, 64),
                                         (8, 16007, 4, 100)])
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


def _deadline_main(rank, world, port, out_dir, withheld, deadline):
    import datetime
    import glob
    import json
    import time
    sys.path.insert(0, ROOT)
    from heteromm_b200 import shard
    from heteromm_b200._abi import HMM_ERR_TIMEOUT
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        nq, k = 3, 5
        sc = torch.arange(nq * k, dtype=torch.float32).reshape(nq, k).flip(1) + 100 * rank
        ix = torch.arange(nq * k, dtype=torch.int64).reshape(nq, k) + 1000 * rank

        def merge(gs, gi, kk):   # host merge: (score desc, index asc), as hmm_shard_merge_topk
            s = gs.permute(1, 0, 2).reshape(nq, -1)
            i = gi.permute(1, 0, 2).reshape(nq, -1)
            out_s, out_i = [], []
            for r in range(nq):
                order = sorted(range(s.shape[1]), key=lambda c: (-float(s[r, c]), int(i[r, c])))[:kk]
                out_s.append(s[r, order])
                out_i.append(i[r, order])
            return torch.stack(out_s), torch.stack(out_i)

        rec = {"rank": rank}
        if rank == withheld:
            # withhold the contribution until every other rank has given up on
            # it, then contribute late so that their abandoned collective ends
            t0 = time.monotonic()
            while (len(glob.glob(os.path.join(out_dir, "gave_up*"))) < world - 1 and
                   time.monotonic() - t0 < 30):
                time.sleep(0.01)
            rec["others_gave_up"] = len(glob.glob(os.path.join(out_dir, "gave_up*")))
            shard.gather_merge(sc, ix, k, merge)
        else:
            t0 = time.monotonic()
            try:
                s, i = shard.gather_merge(sc, ix, k, merge, deadline_s=deadline)
                rec["result"] = [s.tolist(), i.tolist()]
            except shard.ExchangeTimeout as e:
                rec["timeout_s"] = time.monotonic() - t0
                rec["status_ok"] = e.status == HMM_ERR_TIMEOUT
                open(os.path.join(out_dir, f"gave_up{rank}"), "w").close()
                e.work.wait()   # the late contribution completes the abandoned collective
                rec["drained"] = True
        with open(os.path.join(out_dir, f"rec{rank}.json"), "w") as f:
            json.dump(rec, f)
    finally:
        dist.destroy_process_group()


def _free_port():
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,withheld", [(2, 1), (3, 0)])
def test_withheld_rank_times_out_instead_of_hanging(tmp_path, world, withheld):
    """One rank withholds its contribution to the candidate all-gather; every
    other rank's exchange gives up at its host deadline with HMM_ERR_TIMEOUT
    (the reference would exit the process) instead of waiting for the group's
    60 s timeout.  The withheld rank then contributes late, so every rank
    leaves the group cleanly."""
    import json
    deadline = 1.0
    mp.spawn(_deadline_main, args=(world, _free_port(), str(tmp_path), withheld, deadline),
             nprocs=world, join=True)
    for r in range(world):
        rec = json.loads((tmp_path / f"rec{r}.json").read_text())
        if r == withheld:
            assert rec["others_gave_up"] == world - 1
        else:
            assert rec["status_ok"] and rec["drained"]
            assert deadline <= rec["timeout_s"] < deadline + 5.0


def test_deadline_exchange_equals_plain_exchange(tmp_path):
    """With every rank present, the deadline-bounded exchange returns the same
    merged candidates as the plain one."""
    import json
    mp.spawn(_deadline_main, args=(2, _free_port(), str(tmp_path), -1, 30.0), nprocs=2,
             join=True)
    recs = [json.loads((tmp_path / f"rec{r}.json").read_text()) for r in range(2)]
    assert recs[0]["result"] == recs[1]["result"]
    s, i = recs[0]["result"]
    # rank 1's scores (100 + ...) all beat rank 0's; each row is best first
    assert all(v >= 100 for row in s for v in row)
    assert all(row == sorted(row, reverse=True) for row in s)
