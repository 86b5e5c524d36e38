"""GPU parity of the tensor-core (tcgen05) bf16 scoring path with exact
top-k selection (hmm_ip_topk_bf16 for dim 128, k <= 128, n > 8192 rows)
against the oracle: bit-exact indices and scores."""
import numpy as np
import pytest
import torch

import gen
import heteromm_b200 as hmm
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def dev(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def run(cuda, mem, qry, k, off=0):
    idx, sc = hmm.ip_topk_bf16(dev(mem.view(np.int16), cuda), dev(qry.view(np.int16), cuda), k, off)
    torch.cuda.synchronize()
    return idx.cpu().numpy(), sc.cpu().numpy()


@pytest.mark.parametrize("n,nq,k,seed", [
    (20000, 16, 100, 1),      # a few tiles per SM
    (12345, 1, 64, 2),        # one query (255 padded query rows), ragged last tile
    (9000, 300, 32, 3),       # two query passes (256 + 44)
    (300000, 256, 100, 4),    # every SM busy for many tiles
])
def test_tc_matches_oracle(cuda, n, nq, k, seed):
    mem = gen.bf16_bits(gen.normal_f32(seed * 7, (n, 128)))
    qry = gen.bf16_bits(gen.normal_f32(seed * 7 + 1, (nq, 128)))
    idx, sc = run(cuda, mem, qry, k, 1000)
    oidx, osc = O.ip_topk_bf16(mem, qry, k, 1000)
    assert np.array_equal(idx, oidx)
    assert np.array_equal(sc.view(np.uint32), osc.view(np.uint32))


def test_tc_duplicate_rows_and_ties(cuda):
    """Many identical rows: every copy ties, only the lowest indices may win."""
    n, nq, k = 30000, 8, 100
    base = gen.bf16_bits(gen.normal_f32(51, (500, 128)))
    mem = base[np.arange(n) % 500]
    qry = gen.bf16_bits(gen.normal_f32(52, (nq, 128)))
    idx, sc = run(cuda, mem, qry, k)
    oidx, osc = O.ip_topk_bf16(mem, qry, k)
    assert np.array_equal(idx, oidx)
    assert np.array_equal(sc.view(np.uint32), osc.view(np.uint32))


def test_tc_large_magnitudes_and_zero_rows(cuda):
    n, nq, k = 20000, 4, 50
    x = gen.normal_f32(61, (n, 128))
    x[::3] *= 1e4
    x[5::7] = 0.0
    mem = gen.bf16_bits(x)
    qry = gen.bf16_bits(gen.normal_f32(62, (nq, 128)) * 100)
    idx, sc = run(cuda, mem, qry, k)
    oidx, osc = O.ip_topk_bf16(mem, qry, k)
    assert np.array_equal(idx, oidx)
    assert np.array_equal(sc.view(np.uint32), osc.view(np.uint32))


def _nonfinite_rows(n):
    """N(0,1) rows with a few +-inf rows, rows whose products overflow fp32,
    NaN rows and +-0 rows."""
    x = gen.normal_f32(101, (n, 128))
    i = np.arange(n)
    x[i % 997 == 3, 7] = np.nan
    x[i % 20011 == 5, 11] = np.inf
    x[i % 20021 == 6, 13] = -np.inf
    x[i % 7919 == 7] *= np.float32(1e37)     # |products| past 3.4e38
    x[i % 1031 == 9] = 0.0
    x[i % 1033 == 10] = -0.0
    return gen.bf16_bits(x)


def test_tc_nonfinite_and_overflowing_rows(cuda):
    """NaN rows (rank last), +-inf rows, rows whose bf16 x bf16 products
    overflow fp32 (the reference rounds each product before adding it, so
    inf - huge stays inf where a fused multiply-add would not) and +-0 rows,
    on a shard larger than the sample pass covers, so that both passes meet
    them; each query's top-100 holds infinite and finite scores."""
    n, nq, k = 200_000, 16, 100
    mem = _nonfinite_rows(n)
    qry = gen.bf16_bits(gen.normal_f32(102, (nq, 128)) * np.float32(4.0))
    idx, sc = run(cuda, mem, qry, k)
    oidx, osc = O.ip_topk_bf16(mem, qry, k)
    assert np.isinf(osc).any() and np.isfinite(osc).all(axis=1).sum() < nq
    assert np.isfinite(osc[:, -1]).all()
    assert np.array_equal(idx, oidx)
    assert np.array_equal(sc.view(np.uint32), osc.view(np.uint32))


def test_product_overflow_against_a_large_partial_sum(cuda):
    """Rows whose second product overflows fp32 while the partial sum before it
    is large and of the other sign: -3e38 + (3e38 * 2).  The reference rounds
    the product to +inf before adding it, so the score is +inf; a fused
    multiply-add would keep it finite (3e38).  The tensor-core path (60,000
    rows) and the CUDA-core path (8,192 rows) must both give the oracle's bits."""
    k = 50
    for n in (60_000, 8192):
        x = gen.normal_f32(105, (n, 128))
        rows = np.arange(16) * (n // 16) + 7
        x[rows, 0] = -3.0e38
        x[rows, 1] = 3.0e38
        mem = gen.bf16_bits(x)
        q = gen.normal_f32(106, (4, 128))
        q[0, 0], q[0, 1] = 1.0, 2.0
        qry = gen.bf16_bits(q)
        idx, sc = run(cuda, mem, qry, k)
        oidx, osc = O.ip_topk_bf16(mem, qry, k)
        assert np.isposinf(osc[0, :16]).all() and np.array_equal(oidx[0, :16], rows)
        assert np.array_equal(idx, oidx)
        assert np.array_equal(sc.view(np.uint32), osc.view(np.uint32))


def test_tc_sharded_merge(cuda):
    n, nq, k, shards = 80000, 32, 100, 4
    mem = gen.bf16_bits(gen.normal_f32(71, (n, 128)))
    qry = gen.bf16_bits(gen.normal_f32(72, (nq, 128)))
    per = n // shards
    cs, ci = [], []
    for s in range(shards):
        i, v = hmm.ip_topk_bf16(dev(mem[s * per:(s + 1) * per].view(np.int16), cuda),
                                dev(qry.view(np.int16), cuda), k, s * per)
        cs.append(v); ci.append(i)
    ms, mi = hmm.shard_merge_topk(torch.stack(cs), torch.stack(ci), k)
    oidx, osc = O.ip_topk_bf16(mem, qry, k)
    assert np.array_equal(mi.cpu().numpy(), oidx)
    assert np.array_equal(ms.cpu().numpy().view(np.uint32), osc.view(np.uint32))


def test_tc_pool_overflow_falls_back_to_exact(cuda):
    """Rows ordered so that query 0's score is the row index: every row beats
    the running top-k.  The sample pass that sets the starting threshold sees
    tiles spread over the shard, the last of them about n / (its tile count)
    rows before the end; all the rows after it enter query 0's candidate pool,
    which fills up (more than 8,192 of them at 6,000,000 rows).  The call must
    notice the dropped candidates and recompute the pass exactly (more kernel
    launches than the tensor-core path's four)."""
    from heteromm_b200 import _abi
    n, nq, k = 6_000_000, 4, 100
    x = np.random.default_rng(81).standard_normal((n, 128), dtype=np.float32)
    i = np.arange(n)
    # bf16-exact parts of the row index: 65536 * a + 256 * b + c, each < 256
    x[:, 0] = (65536 * (i // 65536)).astype(np.float32)
    x[:, 1] = (256 * ((i // 256) % 256)).astype(np.float32)
    x[:, 2] = (i % 256).astype(np.float32)
    mem = gen.bf16_bits(x)
    del x
    q = gen.normal_f32(82, (nq, 128))
    q[0] = 0.0
    q[0, :3] = 1.0                    # score of row i for query 0 is exactly i
    qry = gen.bf16_bits(q)
    l0 = _abi.kernel_launches()
    idx, sc = run(cuda, mem, qry, k)
    launches = _abi.kernel_launches() - l0
    oidx, osc = O.ip_topk_bf16(mem, qry, k)
    assert np.array_equal(idx[0], np.arange(n - 1, n - 1 - k, -1))
    assert np.array_equal(idx, oidx)
    assert np.array_equal(sc.view(np.uint32), osc.view(np.uint32))
    assert launches > 4, launches


def test_tc_normal_call_launch_count(cuda):
    """Sample pass, starting thresholds, scoring pass, pool merge."""
    from heteromm_b200 import _abi
    mem = gen.bf16_bits(gen.normal_f32(91, (20000, 128)))
    qry = gen.bf16_bits(gen.normal_f32(92, (8, 128)))
    run(cuda, mem, qry, 10)
    l0 = _abi.kernel_launches()
    run(cuda, mem, qry, 10)
    assert _abi.kernel_launches() - l0 == 4


def test_tc_two_pass_shard(cuda):
    """A 4Mi-row shard with a ragged last tile and a global row offset: the
    sample pass over tiles spread across the shard (its last tile ragged too),
    then one scoring pass over every row."""
    n, nq, k = (1 << 22) + 12345, 8, 100
    mem = gen.bf16_bits(gen.normal_f32(95, (n, 128)))
    qry = gen.bf16_bits(gen.normal_f32(96, (nq, 128)))
    idx, sc = run(cuda, mem, qry, k, 777)
    oidx, osc = O.ip_topk_bf16(mem, qry, k, 777)
    assert np.array_equal(idx, oidx)
    assert np.array_equal(sc.view(np.uint32), osc.view(np.uint32))
