"""The min/max page summaries (the reference's MinMaxIndexMemory layout) and
the min/max-bound block selector of the oracle: summaries equal NumPy's
min / max per block, and the bound is an upper bound of q.k for every key of
its block (checked in float64, where the fp32 products are exact)."""
import numpy as np

from oracle import oracle as O


def test_minmax_summaries_and_bound():
    rng = np.random.default_rng(7)
    for L, D, page in [(300, 16, 64), (64, 8, 64), (65, 32, 7), (1, 4, 3)]:
        keys = rng.standard_normal((L, D)).astype(np.float32)
        mm = O.block_minmax_f32(keys, page)
        nb = (L + page - 1) // page
        assert mm.shape == (nb, 2, D)
        for b in range(nb):
            blk = keys[b * page:(b + 1) * page]
            assert np.array_equal(mm[b, 0], blk.min(0)) and np.array_equal(mm[b, 1], blk.max(0))
        for _ in range(5):
            q = rng.standard_normal(D).astype(np.float32)
            q64, mm64 = q.astype(np.float64), mm.astype(np.float64)
            u = np.maximum(q64 * mm64[:, 0], q64 * mm64[:, 1]).sum(1)
            for b in range(nb):
                dots = keys[b * page:(b + 1) * page].astype(np.float64) @ q64
                assert u[b] >= dots.max() - 1e-12 * max(1.0, abs(u[b]))
            sel = O.block_select_minmax(q, mm, nb + 2)
            assert sel[-2:].tolist() == [-1, -1]
            assert sorted(sel[:nb].tolist()) == list(range(nb))
