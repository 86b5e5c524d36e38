"""GPU FP8 DSA lightning indexer (hmm_dsa_indexer_fp8) against the oracle's
exact scores.

The tensor core multiplies e4m3 values exactly but accumulates the 128
products of a head in fp32 with an undocumented order and width, and the
head sum is fp32 FMA.  The stated tolerance per score is
    GAMMA * sum_h w_h * sum_d |q_hd| |k_d|  +  HEADSUM_REL * |score|
with GAMMA = 2^-10 (128x the worst fp32 sequential rounding of 128 terms)
and HEADSUM_REL = 64 * 2^-23.  Selections must equal the exact top-k except
among keys whose exact scores lie within twice the tolerance of the k-th."""
import numpy as np
import pytest
import torch

import gen
import heteromm_b200 as hmm
from oracle import oracle as O

pytestmark = pytest.mark.gpu

GAMMA = 2.0 ** -10
HEADSUM_REL = 64 * 2.0 ** -23


def e4m3_values():
    v = np.zeros(256)
    for c in range(256):
        e, m = (c >> 3) & 15, c & 7
        mag = 0.0 if (e == 15 and m == 7) else (m * 2.0 ** -9 if e == 0 else (1 + m / 8) * 2.0 ** (e - 7))
        v[c] = -mag if c & 0x80 else mag
    return v


def inputs(seed, T, H, L):
    x = gen.normal_f32(seed, (T, H, 128))
    y = gen.normal_f32(seed + 1, (L, 128))
    q = gen.e4m3_bits(x * (448.0 / np.abs(x).max()))
    k = gen.e4m3_bits(y * (448.0 / np.abs(y).max()))
    w = gen.uniform01_f32(seed + 2, (T, H))
    return q, k, w


@pytest.mark.parametrize("T,H,L,pos0,topk", [
    (32, 64, 2048, 2048 - 32, 256),    # the config-4 shape, scaled down
    (37, 16, 1000, -1, 64),            # early tokens see fewer keys than k; ragged group
    (24, 32, 1500, 2000, 100),         # every key visible
    (16, 64, 8192, 8192 - 16, 256),    # long rows: the sampled per-row selection
])
def test_dsa_fp8_matches_exact_within_tolerance(cuda, T, H, L, pos0, topk):
    q, k, w = inputs(800 + T, T, H, L)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)   # noqa: E731
    idx, sc, full = hmm.dsa_indexer_fp8(dev(q), dev(k), dev(w), pos0, topk, want_all_scores=True)
    idx, sc, full = idx.cpu().numpy(), sc.cpu().numpy(), full.cpu().numpy()
    exact = O.dsa_scores_fp8(q, k, w, pos0)

    vals = e4m3_values()
    qa, ka = np.abs(vals[q]), np.abs(vals[k])
    l1 = np.einsum("thd,ld->thl", qa, ka)                     # sum_d |q||k| per head
    tol = GAMMA * np.einsum("th,thl->tl", w.astype(np.float64), l1) + HEADSUM_REL * np.abs(exact)
    vis = np.isfinite(exact)
    assert np.array_equal(vis, np.isfinite(full))
    err = np.abs(full[vis].astype(np.float64) - exact[vis])
    ratio = (err / tol[vis]).max()
    print(f"max |gpu - exact| / tolerance = {ratio:.3g}")
    assert ratio <= 1.0

    for t in range(T):
        n_vis = int(vis[t].sum())
        m = min(topk, n_vis)
        assert (idx[t, m:] == -1).all() and (idx[t, :m] >= 0).all()
        got = idx[t, :m]
        assert np.array_equal(sc[t, :m], full[t, got])             # reported = computed scores
        assert (np.diff(sc[t, :m]) <= 0).all()                     # best first
        assert (got <= pos0 + t).all()                              # causal
        # the selection is exact over the kernel's own scores
        own = np.lexsort((np.arange(L), -full[t].astype(np.float64)))[:m]
        assert np.array_equal(got, own)
        if m == 0:
            continue
        order = np.lexsort((np.arange(L), -exact[t]))               # exact ranking, ties lowest
        want = order[:m]
        kth = exact[t, want[-1]]
        slack = 2 * tol[t, vis[t]].max()
        extra = np.setdiff1d(got, want)
        missing = np.setdiff1d(want, got)
        assert len(extra) == len(missing)
        assert (exact[t, extra] >= kth - slack).all()
        assert (exact[t, missing] <= kth + slack).all()


@pytest.mark.parametrize("T,chunks", [(700, 1), (700, 3), (700, None), (1500, None)])
def test_dsa_host_pipeline_equals_device_call(cuda, T, chunks):
    """dsa_indexer_fp8_host (host inputs and outputs, the token slices'
    transfers overlapped with the indexer) returns what dsa_indexer_fp8 returns
    on the same inputs, bit for bit: equal slices with a ragged last one, and
    the wave-sized slices (two at 700 tokens, three at 1,500 on 148 SMs)."""
    H, L, topk = 64, 4096, 256
    pos0 = L - T
    q, k, w = inputs(1700 + T + (chunks or 0), T, H, L)
    qd = torch.from_numpy(np.ascontiguousarray(q)).to(cuda)
    kd = torch.from_numpy(np.ascontiguousarray(k)).to(cuda)
    wd = torch.from_numpy(np.ascontiguousarray(w)).to(cuda)
    ref_i, ref_s = hmm.dsa_indexer_fp8(qd, kd, wd, pos0, topk)
    qh = torch.from_numpy(np.ascontiguousarray(q)).pin_memory()
    wh = torch.from_numpy(np.ascontiguousarray(w)).pin_memory()
    for _ in range(2):   # twice: the copy streams are reused
        i, s = hmm.dsa_indexer_fp8_host(qh, kd, wh, pos0, topk, chunks=chunks)
        assert not i.is_cuda and i.is_pinned()
        assert torch.equal(i, ref_i.cpu())
        assert torch.equal(s.view(torch.int32), ref_s.cpu().view(torch.int32))
