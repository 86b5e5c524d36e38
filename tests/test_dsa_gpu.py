"""GPU FP8 DSA lightning indexer (hmm_dsa_indexer_fp8) against the oracle.

The oracle restates indexer_top_ref (kernels/dsa_indexer/indexer_tb.cpp:27-56)
for e4m3 inputs: exact integer dots, ReLU, fp32 w_h * x in head order, then
the top-k best first (ties to the lowest key).  The selection must equal it
bit for bit: the indices in order and the scores.

The tensor-core pass's own scores (returned by want_all_scores) are
approximations whose error the selection relies on being within
    GAMMA * sum_h |w_h| sum_d |q_hd| |k_d|  +  HEADSUM_REL * |score|
(GAMMA = 2^-10 for the tensor core's fp32 accumulation, 128x the worst case of
sequential fp32; HEADSUM_REL = 64 * 2^-23); that assumption is checked too."""
import numpy as np
import pytest
import torch

import gen
import heteromm_b200 as hmm
from heteromm_b200 import _abi
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


def dev(a, cuda):
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def check_exact(cuda, q, k, w, pos0, topk):
    idx, sc = hmm.dsa_indexer_fp8(dev(q, cuda), dev(k, cuda), dev(w, cuda), pos0, topk)
    oi, osc = O.dsa_indexer_fp8(q, k, w, pos0, topk)
    idx, sc = idx.cpu().numpy(), sc.cpu().numpy()
    bad = [t for t in range(q.shape[0]) if not np.array_equal(idx[t], oi[t])]
    assert not bad, f"tokens {bad[:8]} differ from the oracle's ranking"
    assert np.array_equal(sc.view(np.uint32), osc.view(np.uint32))
    return idx, sc


@pytest.mark.parametrize("T,H,L,pos0,topk", [
    (32, 64, 2048, 2048 - 32, 256),    # the config-4 shape, scaled down (every row fits the band)
    (37, 16, 1000, -1, 64),            # early tokens see fewer keys than k; ragged group
    (24, 32, 1500, 2000, 100),         # every key visible
    (16, 64, 20000, 20000 - 16, 256),  # long rows: the candidate band of each token
    (40, 64, 30000, 30000 - 40, 2048), # long rows, the config's top-2,048
])
def test_dsa_fp8_equals_oracle(cuda, T, H, L, pos0, topk):
    q, k, w = inputs(800 + T, T, H, L)
    check_exact(cuda, q, k, w, pos0, topk)


def test_dsa_fp8_config4_first_and_last_tokens(cuda):
    """131,072 keys, 64 heads, top-2,048, at the positions of config 4's first
    eight and last eight query tokens (token t at 126,976 + t)."""
    L, H, topk = 131072, 64, 2048
    p0 = L - 4096
    x = gen.normal_f32(901, (16, H, 128))
    y = gen.normal_f32(902, (L, 128))
    q = gen.e4m3_bits(x * (448.0 / np.abs(x).max()))
    k = gen.e4m3_bits(y * (448.0 / np.abs(y).max()))
    w = gen.uniform01_f32(903, (16, H))
    check_exact(cuda, q[:8], k, w[:8], p0, topk)
    check_exact(cuda, q[8:], k, w[8:], p0 + 4088, topk)


def test_dsa_tensor_core_scores_within_stated_bound(cuda):
    T, H, L, pos0, topk = 32, 64, 4096, 4096 - 32, 256
    q, k, w = inputs(950, T, H, L)
    _, _, full = hmm.dsa_indexer_fp8(dev(q, cuda), dev(k, cuda), dev(w, cuda), pos0, topk,
                                     want_all_scores=True)
    full = full.cpu().numpy()
    exact = O.dsa_scores_fp8(q, k, w, pos0)
    vals = e4m3_values()
    l1 = np.einsum("thd,ld->thl", np.abs(vals[q]), np.abs(vals[k]))
    tol = GAMMA * np.einsum("th,thl->tl", np.abs(w).astype(np.float64), l1) + \
        HEADSUM_REL * np.abs(exact)
    vis = np.isfinite(exact)
    assert np.array_equal(vis, np.isfinite(full))
    ratio = (np.abs(full[vis].astype(np.float64) - exact[vis]) / tol[vis]).max()
    print(f"max |tensor-core score - exact| / bound = {ratio:.3g}")
    assert ratio <= 1.0


def test_dsa_duplicate_keys_take_the_exact_row_path(cuda):
    """Keys drawn from only six distinct rows: 10,000 scores tie with each
    other, so the band of a token does not fit and every token is recomputed
    from its exact row; ties go to the lowest key index."""
    T, H, L, topk = 6, 32, 60000, 512
    q, kd, w = inputs(970, T, H, 6)
    k = kd[np.arange(L) % 6]
    check_exact(cuda, q, k, w, L - T, topk)


def test_dsa_biased_sample_takes_the_exact_row_path(cuda):
    """Only the sampled keys (j = floor(i L / 4096)) carry the strong component
    that every query shares: the threshold taken from the sample then sits near
    the sample's top, fewer than k keys of the row reach it, the check on the
    rescored candidates fails and every token is recomputed from its exact row
    (two more launches), still equal to the oracle."""
    from heteromm_b200 import _abi
    T, H, L, topk = 8, 64, 20000, 256
    x = gen.normal_f32(1901, (T, H, 128)) * 60.0
    x[..., 0] = 448.0
    y = gen.normal_f32(1902, (L, 128)) * 60.0
    y[:, 0] = 0.0
    y[(np.arange(4096) * L) // 4096, 0] = 448.0
    q, k = gen.e4m3_bits(x), gen.e4m3_bits(y)
    w = gen.uniform01_f32(1903, (T, H))
    check_exact(cuda, q, k, w, L - T, topk)        # warm: one-time kernel attributes
    l0 = _abi.kernel_launches()
    check_exact(cuda, q, k, w, L - T, topk)
    assert _abi.kernel_launches() - l0 == 12       # 10 + the exact rows and their top-k


def test_dsa_identical_keys(cuda):
    T, H, L, topk = 5, 64, 9000, 64
    q, kd, w = inputs(980, T, H, 1)
    k = np.repeat(kd, L, axis=0)
    idx, _ = check_exact(cuda, q, k, w, L - T, topk)
    assert (idx == np.arange(topk)).all()


def test_dsa_rejects_nan_encoding(cuda):
    q, k, w = inputs(990, 8, 64, 3000)
    k[17, 5] = 0x7f
    with pytest.raises(hmm.HmmError) as e:
        hmm.dsa_indexer_fp8(dev(q, cuda), dev(k, cuda), dev(w, cuda), 3000 - 8, 64)
    assert e.value.status == _abi.HMM_ERR_INVALID


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
