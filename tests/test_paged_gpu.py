"""GPU parity of the paged-KV path (block summaries, block -> page expansion,
block-sparse decode attention and the fused decode step) against the oracle.

Bit-exact: summaries, selected blocks, page lists.  Attention outputs are
compared with the fp32 tolerance the entry point states (ATOL / RTOL below):
the device expf and the summation order differ from glibc and from the
reference's sequential order."""
import numpy as np
import pytest
import torch

import gen
import heteromm_b200 as hmm
from heteromm_b200._abi import HMM_ERR_BOUNDS, HmmError
from oracle import oracle as O

pytestmark = pytest.mark.gpu

RTOL = 2e-5
ATOL = 2e-6


def T(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def make_cache(seed, n_seq, L, D, pt, spare=3):
    """Logical K/V [n_seq, L, D] bf16 bits scattered over physical pages in a
    seeded random order (plus `spare` unused pages)."""
    pps = (L + pt - 1) // pt
    keys = gen.bf16_bits(gen.normal_f32(seed, (n_seq, L, D)))
    vals = gen.bf16_bits(gen.normal_f32(seed + 1, (n_seq, L, D)))
    n_pages = n_seq * pps + spare
    perm = np.argsort(gen.uniform_f64(seed + 2, n_pages), kind="stable")
    table = perm[:n_seq * pps].reshape(n_seq, pps).astype(np.int32)
    pad = np.zeros((n_seq, pps * pt - L, D), np.uint16)
    kp = np.zeros((n_pages, pt, D), np.uint16)
    vp = np.zeros((n_pages, pt, D), np.uint16)
    kp[table.reshape(-1)] = np.concatenate([keys, pad], axis=1).reshape(n_seq * pps, pt, D)
    vp[table.reshape(-1)] = np.concatenate([vals, pad], axis=1).reshape(n_seq * pps, pt, D)
    return keys, vals, kp, vp, table


def dev_cache(cuda, kp, vp, table):
    return (T(kp.view(np.int16), cuda), T(vp.view(np.int16), cuda), T(table, cuda))


@pytest.mark.parametrize("page", [8, 7, 1, 500])
def test_summary_f32_reference_form(cuda, page):
    keys = gen.normal_f32(301, (3, 333, 64))
    W = gen.normal_f32(302, (48, 64))
    out = hmm.paged_kv_summary_f32(T(keys, cuda), page, T(W, cuda)).cpu().numpy()
    plain = hmm.paged_kv_summary_f32(T(keys, cuda), page).cpu().numpy()
    for s in range(3):
        ref = O.paged_kv_summary_f32(keys[s], W, page)
        assert np.array_equal(out[s].view(np.uint32), ref.view(np.uint32))
        assert np.array_equal(plain[s].view(np.uint32),
                              O.block_mean_f32(keys[s], page).view(np.uint32))


def test_summary_f32_empty(cuda):
    keys = torch.empty((2, 0, 16), dtype=torch.float32, device=cuda)
    assert hmm.paged_kv_summary_f32(keys, 4).shape == (2, 0, 16)


@pytest.mark.parametrize("L,D,pt,bt", [(1000, 64, 16, 64), (777, 128, 16, 40),
                                       (300, 8, 5, 5), (64, 512, 16, 64)])
def test_paged_summary_bf16(cuda, L, D, pt, bt):
    keys, _, kp, vp, table = make_cache(310 + D, 3, L, D, pt)
    k, _, tb = dev_cache(cuda, kp, vp, table)
    out = hmm.paged_kv_summary_bf16(k, tb, L, bt).cpu().numpy()
    for s in range(3):
        ref = O.block_mean_f32(gen.bf16_to_f32(keys[s]), bt)
        assert np.array_equal(out[s].view(np.uint32), ref.view(np.uint32))


def test_block_pages(cuda):
    n_seq, pps, ppb = 5, 40, 4
    table = gen.ints(320, (n_seq, pps), 0, 100000).astype(np.int32)
    # in range, past the end (clipped / empty), partially past the end, negative
    blocks = gen.ints(321, (n_seq, 12), -2, 12).astype(np.int32)
    pages, counts = hmm.block_pages(T(table, cuda), T(blocks, cuda), ppb)
    pages, counts = pages.cpu().numpy(), counts.cpu().numpy()
    for s in range(n_seq):
        ref = O.block_pages(table, s, blocks[s], ppb)
        assert counts[s] == ref.size
        assert np.array_equal(pages[s, :ref.size], ref)
        assert (pages[s, ref.size:] == -1).all()


@pytest.mark.parametrize("L,D,pt,bt,nsel", [(1000, 64, 16, 64, 6), (4096, 128, 16, 64, 64),
                                            (2000, 256, 16, 32, 10), (333, 32, 7, 21, 3),
                                            (1000, 128, 8, 64, 5)])
def test_block_sparse_attention(cuda, L, D, pt, bt, nsel):
    n_seq = 4
    keys, vals, kp, vp, table = make_cache(330 + L, n_seq, L, D, pt)
    nb = (L + bt - 1) // bt
    blocks = np.stack([np.argsort(gen.uniform_f64(331 + s, nb))[:nsel]
                       for s in range(n_seq)]).astype(np.int32)
    blocks[0, 0] = nb - 1                  # the partial last block
    blocks[1, -1] = nb + 5                 # past the end: contributes no tokens
    q = gen.bf16_bits(gen.normal_f32(332, (n_seq, D)))
    k, v, tb = dev_cache(cuda, kp, vp, table)
    out = hmm.block_sparse_attention_bf16(T(q.view(np.int16), cuda), k, v, tb, L, bt,
                                          T(blocks, cuda)).cpu().numpy()
    for s in range(n_seq):
        ref = O.block_sparse_attention_f32(gen.bf16_to_f32(keys[s]), gen.bf16_to_f32(vals[s]),
                                           blocks[s], gen.bf16_to_f32(q[s]), bt)
        np.testing.assert_allclose(out[s], ref, rtol=RTOL, atol=ATOL)


def test_block_sparse_attention_empty_selection(cuda):
    keys, vals, kp, vp, table = make_cache(340, 2, 100, 16, 4)
    k, v, tb = dev_cache(cuda, kp, vp, table)
    q = T(gen.bf16_bits(gen.normal_f32(341, (2, 16))).view(np.int16), cuda)
    none = torch.empty((2, 0), dtype=torch.int32, device=cuda)
    assert (hmm.block_sparse_attention_bf16(q, k, v, tb, 100, 8, none) == 0).all()
    past = torch.full((2, 3), 50, dtype=torch.int32, device=cuda)   # all past the end
    assert (hmm.block_sparse_attention_bf16(q, k, v, tb, 100, 8, past) == 0).all()


def decode_oracle(keys, vals, q, bt, top):
    kf, vf, qf = gen.bf16_to_f32(keys), gen.bf16_to_f32(vals), gen.bf16_to_f32(q)
    summ = O.block_mean_f32(kf, bt)
    sc = O.ip_score_f32(summ, qf[None])[0]
    blocks = O.topk_f32(sc, min(top, summ.shape[0]))
    return blocks, O.block_sparse_attention_f32(kf, vf, blocks, qf, bt)


@pytest.mark.parametrize("n_seq,L,D,pt,bt,top", [(6, 2000, 64, 16, 64, 8),
                                                 (4, 32768, 128, 16, 64, 64),
                                                 (3, 130, 16, 16, 64, 5)])
def test_decode_step(cuda, n_seq, L, D, pt, bt, top):
    keys, vals, kp, vp, table = make_cache(350 + n_seq, n_seq, L, D, pt)
    q = gen.bf16_bits(gen.normal_f32(351, (n_seq, D)))
    k, v, tb = dev_cache(cuda, kp, vp, table)
    summ = hmm.paged_kv_summary_bf16(k, tb, L, bt)
    blocks, out = hmm.block_sparse_decode_bf16(T(q.view(np.int16), cuda), summ, k, v, tb, L, bt,
                                               top)
    blocks, out = blocks.cpu().numpy(), out.cpu().numpy()
    nb = (L + bt - 1) // bt
    for s in range(n_seq):
        rb, ro = decode_oracle(keys[s], vals[s], q[s], bt, top)
        m = min(top, nb)
        assert np.array_equal(blocks[s, :m], rb)
        assert (blocks[s, m:] == -1).all()
        np.testing.assert_allclose(out[s], ro, rtol=RTOL, atol=ATOL)


def test_bounds_are_reported(cuda):
    keys, vals, kp, vp, table = make_cache(360, 2, 64, 16, 16)
    table[1, 2] = kp.shape[0] + 7          # names a page that does not exist
    k, v, tb = dev_cache(cuda, kp, vp, table)
    with pytest.raises(HmmError) as e:
        hmm.paged_kv_summary_bf16(k, tb, 64, 16)
    assert e.value.status == HMM_ERR_BOUNDS
    q = T(gen.bf16_bits(gen.normal_f32(361, (2, 16))).view(np.int16), cuda)
    with pytest.raises(HmmError) as e:
        hmm.block_sparse_attention_bf16(q, k, v, tb, 64, 16,
                                        torch.tensor([[0, 2], [1, 2]], dtype=torch.int32,
                                                     device=cuda))
    assert e.value.status == HMM_ERR_BOUNDS
    ok_tb = T(make_cache(360, 2, 64, 16, 16)[4], cuda)
    with pytest.raises(HmmError) as e:
        hmm.block_sparse_attention_bf16(q, k, v, ok_tb, 64, 16,
                                        torch.tensor([[0, -1], [1, 2]], dtype=torch.int32,
                                                     device=cuda))
    assert e.value.status == HMM_ERR_BOUNDS


@pytest.mark.parametrize("L,D,bt,nsel", [(333, 64, 8, 5), (1000, 128, 64, 6), (50, 4, 7, 3)])
def test_block_sparse_attention_f32_contiguous(cuda, L, D, bt, nsel):
    """The reference's own layout: contiguous fp32 K/V, fp32 query."""
    n_seq = 3
    keys = gen.normal_f32(370 + L, (n_seq, L, D))
    vals = gen.normal_f32(371 + L, (n_seq, L, D))
    q = gen.normal_f32(372 + L, (n_seq, D))
    nb = (L + bt - 1) // bt
    blocks = np.stack([np.argsort(gen.uniform_f64(373 + s, nb))[:nsel]
                       for s in range(n_seq)]).astype(np.int32)
    blocks[2, 0] = nb + 3                  # past the end
    out = hmm.block_sparse_attention_f32(T(q, cuda), T(keys, cuda), T(vals, cuda), bt,
                                         T(blocks, cuda)).cpu().numpy()
    for s in range(n_seq):
        ref = O.block_sparse_attention_f32(keys[s], vals[s], blocks[s], q[s], bt)
        np.testing.assert_allclose(out[s], ref, rtol=RTOL, atol=ATOL)


def test_decode_async_matches_sync_and_reports_bounds(cuda):
    from heteromm_b200.paged import check_status
    keys, vals, kp, vp, table = make_cache(380, 3, 1000, 64, 16)
    q = T(gen.bf16_bits(gen.normal_f32(381, (3, 64))).view(np.int16), cuda)
    k, v, tb = dev_cache(cuda, kp, vp, table)
    summ = hmm.paged_kv_summary_bf16(k, tb, 1000, 64)
    b0, o0 = hmm.block_sparse_decode_bf16(q, summ, k, v, tb, 1000, 64, 6)
    st = torch.zeros(1, dtype=torch.int32, device=cuda)
    b1, o1 = hmm.block_sparse_decode_bf16(q, summ, k, v, tb, 1000, 64, 6, status=st)
    check_status(st)
    assert torch.equal(b0, b1) and torch.equal(o0, o1)
    bad = table.copy()
    bad[1, 3] = kp.shape[0] + 5
    st.zero_()
    hmm.block_sparse_decode_bf16(q, summ, k, v, T(bad, cuda), 1000, 64, 64, status=st)
    with pytest.raises(HmmError) as e:
        check_status(st)
    assert e.value.status == HMM_ERR_BOUNDS
