"""The CUDA entry points run directly on the inputs of the committed golden
fixtures (tests/golden/*.npz, produced by the reference's own code) and are
compared with the reference's outputs stored there, with the same rules as
the oracle pins (tests/test_oracle_pins.py): bit-exact, or up to the order
inside equal-score groups where the reference's sort is unstable, or the
stated fp tolerance for the softmax."""
import os

import numpy as np
import pytest
import torch

import gen
import heteromm_b200 as hmm
import make_golden as mg
from test_oracle_pins import assert_same_up_to_ties, visible_scores

pytestmark = pytest.mark.gpu
GOLDEN = os.path.dirname(gen.__file__)


def load(name):
    return np.load(os.path.join(GOLDEN, f"{name}.npz"))


def T(a, cuda):
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def test_flat_f32_fixture(cuda):
    g = load("flat_f32")
    mem, qry = mg.flat_inputs()
    sc = hmm.ip_score_f32(T(mem, cuda), T(qry, cuda)).cpu().numpy()
    assert np.array_equal(sc.view(np.uint32), g["scores"].view(np.uint32))
    idx, _, bm = hmm.ip_topk_f32(T(mem, cuda), T(qry, cuda), int(g["k"]), float(g["threshold"]))
    assert np.array_equal(idx.cpu().numpy(), g["idx"])
    assert np.array_equal(bm.cpu().numpy().view(np.uint64), g["bitmap"])


def test_topk_edge_fixture(cuda):
    g = load("topk_edge")
    s = mg.topk_edge_inputs()
    for key, k in (("idx64", 64), ("idx_all", 4096)):
        ref = g[key][:k]
        mine = hmm.topk_f32(T(s[None], cuda), min(k, s.size))[0].cpu().numpy()[0][: ref.size]
        assert np.array_equal(s[mine], s[ref])
        kth = s[ref[-1]]
        full = s[ref] != kth
        assert set(mine[full].tolist()) == set(ref[full].tolist())
        for v in np.unique(s[mine]):
            grp = mine[s[mine] == v]
            assert np.array_equal(grp, np.sort(grp))      # lowest index inside a tie group
    bm = hmm.threshold_bitmap_f32(T(s[None], cuda), 0.0).cpu().numpy()[0]
    assert np.array_equal(bm.view(np.uint64), g["bitmap"])


def test_paged_kv_fixture(cuda):
    g = load("paged_kv")
    keys, W = mg.paged_inputs()
    for key, p, kk in (("p8", 8, keys), ("p7", 7, keys), ("p1", 1, keys[:20])):
        out = hmm.paged_kv_summary_f32(T(kk, cuda), p, T(W, cuda)).cpu().numpy()
        assert np.array_equal(out.view(np.uint32), g[key].view(np.uint32)), key


def test_block_sparse_attention_fixture(cuda):
    g = load("bsa")
    k, v, q, blocks = mg.bsa_inputs()
    out = hmm.block_sparse_attention_f32(T(q, cuda), T(k, cuda), T(v, cuda), 8,
                                         T(blocks.astype(np.int32), cuda)).cpu().numpy()
    np.testing.assert_allclose(out, g["out"], rtol=2e-5, atol=2e-6)


def test_indexer_fixtures(cuda):
    past, qq, nk = mg.idx_inputs()
    dp, dq, dn = (T(a, cuda) for a in (past, qq, nk))
    lsv = hmm.lserve_topk_i16(dp, dq, dn, 64, 16).cpu().numpy()
    bud = hmm.seer_budget_i16(dp, dq, dn, 64).cpu().numpy()
    for q in range(qq.shape[0]):
        sc = visible_scores(past, qq, nk, q)
        nb = (sc.size + 15) // 16
        blk = np.array([sc[16 * b:16 * b + 16].max() for b in range(nb)], np.float32)
        assert_same_up_to_ties(lsv[q], load("lserve")["idx"][q], lambda i: blk[i])
        assert_same_up_to_ties(bud[q], load("seer_budget")["idx"][q], lambda i: sc[i])
    words = hmm.seer_threshold_i16(dp, dq, dn, 20000).cpu().numpy()
    assert np.array_equal(words.view(np.uint64), load("seer_threshold")["words"])


def test_bm25_fixture(cuda):
    """The reference sums query terms in unordered_map order, this build in
    ascending term order: indices may differ only where fp64 scores are
    within a relative 1e-12 of each other."""
    g = load("bm25")
    tp, pd, pt, dl, qs = mg.bm25_inputs()
    idx, sc = hmm.BM25Index(tp, pd, pt, dl, cuda).topk(T(qs.astype(np.int32), cuda), 64)
    idx, sc = idx.cpu().numpy(), sc.cpu().numpy()
    from oracle import oracle as O
    _, osc = O.bm25_topk(tp, pd, pt, dl, qs, 64)
    for q in range(qs.shape[0]):
        ref = g["idx"][q]
        for i in np.nonzero(idx[q] != ref)[0]:
            assert abs(sc[q, i] - osc[q, i]) <= 1e-12 * max(1.0, abs(osc[q, i]))
            assert abs(sc[q, i] - sc[q, min(i + 1, 63)]) <= 1e-12 * abs(sc[q, i]) or \
                abs(sc[q, i] - sc[q, max(i - 1, 0)]) <= 1e-12 * abs(sc[q, i])
