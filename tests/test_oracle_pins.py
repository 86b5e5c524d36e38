"""Pins the CPU oracle (oracle/hmm_oracle.c) to the reference.

1. Golden fixtures (tests/golden/*.npz) produced by the reference's own code,
   compiled from its sources (tests/golden/make_golden.py).
2. When the reference's compiled code is present (oracle/_ref, built in the
   container that has the reference checkout), live comparisons on further
   seeds and the reference's own doctest binaries.
"""
import os
import subprocess

import numpy as np
import pytest

import gen
import make_golden as mg
from oracle import oracle as O

GOLDEN = os.path.dirname(gen.__file__)


def load(name):
    return np.load(os.path.join(GOLDEN, f"{name}.npz"))


def test_flat_f32_golden():
    g = load("flat_f32")
    mem, qry = mg.flat_inputs()
    assert mg.digest(mem, qry) == str(g["digest"])
    idx, bm, sc = O.ip_topk_f32(mem, qry, int(g["k"]), float(g["threshold"]), want_scores=True)
    assert np.array_equal(sc.view(np.uint32), g["scores"].view(np.uint32))
    assert np.array_equal(idx, g["idx"])
    assert np.array_equal(bm, g["bitmap"])


def test_topk_edge_golden():
    """Ties, -0.0/+0.0 and k > n.  The reference's partial_sort leaves the order
    inside a group of equal scores unspecified; the oracle breaks ties by the
    lowest index.  Score sequences must agree exactly, and so must the index
    sets of every fully-included tie group."""
    g = load("topk_edge")
    s = mg.topk_edge_inputs()
    assert mg.digest(s) == str(g["digest"])
    for key, k in (("idx64", 64), ("idx_all", 6000)):
        ref = g[key]
        mine = O.topk_f32(s, k)[: ref.size]
        assert np.array_equal(s[mine], s[ref])
        kth = s[ref[-1]]
        full = s[ref] != kth if ref.size < s.size else np.ones(ref.size, bool)
        assert set(mine[full].tolist()) == set(ref[full].tolist())
        # lowest-index rule inside each tie group
        for v in np.unique(s[mine]):
            grp = mine[s[mine] == v]
            assert np.array_equal(grp, np.sort(grp))
    assert np.array_equal(O.threshold_bitmap_f32(s, 0.0), g["bitmap"])


def test_paged_kv_golden():
    g = load("paged_kv")
    keys, W = mg.paged_inputs()
    assert mg.digest(keys, W) == str(g["digest"])
    for key, p, kk in (("p8", 8, keys), ("p7", 7, keys), ("p1", 1, keys[:20])):
        out = O.paged_kv_summary_f32(kk, W, p)
        assert np.array_equal(out.view(np.uint32), g[key].view(np.uint32)), key


def test_block_sparse_attention_golden():
    g = load("bsa")
    k, v, q, blocks = mg.bsa_inputs()
    assert mg.digest(k, v, q, blocks) == str(g["digest"])
    out = O.block_sparse_attention_f32(k, v, blocks, q, 8)
    assert np.array_equal(out.view(np.uint32), g["out"].view(np.uint32))


def test_dsa_i16_golden():
    g = load("dsa_i16")
    q, k, w = mg.dsa_inputs()
    assert mg.digest(q, k, w) == str(g["digest"])
    idx, _ = O.dsa_indexer_i16(q, k, w, 2048)
    assert np.array_equal(idx, g["idx"])


def visible_scores(past, qq, nk, q):
    """(float)(int64 dot) of query q against every key it sees (positions
    0..L+q/8; position L+g holds new key min(8g+7, q))."""
    L = past.shape[0]
    cur = L + q // 8
    keys = [past[p] if p < L else nk[min(8 * (p - L) + 7, q)] for p in range(cur + 1)]
    return (np.stack(keys).astype(np.int64) @ qq[q].astype(np.int64)).astype(np.float32)


def assert_same_up_to_ties(mine, ref, score_of):
    """Equal score sequences; positions may differ only inside equal-score groups."""
    assert mine.shape == ref.shape
    sm, sr = score_of(mine), score_of(ref)
    assert np.array_equal(sm, sr)
    for v in np.unique(sm):
        if (sm == v).sum() and v != sr[-1]:
            assert set(mine[sm == v].tolist()) == set(ref[sr == v].tolist())


def test_lserve_seer_golden():
    """The reference's std::sort leaves equal block/token scores in arbitrary
    order (the oracle takes the lowest index), so orders are compared up to
    ties."""
    past, qq, nk = mg.idx_inputs()
    for name in ("lserve", "seer_budget", "seer_threshold"):
        assert mg.digest(past, qq, nk) == str(load(name)["digest"])
    lsv, bud = O.lserve_topk_i16(past, qq, nk), O.seer_budget_i16(past, qq, nk)
    for q in range(qq.shape[0]):
        sc = visible_scores(past, qq, nk, q)
        nb = (sc.size + 15) // 16
        blk = np.array([sc[16 * b:16 * b + 16].max() for b in range(nb)], np.float32)
        assert_same_up_to_ties(lsv[q], load("lserve")["idx"][q], lambda i: blk[i])
        assert_same_up_to_ties(bud[q], load("seer_budget")["idx"][q], lambda i: sc[i])
    assert np.array_equal(O.seer_threshold_i16(past, qq, nk, 20000), load("seer_threshold")["words"])


def test_bm25_golden():
    """The reference sums query terms in unordered_map order, the oracle in
    ascending term order; fp64 sums may differ in the last bit, so indices
    are compared after dropping near-ties (relative gap < 1e-12)."""
    g = load("bm25")
    tp, pd, pt, dl, qs = mg.bm25_inputs()
    assert mg.digest(tp, pd, pt, dl, qs) == str(g["digest"])
    idx, sc = O.bm25_topk(tp, pd, pt, dl, qs, 64)
    for q in range(qs.shape[0]):
        ref = g["idx"][q]
        mism = np.nonzero(idx[q] != ref)[0]
        for i in mism:
            # a mismatch is only allowed between (near-)equal scores
            j = np.nonzero(ref == idx[q][i])[0]
            assert j.size == 1 or i == 63
            assert abs(sc[q][i] - sc[q][min(i + 1, 63)]) <= 1e-12 * abs(sc[q][i]) or \
                   abs(sc[q][i] - sc[q][max(i - 1, 0)]) <= 1e-12 * abs(sc[q][i])


def test_bf16_score_rounds_each_product():
    """The oracle's bf16 score is the reference's loop `s += a * b` in fp32 with
    no contraction: a product that overflows becomes +inf before it is added,
    so -3e38 + 3e38 * 2 scores +inf (a fused multiply-add would give 3e38), and
    an ordinary row keeps its plain sequential sum."""
    mem = np.zeros((3, 128), np.float32)
    mem[0, 0], mem[0, 1] = -3.0e38, 3.0e38
    mem[1, :4] = [1.5, -2.0, 0.25, 8.0]
    mem[2, 0], mem[2, 1] = 3.0e38, -3.0e38
    q = np.zeros((1, 128), np.float32)
    q[0, :4] = [1.0, 2.0, 4.0, 0.5]
    idx, sc = O.ip_topk_bf16(gen.bf16_bits(mem), gen.bf16_bits(q), 3)
    assert idx[0].tolist() == [0, 1, 2]
    assert np.isposinf(sc[0, 0]) and sc[0, 1] == np.float32(2.5) and np.isneginf(sc[0, 2])


def test_e4m3_decode_table():
    vals = O.e4m3_to_f32(np.arange(256, dtype=np.uint8))
    assert vals[0x38] == 1.0 and vals[0x7E] == 448.0 and vals[0xFE] == -448.0
    assert vals[0x01] == 2.0 ** -9 and vals[0x08] == 2.0 ** -6
    # round trip of the generator's encoder on representable values
    codes = np.array([c for c in range(256) if c not in (0x7F, 0xFF, 0x80)], np.uint8)
    assert np.array_equal(gen.e4m3_bits(vals[codes]), codes)


def test_fp8_dsa_score_is_exact_dot():
    """orc_dsa_score_fp8 == fp32 head sum of float(ReLU(exact dot)) with the
    reference's association (indexer_tb.cpp:27-46)."""
    q = gen.e4m3_bits(gen.normal_f32(171, (4, 128)) * 100)
    k = gen.e4m3_bits(gen.normal_f32(172, (50, 128)) * 100)
    w = gen.uniform01_f32(173, (4,))
    qv, kv = O.e4m3_to_f32(q).astype(np.float64), O.e4m3_to_f32(k).astype(np.float64)
    idx, sc = O.dsa_indexer_fp8(q[None], k, w[None], pos0=49, topk=50)
    for j in range(50):
        total = np.float32(0)
        for h in range(4):
            x = np.float32(max(float(qv[h] @ kv[j]), 0.0))
            total = np.float32(total + np.float32(w[h] * x))
        assert sc[0][list(idx[0]).index(j)] == total


# ----------------------------------------------------- live reference pins

ref_needed = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built here")


@ref_needed
@pytest.mark.parametrize("seed", [1, 2, 3])
def test_flat_live(seed):
    mem = gen.normal_f32(seed * 10, (2049, 96))
    qry = gen.normal_f32(seed * 10 + 1, (3, 96))
    idx, bm, sc = O.ip_topk_f32(mem, qry, 100, 5.0, want_scores=True)
    rf = O.RefFlatMemory(mem)
    ridx, rbm = rf.pipeline(qry, 100, 5.0, n_threads=2)
    assert np.array_equal(idx, ridx)
    assert np.array_equal(bm, rbm)


@ref_needed
def test_indexers_live():
    for seed in (201, 301):
        q, k, w = (gen.ints(seed, (16, 128), -128, 127).astype(np.int16),
                   gen.ints(seed + 1, (2500, 128), -128, 127).astype(np.int16),
                   (gen.uniform01_f32(seed + 2, (16,)) * 2).astype(np.float32))
        assert np.array_equal(O.dsa_indexer_i16(q, k, w, 2048)[0], O.ref_dsa_i16(q, k, w))
        past, qq, nk = mg.idx_inputs(L=1280, nq=24, seed=seed)
        lsv, rl = O.lserve_topk_i16(past, qq, nk), O.ref_lserve_i16(past, qq, nk)
        bud, rb = O.seer_budget_i16(past, qq, nk), O.ref_seer_budget_i16(past, qq, nk)
        for q in range(qq.shape[0]):
            sc = visible_scores(past, qq, nk, q)
            blk = np.array([sc[16 * b:16 * b + 16].max() for b in range((sc.size + 15) // 16)])
            assert_same_up_to_ties(lsv[q], rl[q], lambda i: blk[i])
            assert_same_up_to_ties(bud[q], rb[q], lambda i: sc[i])
        assert np.array_equal(O.seer_threshold_i16(past, qq, nk, 15000),
                              O.ref_seer_threshold_i16(past, qq, nk, 15000))


@ref_needed
def test_paged_decode_live():
    keys = gen.normal_f32(401, (1000, 64))
    vals = gen.normal_f32(402, (1000, 64))
    q = gen.normal_f32(403, (64,))
    blocks, out = O.ref_paged_decode_f32(keys, vals, q, 64, 4)
    summ = O.block_mean_f32(keys, 64)
    sc = O.ip_score_f32(summ, q[None])[0]
    mine = O.topk_f32(sc, 4)
    assert np.array_equal(mine, blocks)
    assert np.array_equal(O.block_sparse_attention_f32(keys, vals, mine, q, 64).view(np.uint32),
                          out.view(np.uint32))


@ref_needed
def test_reference_doctests_pass():
    """The reference's own 5 unit-test binaries (50 assertions) run green."""
    ref_dir = os.path.join(os.path.dirname(O.__file__), "_ref")
    for t in ("innerproduct", "topk_retrieval", "threshold_retrieval", "paged_kv_index_builder",
              "block_sparse_attention"):
        r = subprocess.run([os.path.join(ref_dir, f"test_{t}")], capture_output=True, text=True)
        assert r.returncode == 0 and "Status: SUCCESS" in r.stdout, (t, r.stdout[-500:])
