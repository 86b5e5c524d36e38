"""Generates the golden fixtures in tests/golden/*.npz by running the
reference's OWN CPU code, compiled from its sources by oracle/build_ref.sh.

Inputs are regenerated from seeds by tests/golden/gen.py; each fixture stores
the seeds and shapes, a SHA-256 of the input bytes (to catch generator drift)
and the reference's outputs.  Run in a container that has the reference
checkout:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import gen  # noqa: E402
from oracle import oracle as O  # noqa: E402


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def flat_inputs(n=3000, d=128, nq=4):
    return gen.normal_f32(101, (n, d)), gen.normal_f32(102, (nq, d))


def topk_edge_inputs():
    s = gen.normal_f32(111, (5000,))
    s = np.round(s * 4) / 4            # many exact ties
    s[17] = -0.0
    s[18] = 0.0
    s[100:110] = s.max()               # a tie at the top
    return s.astype(np.float32)


def paged_inputs(L=333, D=64, out=16):
    return gen.normal_f32(121, (L, D)), gen.normal_f32(122, (out, D))


def bsa_inputs(L=333, D=64):
    k = gen.normal_f32(131, (L, D))
    v = gen.normal_f32(132, (L, D))
    q = gen.normal_f32(133, (D,))
    blocks = np.array([5, 0, 41, 3, 40, 7], np.int32)   # block 41 is partial, 40 full
    return k, v, q, blocks


def dsa_inputs(L=4096):
    q = gen.ints(141, (16, 128), -128, 127).astype(np.int16)
    k = gen.ints(142, (L, 128), -128, 127).astype(np.int16)
    w = (gen.uniform01_f32(143, (16,)) * 2).astype(np.float32)
    return q, k, w


def idx_inputs(L=1152, nq=16, seed=151):
    past = gen.ints(seed, (L, 128), -100, 100).astype(np.int16)
    qq = gen.ints(seed + 1, (nq, 128), -100, 100).astype(np.int16)
    nk = gen.ints(seed + 2, (nq, 128), -100, 100).astype(np.int16)
    return past, qq, nk


def bm25_inputs():
    tp, pd, pt, dl = gen.bm25_corpus(161, 2000, 500, 60.0)
    qs = gen.bm25_queries(162, 8, 8, 500)
    return tp, pd, pt, dl, qs


def main() -> None:
    if not O.ref_available():
        O.build()
    out = {}
    mem, qry = flat_inputs()
    idx = np.stack([O.ref_topk_f32(O.ref_ip_score_f32(mem, q), 64) for q in qry])
    scores = np.stack([O.ref_ip_score_f32(mem, q) for q in qry])
    thr = np.float32(2.0 * np.sqrt(np.float32(128.0)))
    bm = np.stack([O.ref_threshold_f32(s, thr) for s in scores])
    out["flat_f32"] = dict(digest=digest(mem, qry), idx=idx, bitmap=bm, scores=scores,
                           threshold=thr, k=64)

    s = topk_edge_inputs()
    out["topk_edge"] = dict(digest=digest(s), idx64=O.ref_topk_f32(s, 64),
                            idx_all=O.ref_topk_f32(s, 6000), bitmap=O.ref_threshold_f32(s, 0.0))

    keys, W = paged_inputs()
    out["paged_kv"] = dict(digest=digest(keys, W), p8=O.ref_paged_kv_summary_f32(keys, W, 8),
                           p7=O.ref_paged_kv_summary_f32(keys, W, 7),
                           p1=O.ref_paged_kv_summary_f32(keys[:20], W, 1))

    k, v, q, blocks = bsa_inputs()
    out["bsa"] = dict(digest=digest(k, v, q, blocks),
                      out=O.ref_block_sparse_attention_f32(k, v, blocks, q, 8))

    q, kk, w = dsa_inputs()
    out["dsa_i16"] = dict(digest=digest(q, kk, w), idx=O.ref_dsa_i16(q, kk, w))

    past, qq, nk = idx_inputs()
    out["lserve"] = dict(digest=digest(past, qq, nk), idx=O.ref_lserve_i16(past, qq, nk))
    out["seer_budget"] = dict(digest=digest(past, qq, nk), idx=O.ref_seer_budget_i16(past, qq, nk))
    out["seer_threshold"] = dict(digest=digest(past, qq, nk),
                                 words=O.ref_seer_threshold_i16(past, qq, nk, 20000))

    tp, pd, pt, dl, qs = bm25_inputs()
    r = O.RefBM25(tp, pd, pt, dl.size)
    out["bm25"] = dict(digest=digest(tp, pd, pt, dl, qs), idx=np.stack([r.query(t) for t in qs]))

    for name, arrs in out.items():
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrs)
        print(name, {k: getattr(v, "shape", v) for k, v in arrs.items() if k != "digest"})


if __name__ == "__main__":
    main()
