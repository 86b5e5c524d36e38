"""The heteromm_cpp_kernels Python module (bindings of the C++ step API under
the names the reference's pipeline generator calls, python_dispatch_pass.h:
518-540) on the CPU: its `_cpu` functions against the oracle, and the calling
conventions of the generated pipeline (positional data, keyword parameters,
unknown keywords ignored).  The `_gpu` functions are checked against these in
tests/test_py_kernels_gpu.py."""
import math
import sys

import numpy as np
import pytest

from heteromm_b200 import build as B
from oracle import oracle as O

NAMES = ["InnerProductCompute", "TopKRetrieval", "ThresholdRetrieval",
         "InnerProductTopKRetrieval", "PagedKVIndexBuilder", "BlockSparseAttention",
         "FusedBM25Retrieval"]


@pytest.fixture(scope="module")
def K():
    B.build()
    if not B.build_py_kernels():
        pytest.skip("pybind11 is not installed")
    sys.path.insert(0, B.LIB_DIR)
    import heteromm_cpp_kernels
    return heteromm_cpp_kernels


def test_generator_names_exported(K):
    for n in NAMES:
        for kt in ("cpu", "gpu"):
            assert callable(getattr(K, f"{n}_{kt}"))


def test_flat_steps_match_oracle(K):
    rng = np.random.default_rng(11)
    mem = rng.standard_normal((700, 48)).astype(np.float32)
    q = rng.standard_normal(48).astype(np.float32)
    s = K.InnerProductCompute_cpu(mem, q, k=5, threshold=0.0, page_size=9)   # extra keywords ignored
    np.testing.assert_array_equal(s, O.ip_score_f32(mem, q)[0])
    np.testing.assert_array_equal(K.TopKRetrieval_cpu(s, k=37), O.topk_f32(s, 37))
    assert K.TopKRetrieval_cpu(s).size == 64   # the reference's default k
    words = O.threshold_bitmap_f32(s, 2.5)
    sel = np.flatnonzero(np.unpackbits(words.view(np.uint8), bitorder="little")[:s.size])
    np.testing.assert_array_equal(K.ThresholdRetrieval_cpu(s, threshold=2.5), sel)
    idx, _, _ = O.ip_topk_f32(mem, q, 10)
    np.testing.assert_array_equal(K.InnerProductTopKRetrieval_cpu(mem, q, k=10), idx[0])


def test_paged_steps_match_oracle(K):
    rng = np.random.default_rng(12)
    keys = rng.standard_normal((333, 32)).astype(np.float32)
    vals = rng.standard_normal((333, 32)).astype(np.float32)
    w = rng.standard_normal((24, 32)).astype(np.float32)
    summ = K.PagedKVIndexBuilder_cpu((keys, vals), page_size=7, weight=w)
    np.testing.assert_array_equal(summ, O.paged_kv_summary_f32(keys, w, 7))
    ident = K.PagedKVIndexBuilder_cpu({"keys": keys, "values": vals}, page_size=7)
    np.testing.assert_array_equal(ident, O.paged_kv_summary_f32(keys, np.eye(32, dtype=np.float32), 7))
    q = rng.standard_normal(32).astype(np.float32)
    blocks = np.array([3, 47, 0, 12], np.int32)   # 47: the ragged last block
    out = K.BlockSparseAttention_cpu(q, (keys, vals), blocks, q, page_size=7)
    ref = O.block_sparse_attention_f32(keys, vals, blocks, q, 7)
    np.testing.assert_allclose(out, ref, rtol=2e-5, atol=2e-6)
    # input_data None: the query is attended
    np.testing.assert_array_equal(K.BlockSparseAttention_cpu(q, (keys, vals), blocks, None, page_size=7), out)


def _bm25_top64(docs, term):
    """The reference's BM25 (bm25_fpga_retrieval.cpp:158-199) for a one-term
    query, in Python doubles: top-64 by (score desc, document asc)."""
    n = len(docs)
    dl = [sum(d.values()) for d in docs]
    avgdl = sum(dl) / n
    df = sum(1 for d in docs if term in d)
    k1, b = 1.2, 0.75
    sc = [0.0] * n
    if df:
        idf = math.log((n - df + 0.5) / (df + 0.5) + 1.0)
        for i, d in enumerate(docs):
            if term in d:
                tf = d[term]
                sc[i] = idf * (tf * (k1 + 1.0)) / (tf + k1 * (1.0 - b + b * dl[i] / avgdl))
    return sorted(range(n), key=lambda i: (-sc[i], i))[:64]


def test_bm25_matches_formula(K):
    rng = np.random.default_rng(13)
    docs = []
    for _ in range(400):
        d = {}
        for t in rng.integers(0, 60, size=rng.integers(3, 30)):
            d[int(t) * 3 + 1] = d.get(int(t) * 3 + 1, 0) + int(rng.integers(1, 4))
        docs.append(d)
    for term in (1, 4, 91, 178, 2):   # 2: in no document
        got = K.FusedBM25Retrieval_cpu(docs, {term: 1}, k=10)
        assert list(got) == _bm25_top64(docs, term)
        assert list(K.FusedBM25Retrieval_cpu(docs, [term])) == list(got)


def test_bad_arguments_raise(K):
    with pytest.raises(TypeError):
        K.ThresholdRetrieval_cpu(np.zeros(4, np.float32))        # threshold is required
    with pytest.raises(TypeError):
        K.InnerProductCompute_cpu(np.zeros((4, 4), np.float32))  # query missing
    with pytest.raises(ValueError):
        K.InnerProductCompute_cpu(np.zeros(4, np.float32), np.zeros(4, np.float32))
