"""heteromm_cpp_kernels on a B200: every `<StepClass>_gpu` function (the GPU
work of the step's KernelType::GPU arm, i.e. this library's CUDA kernels)
against its `_cpu` twin on the same inputs, on both of its routes: NumPy
buffers handed to the GPU work directly, and other shapes through the step
objects.  Bit-exact except BlockSparseAttention, whose
softmax uses the device exp and another summation order (rtol 2e-5, atol
2e-6, as in tests/cpp/test_steps_gpu.cpp)."""
import sys

import numpy as np
import pytest

from heteromm_b200 import build as B

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def K():
    B.build()
    if not B.build_py_kernels():
        pytest.skip("pybind11 is not installed")
    sys.path.insert(0, B.LIB_DIR)
    import heteromm_cpp_kernels
    return heteromm_cpp_kernels


def test_flat_steps(K):
    rng = np.random.default_rng(21)
    mem = rng.standard_normal((3000, 96)).astype(np.float32)
    q = rng.standard_normal(96).astype(np.float32)
    s_cpu = K.InnerProductCompute_cpu(mem, q)
    np.testing.assert_array_equal(K.InnerProductCompute_gpu(mem, q), s_cpu)
    sc = rng.standard_normal(5000).astype(np.float32)
    sc[::7] = 1.5   # exact ties: lowest index first
    for k in (1, 17, 300, 4096):
        np.testing.assert_array_equal(K.TopKRetrieval_gpu(sc, k=k), K.TopKRetrieval_cpu(sc, k=k))
    np.testing.assert_array_equal(K.TopKRetrieval_gpu(sc[:3000], k=6000),
                                  K.TopKRetrieval_cpu(sc[:3000], k=6000))
    np.testing.assert_array_equal(K.ThresholdRetrieval_gpu(sc, threshold=0.5),
                                  K.ThresholdRetrieval_cpu(sc, threshold=0.5))
    np.testing.assert_array_equal(K.InnerProductTopKRetrieval_gpu(mem, q, k=10),
                                  K.InnerProductTopKRetrieval_cpu(mem, q, k=10))


def test_paged_steps(K):
    rng = np.random.default_rng(22)
    keys = rng.standard_normal((333, 64)).astype(np.float32)
    w = rng.standard_normal((24, 64)).astype(np.float32)
    np.testing.assert_array_equal(K.PagedKVIndexBuilder_gpu((keys, keys), page_size=7, weight=w),
                                  K.PagedKVIndexBuilder_cpu((keys, keys), page_size=7, weight=w))
    k2 = rng.standard_normal((500, 128)).astype(np.float32)
    v2 = rng.standard_normal((500, 128)).astype(np.float32)
    q = rng.standard_normal(128).astype(np.float32)
    blocks = np.array([3, 62, 0, 17, 100], np.int32)   # 62: ragged; 100: past the end
    np.testing.assert_allclose(K.BlockSparseAttention_gpu(q, (k2, v2), blocks, q, page_size=8),
                               K.BlockSparseAttention_cpu(q, (k2, v2), blocks, q, page_size=8),
                               rtol=2e-5, atol=2e-6)
    with pytest.raises(RuntimeError):   # a negative block id is reported, not followed
        K.BlockSparseAttention_gpu(q, (k2, v2), np.array([1, -2], np.int32), q, page_size=8)


def test_bm25(K):
    rng = np.random.default_rng(23)
    docs = []
    for _ in range(3000):
        d = {}
        for _ in range(int(rng.integers(3, 40))):
            t = int(rng.integers(0, 200)) * 3 + 5
            d[t] = d.get(t, 0) + int(rng.integers(1, 5))
        docs.append(d)
    for i in range(12):   # queries of at most two tokens: order-free fp64 sums
        query = {int(rng.integers(0, 200)) * 3 + 5: 1}
        if i % 2:
            query[int(rng.integers(0, 200)) * 3 + 5] = 2
        np.testing.assert_array_equal(K.FusedBM25Retrieval_gpu(docs, query),
                                      K.FusedBM25Retrieval_cpu(docs, query))


def test_direct_and_step_routes_agree(K):
    rng = np.random.default_rng(24)
    wide = rng.standard_normal((2000, 100)).astype(np.float32)
    q = rng.standard_normal(96).astype(np.float32)
    # 100 columns for a 96-wide query: the step route, which reads the first 96
    np.testing.assert_array_equal(K.InnerProductCompute_gpu(wide, q), K.InnerProductCompute_cpu(wide, q))
    np.testing.assert_array_equal(K.InnerProductCompute_gpu(np.ascontiguousarray(wide[:, :96]), q),
                                  K.InnerProductCompute_cpu(wide, q))
    np.testing.assert_array_equal(K.InnerProductTopKRetrieval_gpu(wide, q, k=20),
                                  K.InnerProductTopKRetrieval_cpu(wide, q, k=20))
    keys = rng.standard_normal((130, 32)).astype(np.float32)
    eye = np.eye(32, dtype=np.float32)
    np.testing.assert_array_equal(K.PagedKVIndexBuilder_gpu((keys, keys), page_size=16),
                                  K.PagedKVIndexBuilder_cpu((keys, keys), page_size=16, weight=eye))
    # a weight of the wrong width: the step route, which returns no summaries
    bad = K.PagedKVIndexBuilder_gpu((keys, keys), page_size=16, weight=eye[:, :8])
    assert bad.size == 0
    with pytest.raises(ValueError):   # values shorter than keys
        K.BlockSparseAttention_gpu(keys[0], (keys, keys[:100]), np.array([0, 2], np.int32), None,
                                   page_size=16)
