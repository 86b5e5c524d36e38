"""Per-call time of heteromm_cpp_kernels at the flat-retrieval shape of the
reference's config 1 (65,536 x 128 fp32 rows, one query, top-64), GPU and CPU
functions, wall clock including the host->device copy of the rows.

    python heteromm_b200/src/py/time_py_kernels.py
"""
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "lib"))
import heteromm_cpp_kernels as K  # noqa: E402


def main():
    rng = np.random.default_rng(1)
    mem = rng.standard_normal((65536, 128)).astype(np.float32)
    q = rng.standard_normal(128).astype(np.float32)
    cases = [
        ("InnerProductTopKRetrieval_gpu", lambda: K.InnerProductTopKRetrieval_gpu(mem, q, k=64)),
        ("InnerProductTopKRetrieval_cpu", lambda: K.InnerProductTopKRetrieval_cpu(mem, q, k=64)),
        ("InnerProductCompute_gpu + TopKRetrieval_gpu",
         lambda: K.TopKRetrieval_gpu(K.InnerProductCompute_gpu(mem, q), k=64)),
        ("InnerProductCompute_cpu + TopKRetrieval_cpu",
         lambda: K.TopKRetrieval_cpu(K.InnerProductCompute_cpu(mem, q), k=64)),
    ]
    for name, fn in cases:
        fn()
        fn()
        n = 10
        t0 = time.perf_counter()
        for _ in range(n):
            fn()
        print("%-45s %.3f ms per call" % (name, (time.perf_counter() - t0) / n * 1e3), flush=True)
    assert np.array_equal(K.InnerProductTopKRetrieval_gpu(mem, q, k=64),
                          K.InnerProductTopKRetrieval_cpu(mem, q, k=64))


if __name__ == "__main__":
    main()
