"""Parity at the benchmark's full shapes, where candidate pools, threshold
refreshes and range skips see their full load: the GPU runs the whole batch,
and a spread subset of its queries is compared bit for bit with the oracle
(the oracle over all rows / documents for those queries).

  - sharded flat retrieval: 64Mi x 128 bf16 rows (the bench's generator),
    256 queries on the GPU, 16 of them checked, top-100
  - BM25: the 1M-document corpus (Zipf(1.1) over 30,522 terms, Poisson(60)
    lengths), 1,024 queries on the GPU, 64 of them checked, top-10
"""
import numpy as np
import pytest
import torch

import gen
import heteromm_b200 as hmm
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_flat_64Mi_rows_256_queries(cuda):
    import bench
    rows = bench.gen_rows(0, bench.N_ROWS, cuda)            # 64Mi x 128 bf16, 16 GiB
    qry = bench.gen_queries(cuda)                            # 256 x 128 bf16
    idx, sc = hmm.ip_topk_bf16(rows.view(torch.int16), qry.view(torch.int16), bench.TOP_K, 0)
    torch.cuda.synchronize()
    pick = np.arange(0, bench.N_QUERIES, 16)                # 16 queries across the batch
    got_i, got_s = idx.cpu().numpy()[pick], sc.cpu().numpy()[pick]
    q_host = qry.view(torch.int16).cpu().numpy().view(np.uint16)[pick]
    rows_host = rows.view(torch.int16).cpu().numpy().view(np.uint16)
    del rows
    torch.cuda.empty_cache()
    want_i, want_s = O.ip_topk_bf16(rows_host, q_host, bench.TOP_K, 0)
    assert np.array_equal(got_i, want_i)
    assert np.array_equal(got_s.view(np.uint32), want_s.view(np.uint32))


def test_bm25_1M_docs_1024_queries(cuda):
    import bench
    tp, pd, tf, dl = gen.bm25_corpus(bench.SEED_CORPUS, bench.B_DOCS, bench.B_VOCAB, bench.B_MEAN)
    q = gen.bm25_queries(bench.SEED_BQ, bench.B_NQ, bench.B_QLEN, bench.B_VOCAB)
    index = hmm.BM25Index(tp, pd, tf, dl, cuda)
    idx, sc = index.topk(torch.from_numpy(np.ascontiguousarray(q, np.int32)).to(cuda), bench.B_K)
    pick = np.arange(0, bench.B_NQ, 16)                     # 64 queries across the batch
    want_i, want_s = O.bm25_topk(tp, pd, tf, dl, q[pick], bench.B_K)
    assert np.array_equal(idx.cpu().numpy()[pick], want_i)
    assert np.array_equal(sc.cpu().numpy()[pick].view(np.uint64), want_s.view(np.uint64))
