"""Host-side BM25 statistics (hmm_bm25_stats_host, no GPU needed) against the
oracle: idf per term and avg_dl, bit-exact."""
import numpy as np

import gen
from heteromm_b200 import bm25
from oracle import oracle as O


def test_stats_host_matches_oracle():
    tp, pd, tf, dl = gen.bm25_corpus(501, 3000, 400, 15.0)
    idf, avg = bm25.stats_host(tp, dl)
    assert np.array_equal(idf.view(np.uint64), O.bm25_idf(tp, dl.size).view(np.uint64))
    assert avg == O.bm25_avgdl(dl)


def test_stats_host_empty_terms_have_zero_idf():
    tp = np.array([0, 0, 3, 3], np.int64)          # terms 0 and 2 have no postings
    dl = np.array([1, 1, 1], np.int32)
    idf, avg = bm25.stats_host(tp, dl)
    assert idf[0] == 0.0 and idf[2] == 0.0 and idf[1] > 0.0
    assert avg == 1.0
