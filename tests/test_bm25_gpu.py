"""GPU parity of the BM25 fused score + top-k (hmm_bm25_topk_csr) against the
oracle: identical doc ids and bit-identical fp64 scores."""
import numpy as np
import pytest
import torch

import gen
import heteromm_b200 as hmm
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def check(cuda, corpus, qterms, k):
    tp, pd, tf, dl = corpus
    index = hmm.BM25Index(tp, pd, tf, dl, cuda)
    idx, sc = index.topk(torch.from_numpy(np.ascontiguousarray(qterms, np.int32)).to(cuda), k)
    oidx, osc = O.bm25_topk(tp, pd, tf, dl, qterms, k)
    assert np.array_equal(idx.cpu().numpy(), oidx)
    assert np.array_equal(sc.cpu().numpy().view(np.uint64), osc.view(np.uint64))


@pytest.mark.parametrize("n_docs,vocab,mean,nq,qlen,k", [
    (5000, 500, 20.0, 32, 8, 10),       # two doc ranges
    (20000, 2000, 40.0, 16, 8, 64),     # five ranges, the reference's k = 64
    (4096, 300, 10.0, 8, 3, 128),       # exactly one range, largest k
    (9000, 50, 5.0, 4, 16, 10),         # small vocabulary: long posting lists
])
def test_bm25_matches_oracle(cuda, n_docs, vocab, mean, nq, qlen, k):
    corpus = gen.bm25_corpus(600 + n_docs, n_docs, vocab, mean)
    q = gen.bm25_queries(601 + n_docs, nq, qlen, vocab)
    check(cuda, corpus, q, k)


def test_bm25_query_edge_cases(cuda):
    corpus = gen.bm25_corpus(610, 7000, 300, 12.0)
    q = np.array([[5, 5, 5, 7],            # repeated term
                  [-1, 300, 1000, 3],      # out-of-vocabulary ids are ignored
                  [-1, -1, -1, -1],        # no terms: every doc scores 0
                  [299, 0, 150, 299]], np.int32)
    check(cuda, corpus, q, 10)


def test_bm25_k_above_doc_count(cuda):
    corpus = gen.bm25_corpus(620, 7, 20, 4.0)
    q = gen.bm25_queries(621, 3, 4, 20)
    check(cuda, corpus, q, 12)


def test_bm25_empty_corpus(cuda):
    tp = np.zeros(11, np.int64)
    index = hmm.BM25Index(tp, np.zeros(0, np.int32), np.zeros(0, np.uint16),
                          np.zeros(0, np.int32), cuda)
    idx, sc = index.topk(torch.tensor([[1, 2]], dtype=torch.int32, device=cuda), 5)
    assert (idx == -1).all() and (sc == 0).all()


def test_bm25_heavy_ties(cuda):
    """Every doc has length 4 and tf 1: docs sharing the query terms tie
    exactly, so the selection must fall back to the lowest doc ids."""
    n_docs, vocab = 10000, 6
    docs_terms = [sorted({(d * 7 + j) % vocab for j in range(4)}) for d in range(n_docs)]
    post = {t: [] for t in range(vocab)}
    for d, ts in enumerate(docs_terms):
        for t in ts:
            post[t].append(d)
    tp = np.zeros(vocab + 1, np.int64)
    tp[1:] = np.cumsum([len(post[t]) for t in range(vocab)])
    pd = np.concatenate([np.array(post[t], np.int32) for t in range(vocab)])
    tf = np.ones(pd.size, np.uint16)
    dl = np.array([len(ts) for ts in docs_terms], np.int32)
    q = np.array([[0, 1], [2, -1], [5, 4], [0, 3]], np.int32)
    check(cuda, (tp, pd, tf, dl), q, 64)
