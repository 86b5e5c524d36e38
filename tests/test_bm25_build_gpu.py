"""The BM25 inverted index built on the device from per-document term counts
(hmm_bm25_csr_from_docs) against the same transpose done on the host, bit for
bit, and the index built from the reference's export files against the index
built from the CSR directly (identical top-k)."""
import numpy as np
import pytest
import torch

from heteromm_b200 import _abi
from heteromm_b200.bm25 import BM25Index, csr_from_docs

from bm25_export_files import corpus, doc_major, term_major, write_export

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n_docs,n_vocab,empty_every", [(1, 7, 0), (1023, 40, 0),
                                                        (5000, 300, 13), (2049, 5, 0)])
def test_device_csr_equals_host_transpose(n_docs, n_vocab, empty_every):
    docs = corpus(n_docs + n_vocab, n_docs, n_vocab, empty_every)
    tp, pd, pt, dl = csr_from_docs(*doc_major(docs), n_vocab)
    tp0, pd0, pt0, dl0, _ = term_major(docs, n_vocab)
    np.testing.assert_array_equal(tp.cpu().numpy(), tp0)
    np.testing.assert_array_equal(pd.cpu().numpy(), pd0)
    np.testing.assert_array_equal(pt.cpu().numpy().view(np.uint16), pt0)
    np.testing.assert_array_equal(dl.cpu().numpy(), dl0)


def test_bad_inputs_are_reported():
    dp = np.array([0, 2, 3], np.int64)
    with pytest.raises(_abi.HmmError):   # term outside the vocabulary
        csr_from_docs(dp, np.array([0, 9, 1], np.int32), np.array([1, 1, 1], np.uint32), 5)
    with pytest.raises(_abi.HmmError):   # a zero count
        csr_from_docs(dp, np.array([0, 3, 1], np.int32), np.array([1, 0, 1], np.uint32), 5)
    with pytest.raises(_abi.HmmError):   # doc_ptr decreasing
        csr_from_docs(np.array([0, 3, 2], np.int64), np.array([0, 3, 1], np.int32),
                      np.array([1, 1, 1], np.uint32), 5)


def test_index_from_docs_and_export(tmp_path):
    n_vocab = 400
    docs = corpus(31, 6000, n_vocab, empty_every=50)
    write_export(str(tmp_path), docs, n_vocab)
    tp0, pd0, pt0, dl0, _ = term_major(docs, n_vocab)
    ref = BM25Index(tp0, pd0, pt0, dl0)
    rng = np.random.default_rng(3)
    q = torch.from_numpy(rng.integers(0, n_vocab, size=(64, 6)).astype(np.int32)).cuda()
    want_i, want_s = ref.topk(q, 10)
    for index in (BM25Index.from_docs(*doc_major(docs), n_vocab),
                  BM25Index.from_export(str(tmp_path)),
                  BM25Index.from_export(str(tmp_path), source="inverted_index")):
        assert index.n_docs == 6000 and index.avg_dl == ref.avg_dl
        got_i, got_s = index.topk(q, 10)
        assert torch.equal(got_i, want_i)
        assert torch.equal(got_s, want_s)
