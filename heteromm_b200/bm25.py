"""BM25 fused score + top-k over a CSR inverted index (the GPU form of the
reference's BM25IndexMemory + FusedBM25Retrieval).

An index is built once from host CSR arrays: the idf and avg_dl come from
the host (hmm_bm25_stats_host, the reference's expressions and libm), the
per-range skips and per-posting score contributions from the device
(hmm_bm25_prepare).  `topk` then scores a batch of queries.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from ._abi import call, load
from .flat import _check, _stream, workspace


def stats_host(term_ptr: np.ndarray, doc_len: np.ndarray):
    """(idf [n_terms] fp64, avg_dl) computed on the host as the reference does."""
    tp = np.ascontiguousarray(term_ptr, np.int64)
    dl = np.ascontiguousarray(doc_len, np.int32)
    idf = np.empty(max(tp.size - 1, 0), np.float64)
    avg = C.c_double(0.0)
    call("hmm_bm25_stats_host", tp.ctypes.data, tp.size - 1, dl.ctypes.data, dl.size,
         idf.ctypes.data, C.byref(avg))
    return idf, avg.value


class BM25Index:
    """Device-resident CSR index with its skips and document factors."""

    def __init__(self, term_ptr, post_doc, post_tf, doc_len, device="cuda"):
        self.device = torch.device(device)
        idf, self.avg_dl = stats_host(term_ptr, doc_len)
        self.n_terms = len(term_ptr) - 1
        self.n_docs = len(doc_len)
        self.n_postings = int(term_ptr[-1]) if len(term_ptr) else 0

        def dev(a, dt):
            return torch.from_numpy(np.ascontiguousarray(a, dt)).to(self.device)

        self.term_ptr = dev(term_ptr, np.int64)
        self.post_doc = dev(post_doc, np.int32)
        self.post_tf = dev(np.asarray(post_tf, np.uint16).view(np.int16), np.int16)
        self.doc_len = dev(doc_len, np.int32)
        self.idf = dev(idf, np.float64)
        ns = load().hmm_bm25_skips_count(self.n_terms, self.n_docs)
        self.skips = torch.empty((max(ns, 1),), dtype=torch.int32, device=self.device)
        self.impact = torch.empty((max(self.n_postings, 1),), dtype=torch.float64,
                                  device=self.device)
        ws = workspace(256, self.device)
        call("hmm_bm25_prepare", self.term_ptr.data_ptr(), self.post_doc.data_ptr(),
             self.post_tf.data_ptr(), self.n_terms, self.doc_len.data_ptr(), self.n_docs,
             self.idf.data_ptr(), C.c_double(self.avg_dl), self.skips.data_ptr(),
             self.impact.data_ptr(), ws.data_ptr(), ws.numel(), _stream())

    def topk(self, qterms: torch.Tensor, k: int):
        """(doc ids [nq, k] int32, scores [nq, k] fp64) for queries [nq, qlen] int32."""
        _check(qterms, torch.int32, "qterms")
        q2 = qterms.reshape(-1, qterms.shape[-1]) if qterms.dim() else qterms
        nq, qlen = q2.shape
        idx = torch.empty((nq, k), dtype=torch.int32, device=self.device)
        sc = torch.empty((nq, k), dtype=torch.float64, device=self.device)
        ws = workspace(load().hmm_bm25_topk_workspace_size(self.n_docs, nq, k), self.device)
        call("hmm_bm25_topk_csr", self.post_doc.data_ptr(), self.impact.data_ptr(),
             self.n_postings, self.n_terms, self.n_docs, self.skips.data_ptr(), q2.data_ptr(),
             nq, qlen, k, idx.data_ptr(), sc.data_ptr(), ws.data_ptr(), ws.numel(), _stream())
        return idx, sc
