"""BM25 fused score + top-k over a CSR inverted index (the GPU form of the
reference's BM25IndexMemory + FusedBM25Retrieval).

An index is built once from CSR arrays (host or device): the idf and avg_dl
come from the host (hmm_bm25_stats_host, the reference's expressions and
libm), the per-range skips and per-posting score contributions from the device
(hmm_bm25_prepare).  `topk` then scores a batch of queries.  The CSR itself can
be built on the device from per-document term counts (`csr_from_docs`,
`BM25Index.from_docs`), e.g. the reference's term_freq.bin export
(`BM25Index.from_export`, file formats in bm25_export.py).
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


def csr_from_docs(doc_ptr, terms, counts, n_terms: int, device="cuda"):
    """Term-major CSR built on the device from per-document term counts
    (hmm_bm25_csr_from_docs): document d's terms and counts are
    [doc_ptr[d], doc_ptr[d+1]) of `terms` (vocabulary index) and `counts`,
    each term at most once per document.  Returns device tensors
    (term_ptr int64 [n_terms+1], post_doc int32, post_tf int16 holding the
    uint16 counts, doc_len int32)."""
    dev = torch.device(device)

    def on(a, np_dt, t_dt):
        if isinstance(a, torch.Tensor):
            return a.to(device=dev, dtype=t_dt).contiguous()
        return torch.from_numpy(np.ascontiguousarray(a, np_dt)).to(dev)

    dp = on(doc_ptr, np.int64, torch.int64)
    tr = on(terms, np.int32, torch.int32)
    ct = on(np.asarray(counts, np.uint32).view(np.int32) if not isinstance(counts, torch.Tensor)
            else counts, np.int32, torch.int32)
    n_docs = dp.numel() - 1
    n_post = int(dp[-1].item()) if n_docs > 0 else 0
    term_ptr = torch.empty(n_terms + 1, dtype=torch.int64, device=dev)
    post_doc = torch.empty(max(n_post, 1), dtype=torch.int32, device=dev)
    post_tf = torch.empty(max(n_post, 1), dtype=torch.int16, device=dev)
    doc_len = torch.empty(max(n_docs, 1), dtype=torch.int32, device=dev)
    ws = workspace(load().hmm_bm25_csr_workspace_size(n_docs, n_terms), dev)
    call("hmm_bm25_csr_from_docs", dp.data_ptr(), tr.data_ptr(), ct.data_ptr(), n_docs, n_terms,
         term_ptr.data_ptr(), post_doc.data_ptr(), post_tf.data_ptr(), doc_len.data_ptr(),
         ws.data_ptr(), ws.numel(), _stream())
    return term_ptr, post_doc[:n_post], post_tf[:n_post], doc_len[:n_docs]


class BM25Index:
    """Device-resident CSR index with its skips and document factors."""

    def __init__(self, term_ptr, post_doc, post_tf, doc_len, device="cuda"):
        """From CSR arrays: NumPy (uploaded) or torch tensors (used on the device
        as they are; post_tf as int16 holding the uint16 counts)."""
        self.device = torch.device(device)

        def host(a):
            return a.cpu().numpy() if isinstance(a, torch.Tensor) else a

        idf, self.avg_dl = stats_host(host(term_ptr), host(doc_len))
        self.n_terms = len(term_ptr) - 1
        self.n_docs = len(doc_len)
        self.n_postings = int(term_ptr[-1]) if len(term_ptr) else 0

        def dev(a, dt):
            if isinstance(a, torch.Tensor):
                return a.to(self.device).contiguous()
            return torch.from_numpy(np.ascontiguousarray(a, dt)).to(self.device)

        self.term_ptr = dev(term_ptr, np.int64)
        self.post_doc = dev(post_doc, np.int32)
        self.post_tf = (dev(post_tf, np.int16) if isinstance(post_tf, torch.Tensor)
                        else dev(np.asarray(post_tf, np.uint16).view(np.int16), np.int16))
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

    @classmethod
    def from_docs(cls, doc_ptr, terms, counts, n_terms: int, device="cuda"):
        """Index of per-document term counts, its CSR built on the device."""
        return cls(*csr_from_docs(doc_ptr, terms, counts, n_terms, device), device=device)

    @classmethod
    def from_export(cls, export_dir: str, device="cuda", source: str = "term_freq"):
        """Index of the reference's BM25 export directory
        (rag_test/export_bm25_data.py): from term_freq.bin, transposed on the
        device (source="term_freq"), or from inverted_index.bin, already term
        major (source="inverted_index").  The vocabulary size comes from
        doc_freq.bin, whose counts are checked against the postings."""
        import os

        from . import bm25_export as E
        df = E.load_doc_freq(os.path.join(export_dir, "doc_freq.bin"))
        if source == "term_freq":
            doc_ptr, terms, counts = E.load_term_freq(os.path.join(export_dir, "term_freq.bin"))
            index = cls.from_docs(doc_ptr, terms, counts, df.size, device)
        elif source == "inverted_index":
            term_ptr, post_doc, post_tf = E.load_inverted_index(
                os.path.join(export_dir, "inverted_index.bin"))
            if term_ptr.size - 1 != df.size:
                raise ValueError("inverted_index.bin and doc_freq.bin differ in vocabulary size")
            # documents without terms appear in no posting: take the count from
            # term_freq.bin's header when it is there
            tf_path = os.path.join(export_dir, "term_freq.bin")
            n_docs = int(post_doc.max()) + 1 if post_doc.size else 0
            if os.path.exists(tf_path):
                n_docs = max(n_docs, E.load_term_freq_num_docs(tf_path))
            doc_len = np.bincount(post_doc, weights=post_tf, minlength=n_docs).astype(np.int32)
            index = cls(term_ptr, post_doc, post_tf, doc_len, device)
        else:
            raise ValueError(f"unknown source {source!r}")
        got = np.diff(index.term_ptr.cpu().numpy())
        if not np.array_equal(got, df.astype(np.int64)):
            raise ValueError("doc_freq.bin disagrees with the postings")
        return index

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
