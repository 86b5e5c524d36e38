"""numpy front end of the CPU oracle (oracle/hmm_oracle.c) and of the
reference's own CPU code built by oracle/build_ref.sh (oracle/_ref/).

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() and by
bench.py's CPU-baseline / reference legs as the checker.  Product code never
imports this module.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "libhmm_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libheteromm_ref.so")

_P = C.c_void_p
_I = C.c_int64


def reference_root() -> str:
    """The reference checkout: $HMM_REFERENCE_ROOT, else a directory named
    "reference" beside this repository."""
    return os.environ.get("HMM_REFERENCE_ROOT") or os.path.join(
        os.path.dirname(os.path.dirname(HERE)), "reference")


def build(force: bool = False) -> None:
    """Compile the oracle (gcc); compile the reference when its checkout exists."""
    if force or not os.path.exists(ORACLE_SO):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    ref = reference_root()
    if os.path.isdir(os.path.join(ref, "toolchain")) and (force or not os.path.exists(REF_SO)):
        subprocess.run([os.path.join(HERE, "build_ref.sh"), ref], check=True,
                       stdout=subprocess.DEVNULL)


_lib = None
_ref = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            build()
        _lib = C.CDLL(ORACLE_SO)
        _lib.orc_f32_key.restype = C.c_uint32
        _lib.orc_f32_key.argtypes = [C.c_float]
        _lib.orc_topk_f32.restype = _I
        _lib.orc_topk_f32_i64.restype = _I
        _lib.orc_paged_kv_summary_f32.restype = _I
        _lib.orc_block_mean_f32.restype = _I
        _lib.orc_block_pages.restype = _I
        _lib.orc_dsa_indexer_i16.restype = _I
        _lib.orc_seer_words_per_query.restype = _I
        _lib.orc_e4m3_scaled.restype = C.c_int32
        _lib.orc_e4m3_scaled.argtypes = [C.c_uint8]
        _lib.orc_dsa_score_fp8.restype = C.c_float
        _lib.orc_bm25_avgdl.restype = C.c_double
        _lib.orc_threshold_bitmap_f32.argtypes = [_P, _I, C.c_float, _P]
        _lib.orc_ip_topk_f32.argtypes = [_P, _I, _I, _P, _I, _I, C.c_float, _P, _P, _P]
    return _lib


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref() -> C.CDLL:
    global _ref
    if _ref is None:
        _ref = C.CDLL(REF_SO)
        for name in ("ref_topk_f32", "ref_threshold_f32", "ref_paged_kv_summary_f32",
                     "ref_dsa_topk", "ref_dsa_heads", "ref_bm25_query"):
            getattr(_ref, name).restype = _I
        for name in ("ref_flat_create_f32", "ref_flat_create_bf16", "ref_bm25_create"):
            getattr(_ref, name).restype = _P
        _ref.ref_threshold_f32.argtypes = [_P, _I, C.c_float, _P]
        _ref.ref_flat_pipeline.argtypes = [_P, _P, _I, _I, _I, C.c_float, C.c_int, _P, _P, _I,
                                           C.c_int]
        _ref.ref_flat_destroy.argtypes = [_P]
        _ref.ref_bm25_destroy.argtypes = [_P]
        _ref.ref_bm25_query.argtypes = [_P, _P, _I, _P]
    return _ref


def _p(a: np.ndarray):
    return a.ctypes.data_as(_P)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# ------------------------------------------------------------------ keys

def f32_key(x: float) -> int:
    return int(lib().orc_f32_key(float(x)))


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bits (finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return r.astype(np.uint16)


# ---------------------------------------------------------------- a-1..a-3

def ip_score_f32(mem, qry):
    mem = _c(mem, np.float32); qry = _c(np.atleast_2d(qry), np.float32)
    n, d = mem.shape if mem.size else (mem.shape[0], qry.shape[1])
    out = np.empty((qry.shape[0], n), np.float32)
    lib().orc_ip_score_f32(_p(mem), _I(n), _I(d), _p(qry), _I(qry.shape[0]), _p(out))
    return out


def ip_score_bf16(mem, qry):
    mem = _c(mem, np.uint16); qry = _c(np.atleast_2d(qry), np.uint16)
    n, d = mem.shape
    out = np.empty((qry.shape[0], n), np.float32)
    lib().orc_ip_score_bf16(_p(mem), _I(n), _I(d), _p(qry), _I(qry.shape[0]), _p(out))
    return out


def topk_f32(scores, k):
    s = _c(scores, np.float32)
    out = np.empty(k, np.int32)
    lib().orc_topk_f32(_p(s), _I(s.size), _I(k), _p(out))
    return out


def threshold_bitmap_f32(scores, thr):
    s = _c(scores, np.float32)
    out = np.empty((s.size + 63) // 64, np.uint64)
    lib().orc_threshold_bitmap_f32(_p(s), _I(s.size), float(thr), _p(out))
    return out


def ip_topk_f32(mem, qry, k, thr=None, want_scores=False):
    """Config-1 fused oracle: returns (idx [nq,k], bitmap [nq,words] or None, scores or None)."""
    mem = _c(mem, np.float32); qry = _c(np.atleast_2d(qry), np.float32)
    n, d = mem.shape[0], qry.shape[1]
    nq = qry.shape[0]
    idx = np.empty((nq, k), np.int32)
    bm = np.empty((nq, (n + 63) // 64), np.uint64) if thr is not None else None
    sc = np.empty((nq, n), np.float32) if want_scores else None
    lib().orc_ip_topk_f32(_p(mem), _I(n), _I(d), _p(qry), _I(nq), _I(k),
                          float(thr if thr is not None else 0.0), _p(idx),
                          _p(bm) if bm is not None else None,
                          _p(sc) if sc is not None else None)
    return idx, bm, sc


def set_threads(n: int) -> None:
    """OpenMP threads of the oracle's parallel loops."""
    lib().orc_set_threads(int(n))


def ip_topk_bf16(mem, qry, k, row_offset=0):
    mem = _c(mem, np.uint16); qry = _c(np.atleast_2d(qry), np.uint16)
    n, d = mem.shape
    nq = qry.shape[0]
    idx = np.empty((nq, k), np.int64)
    sc = np.empty((nq, k), np.float32)
    lib().orc_ip_topk_bf16(_p(mem), _I(n), _I(d), _p(qry), _I(nq), _I(k), _I(row_offset),
                           _p(idx), _p(sc))
    return idx, sc


def shard_merge_topk(cand_scores, cand_idx, k):
    cs = _c(cand_scores, np.float32); ci = _c(cand_idx, np.int64)
    n_shards, nq, kk = cs.shape
    assert kk == k
    out_s = np.empty((nq, k), np.float32)
    out_i = np.empty((nq, k), np.int64)
    lib().orc_shard_merge_topk(_p(cs), _p(ci), _I(n_shards), _I(nq), _I(k), _p(out_s), _p(out_i))
    return out_s, out_i


# -------------------------------------------------------------- a-5..a-7

def paged_kv_summary_f32(keys, weight, page_size):
    keys = _c(keys, np.float32); weight = _c(weight, np.float32)
    L, D = keys.shape if keys.size else (0, weight.shape[1] if weight.size else 0)
    out_dim = weight.shape[0] if weight.size else 0
    pages = (L + page_size - 1) // page_size if L else 0
    out = np.zeros((max(pages, 1), max(out_dim, 1)), np.float32)
    m = lib().orc_paged_kv_summary_f32(_p(keys), _I(L), _I(D), _p(weight), _I(out_dim),
                                       _I(page_size), _p(out))
    return out[:m, :out_dim]


def block_mean_f32(keys, page_size):
    keys = _c(keys, np.float32)
    L, D = keys.shape
    out = np.empty(((L + page_size - 1) // page_size, D), np.float32)
    lib().orc_block_mean_f32(_p(keys), _I(L), _I(D), _I(page_size), _p(out))
    return out


def block_minmax_f32(keys, page_size):
    """[pages][2][D]: per block the min row then the max row (MinMaxIndexMemory)."""
    keys = _c(keys, np.float32)
    L, D = keys.shape
    out = np.empty(((L + page_size - 1) // page_size, 2, D), np.float32)
    lib().orc_block_minmax_f32(_p(keys), _I(L), _I(D), _I(page_size), _p(out))
    return out


def block_select_minmax(q, minmax, top):
    """Top blocks by the min/max upper bound of q.k (-1 past the block count)."""
    q = _c(q, np.float32); mm = _c(minmax, np.float32)
    nb, _, D = mm.shape
    out = np.empty(top, np.int32)
    lib().orc_block_select_minmax(_p(q), _p(mm), _I(nb), _I(D), _I(top), _p(out))
    return out


def block_sparse_attention_f32(keys, values, blocks, q, page_size):
    keys = _c(keys, np.float32); values = _c(values, np.float32)
    blocks = _c(blocks, np.int32); q = _c(q, np.float32)
    L = keys.shape[0]
    D = q.shape[0]
    out = np.empty(D, np.float32)
    lib().orc_block_sparse_attention_f32(_p(keys), _p(values), _I(L), _I(D), _p(blocks),
                                         _I(blocks.size), _p(q), _I(page_size), _p(out))
    return out


def block_pages(page_table, seq, blocks, pages_per_block):
    pt = _c(page_table, np.int32); blocks = _c(blocks, np.int32)
    out = np.empty(blocks.size * pages_per_block, np.int32)
    m = lib().orc_block_pages(_p(pt), _I(pt.shape[1]), _I(seq), _p(blocks), _I(blocks.size),
                              _I(pages_per_block), _p(out))
    return out[:m]


# --------------------------------------------------------------- indexers

def dsa_indexer_i16(q, keys, w, topk):
    q = _c(q, np.int16); keys = _c(keys, np.int16); w = _c(w, np.float32)
    H, D = q.shape
    out = np.empty(topk, np.int32)
    sc = np.empty(topk, np.float32)
    lib().orc_dsa_indexer_i16(_p(q), _I(H), _I(D), _p(keys), _I(keys.shape[0]), _p(w), _I(topk),
                              _p(out), _p(sc))
    return out, sc


def e4m3_to_f32(v: np.ndarray) -> np.ndarray:
    v = np.asarray(v, np.uint8)
    table = np.array([lib().orc_e4m3_scaled(i) for i in range(256)], np.float64) * 2.0 ** -9
    return table[v].astype(np.float32)


def dsa_scores_fp8(q, keys, w, pos0):
    """Every exact FP8 indexer score [T, L] (-inf where not visible)."""
    q = _c(q, np.uint8); keys = _c(keys, np.uint8); w = _c(w, np.float32)
    T, H, D = q.shape
    L = keys.shape[0]
    out = np.empty((T, L), np.float32)
    lib().orc_dsa_scores_fp8(_p(q), _I(T), _I(H), _I(D), _p(keys), _I(L), _p(w), _I(pos0),
                             _p(out))
    return out


def dsa_indexer_fp8(q, keys, w, pos0, topk):
    q = _c(q, np.uint8); keys = _c(keys, np.uint8); w = _c(w, np.float32)
    T, H, D = q.shape
    out = np.empty((T, topk), np.int32)
    sc = np.empty((T, topk), np.float32)
    lib().orc_dsa_indexer_fp8(_p(q), _I(T), _I(H), _I(D), _p(keys), _I(keys.shape[0]), _p(w),
                              _I(pos0), _I(topk), _p(out), _p(sc))
    return out, sc


def lserve_topk_i16(past, queries, new_keys, topk=64, block=16):
    past = _c(past, np.int16); queries = _c(queries, np.int16); new_keys = _c(new_keys, np.int16)
    nq, D = queries.shape
    out = np.empty((nq, topk), np.int32)
    lib().orc_lserve_topk_i16(_p(past), _I(past.shape[0]), _p(queries), _p(new_keys), _I(nq),
                              _I(D), _I(topk), _I(block), _p(out))
    return out


def seer_budget_i16(past, queries, new_keys, topk=64):
    past = _c(past, np.int16); queries = _c(queries, np.int16); new_keys = _c(new_keys, np.int16)
    nq, D = queries.shape
    out = np.empty((nq, topk), np.int32)
    lib().orc_seer_budget_i16(_p(past), _I(past.shape[0]), _p(queries), _p(new_keys), _I(nq),
                              _I(D), _I(topk), _p(out))
    return out


def seer_words_per_query(L, nq):
    return int(lib().orc_seer_words_per_query(_I(L), _I(nq)))


def seer_threshold_i16(past, queries, new_keys, threshold):
    past = _c(past, np.int16); queries = _c(queries, np.int16); new_keys = _c(new_keys, np.int16)
    nq, D = queries.shape
    wpq = seer_words_per_query(past.shape[0], nq)
    out = np.empty((nq, wpq), np.uint64)
    lib().orc_seer_threshold_i16(_p(past), _I(past.shape[0]), _p(queries), _p(new_keys), _I(nq),
                                 _I(D), _I(threshold), _p(out))
    return out


def bm25_topk(term_ptr, post_doc, post_tf, doc_len, qterms, k):
    tp = _c(term_ptr, np.int64); pd = _c(post_doc, np.int32); pt = _c(post_tf, np.uint16)
    dl = _c(doc_len, np.int32); qt = _c(np.atleast_2d(qterms), np.int32)
    nq, qlen = qt.shape
    out = np.empty((nq, k), np.int32)
    sc = np.empty((nq, k), np.float64)
    lib().orc_bm25_topk(_p(tp), _p(pd), _p(pt), _I(tp.size - 1), _p(dl), _I(dl.size), _p(qt),
                        _I(nq), _I(qlen), _I(k), _p(out), _p(sc))
    return out, sc


def bm25_idf(term_ptr, n_docs):
    tp = _c(term_ptr, np.int64)
    out = np.empty(tp.size - 1, np.float64)
    lib().orc_bm25_idf(_p(tp), _I(tp.size - 1), _I(n_docs), _p(out))
    return out


def bm25_avgdl(doc_len):
    dl = _c(doc_len, np.int32)
    return float(lib().orc_bm25_avgdl(_p(dl), _I(dl.size)))


# ------------------------------------------- the reference's own CPU code

def ref_ip_score_f32(mem, q):
    mem = _c(mem, np.float32); q = _c(q, np.float32)
    out = np.empty(mem.shape[0], np.float32)
    ref().ref_ip_score_f32(_p(mem), _I(mem.shape[0]), _I(q.size), _p(q), _p(out))
    return out


def ref_topk_f32(scores, k):
    s = _c(scores, np.float32)
    out = np.full(k, -1, np.int32)
    m = ref().ref_topk_f32(_p(s), _I(s.size), _I(k), _p(out))
    return out[:m]


def ref_threshold_f32(scores, thr):
    s = _c(scores, np.float32)
    out = np.zeros((s.size + 63) // 64, np.uint64)
    ref().ref_threshold_f32(_p(s), _I(s.size), float(thr), _p(out))
    return out


class RefFlatMemory:
    """A reference FlatIndexMemory<float> held across calls (for timing)."""

    def __init__(self, mem, bf16=False):
        self.d = mem.shape[1]
        m = _c(mem, np.uint16 if bf16 else np.float32)
        fn = ref().ref_flat_create_bf16 if bf16 else ref().ref_flat_create_f32
        self.h = fn(_p(m), _I(m.shape[0]), _I(self.d))
        self.n = m.shape[0]

    def pipeline(self, queries, k, thr=None, n_threads=1):
        q = _c(np.atleast_2d(queries), np.float32)
        nq = q.shape[0]
        idx = np.empty((nq, k), np.int32)
        wpq = (self.n + 63) // 64
        words = np.empty((nq, wpq), np.uint64) if thr is not None else np.empty(1, np.uint64)
        ref().ref_flat_pipeline(self.h, _p(q), _I(nq), _I(self.d), _I(k),
                                float(thr if thr is not None else 0.0), int(thr is not None),
                                _p(idx), _p(words), _I(wpq), int(n_threads))
        return idx, (words if thr is not None else None)

    def close(self):
        if self.h:
            ref().ref_flat_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def ref_paged_kv_summary_f32(keys, weight, page_size):
    keys = _c(keys, np.float32); weight = _c(weight, np.float32)
    L, D = keys.shape
    out_dim = weight.shape[0]
    out = np.zeros((max((L + page_size - 1) // page_size, 1), out_dim), np.float32)
    m = ref().ref_paged_kv_summary_f32(_p(keys), _I(L), _I(D), _p(weight), _I(out_dim),
                                       _I(page_size), _p(out))
    return out[:m]


def ref_block_sparse_attention_f32(keys, values, blocks, q, page_size):
    keys = _c(keys, np.float32); values = _c(values, np.float32)
    blocks = _c(blocks, np.int32); q = _c(q, np.float32)
    out = np.empty(q.size, np.float32)
    ref().ref_block_sparse_attention_f32(_p(keys), _p(values), _I(keys.shape[0]), _I(q.size),
                                         _p(blocks), _I(blocks.size), _p(q), _I(page_size),
                                         _p(out))
    return out


def ref_paged_decode_f32(keys, values, q, block, topk):
    keys = _c(keys, np.float32); values = _c(values, np.float32); q = _c(q, np.float32)
    blocks = np.empty(topk, np.int32)
    out = np.empty(q.size, np.float32)
    ref().ref_paged_decode_f32(_p(keys), _p(values), _I(keys.shape[0]), _I(q.size), _p(q),
                               _I(block), _I(topk), _p(blocks), _p(out))
    return blocks, out


def ref_dsa_i16(q, keys, w):
    q = _c(q, np.int16); keys = _c(keys, np.int16); w = _c(w, np.float32)
    out = np.empty(int(ref().ref_dsa_topk()), np.int32)
    ref().ref_dsa_i16(_p(q), _p(keys), _I(keys.shape[0]), _p(w), _p(out))
    return out


def ref_lserve_i16(past, queries, new_keys):
    past = _c(past, np.int16); queries = _c(queries, np.int16); new_keys = _c(new_keys, np.int16)
    out = np.empty((queries.shape[0], 64), np.int32)
    ref().ref_lserve_i16(_p(past), _I(past.shape[0]), _p(queries), _p(new_keys),
                         _I(queries.shape[0]), _p(out))
    return out


def ref_seer_budget_i16(past, queries, new_keys):
    past = _c(past, np.int16); queries = _c(queries, np.int16); new_keys = _c(new_keys, np.int16)
    out = np.empty((queries.shape[0], 64), np.int32)
    ref().ref_seer_budget_i16(_p(past), _I(past.shape[0]), _p(queries), _p(new_keys),
                              _I(queries.shape[0]), _p(out))
    return out


def ref_seer_threshold_i16(past, queries, new_keys, threshold):
    past = _c(past, np.int16); queries = _c(queries, np.int16); new_keys = _c(new_keys, np.int16)
    nq = queries.shape[0]
    wpq = seer_words_per_query(past.shape[0], nq)
    out = np.empty((nq, wpq), np.uint64)
    ref().ref_seer_threshold_i16(_p(past), _I(past.shape[0]), _p(queries), _p(new_keys), _I(nq),
                                 _I(threshold), _I(wpq), _p(out))
    return out


class RefBM25:
    """The reference's BM25IndexMemory + FusedBM25Retrieval CPU kernel."""

    def __init__(self, term_ptr, post_doc, post_tf, n_docs):
        tp = _c(term_ptr, np.int64); pd = _c(post_doc, np.int32); pt = _c(post_tf, np.uint16)
        self.h = ref().ref_bm25_create(_p(tp), _p(pd), _p(pt), _I(tp.size - 1), _I(n_docs))

    def query(self, terms):
        t = _c(terms, np.int32)
        out = np.full(64, -1, np.int32)
        m = ref().ref_bm25_query(self.h, _p(t), _I(t.size), _p(out))
        return out[:m]

    def close(self):
        if self.h:
            ref().ref_bm25_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
