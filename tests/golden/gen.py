"""Deterministic synthetic inputs for the parity tests and golden fixtures.

A counter-based splitmix64 stream drives every generator, so the same seed
gives the same bits on any machine and numpy version.  `normal_f32` is the
sum of three uniforms on [-1, 1) (mean 0, variance 1), computed in float64
and rounded once to float32.
"""
from __future__ import annotations

import numpy as np

_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)
_G = np.uint64(0x9E3779B97F4A7C15)


def splitmix64(seed: int, n: int, offset: int = 0) -> np.ndarray:
    with np.errstate(over="ignore"):
        x = (np.arange(offset, offset + n, dtype=np.uint64) + np.uint64(1)) * _G
        x = x + np.uint64(seed & 0xFFFFFFFFFFFFFFFF) * np.uint64(0xD1B54A32D192ED03)
        x = (x ^ (x >> np.uint64(30))) * _M1
        x = (x ^ (x >> np.uint64(27))) * _M2
        x = x ^ (x >> np.uint64(31))
    return x


def uniform_f64(seed: int, n: int) -> np.ndarray:
    """Uniform on [-1, 1) with 2^-23 resolution."""
    u = (splitmix64(seed, n) >> np.uint64(40)).astype(np.int64)
    return (u - (1 << 23)).astype(np.float64) / float(1 << 23)


def normal_f32(seed: int, shape) -> np.ndarray:
    n = int(np.prod(shape))
    s = uniform_f64(seed, n) + uniform_f64(seed + 0x1000, n) + uniform_f64(seed + 0x2000, n)
    return s.astype(np.float32).reshape(shape)


def ints(seed: int, shape, lo: int, hi: int) -> np.ndarray:
    """Uniform integers in [lo, hi] (inclusive)."""
    n = int(np.prod(shape))
    r = splitmix64(seed, n) % np.uint64(hi - lo + 1)
    return (r.astype(np.int64) + lo).reshape(shape)


def uniform01_f32(seed: int, shape) -> np.ndarray:
    n = int(np.prod(shape))
    u = (splitmix64(seed, n) >> np.uint64(40)).astype(np.float64) / float(1 << 24)
    return u.astype(np.float32).reshape(shape)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns, round to nearest even."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + np.uint64(0x7FFF) + ((u >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)).astype(np.uint16)


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.asarray(h, np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def e4m3_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> OCP e4m3 bit patterns, round to nearest even, saturating to +-448."""
    x = np.asarray(x, np.float64)
    # enumerate the 127 non-negative finite e4m3 values
    vals = []
    for code in range(0x7F):
        e, m = code >> 3, code & 7
        vals.append(m * 2.0 ** -9 if e == 0 else (1 + m / 8) * 2.0 ** (e - 7))
    vals = np.array(vals)
    a = np.minimum(np.abs(x), 448.0)
    i = np.searchsorted(vals, a)            # vals[i-1] < a <= vals[i]
    i = np.clip(i, 1, len(vals) - 1)
    lo, hi = vals[i - 1], vals[i]
    pick_hi = (a - lo > hi - a) | ((a - lo == hi - a) & (i % 2 == 0))
    code = np.where(pick_hi, i, i - 1)
    code = np.where(a == 0, 0, code)
    sign = (x < 0) & (code != 0)
    return (code | (sign.astype(np.int64) << 7)).astype(np.uint8)


def bm25_corpus(seed: int, n_docs: int, vocab: int, mean_len: float, zipf_s: float = 1.1):
    """Synthetic corpus as a CSR inverted index: term ids ~ Zipf(s) over the
    vocabulary, document lengths ~ Poisson(mean_len) (at least 1).
    Returns (term_ptr int64 [vocab+1], post_doc int32, post_tf uint16, doc_len int32)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    ranks = np.arange(1, vocab + 1, dtype=np.float64)
    p = ranks ** -zipf_s
    p /= p.sum()
    lens = np.maximum(rng.poisson(mean_len, n_docs), 1)
    toks = rng.choice(vocab, size=int(lens.sum()), p=p)
    doc = np.repeat(np.arange(n_docs, dtype=np.int64), lens)
    key = toks.astype(np.int64) * n_docs + doc
    uk, tf = np.unique(key, return_counts=True)
    term = (uk // n_docs).astype(np.int64)
    pdoc = (uk % n_docs).astype(np.int32)
    term_ptr = np.zeros(vocab + 1, np.int64)
    np.add.at(term_ptr, term + 1, 1)
    term_ptr = np.cumsum(term_ptr)
    doc_len = np.zeros(n_docs, np.int64)
    np.add.at(doc_len, pdoc, tf)
    return term_ptr, pdoc, tf.astype(np.uint16), doc_len.astype(np.int32)


def bm25_queries(seed: int, nq: int, qlen: int, vocab: int, zipf_s: float = 1.1) -> np.ndarray:
    """nq queries of qlen distinct Zipf-drawn term ids."""
    rng = np.random.Generator(np.random.PCG64(seed))
    ranks = np.arange(1, vocab + 1, dtype=np.float64)
    p = ranks ** -zipf_s
    p /= p.sum()
    out = np.empty((nq, qlen), np.int32)
    for q in range(nq):
        seen: list = []
        while len(seen) < qlen:
            t = int(rng.choice(vocab, p=p))
            if t not in seen:
                seen.append(t)
        out[q] = seen
    return out
