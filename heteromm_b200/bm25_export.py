"""Readers of the reference's BM25 export files (toolchain/rag_test/
export_bm25_data.py:13-27, 180-330), all little-endian:

  doc_freq.bin       [u32 num_vocab] [u32 df] * num_vocab
  vocab_mapping.bin  [u32 num_vocab] [u32 token_id, u32 vocab_idx] * num_vocab
  term_freq.bin      [u32 num_docs] [u64 total_entries] [u64 byte offset] * (num_docs + 1),
                     then per document [u32 n] [u32 vocab_idx, u32 count] * n
  inverted_index.bin [u32 num_vocab] [u64 total_postings] [u64 byte offset] * (num_vocab + 1),
                     then per term [u32 n] [u32 doc_id, u32 tf] * n

Each reader returns NumPy arrays in the CSR form the BM25 kernels take; the
variable-length records are parsed with array operations (one pass over the
file), not a Python loop.
"""
from __future__ import annotations

import numpy as np


def _read(path: str) -> bytes:
    with open(path, "rb") as f:
        return f.read()


def load_doc_freq(path: str) -> np.ndarray:
    """df [num_vocab] uint32, indexed by vocabulary index."""
    b = _read(path)
    n = int(np.frombuffer(b, "<u4", 1, 0)[0])
    if len(b) != 4 + 4 * n:
        raise ValueError(f"{path}: size {len(b)} does not match {n} entries")
    return np.frombuffer(b, "<u4", n, 4).copy()


def load_vocab_mapping(path: str) -> dict:
    """{token_id: vocab_idx}: how query tokens map to the index's terms."""
    b = _read(path)
    n = int(np.frombuffer(b, "<u4", 1, 0)[0])
    if len(b) != 4 + 8 * n:
        raise ValueError(f"{path}: size {len(b)} does not match {n} entries")
    pairs = np.frombuffer(b, "<u4", 2 * n, 4).reshape(n, 2)
    return dict(zip(pairs[:, 0].tolist(), pairs[:, 1].tolist()))


def _records(b: bytes, n_items: int, header: int, path: str):
    """(ptr [n_items+1] int64, first [m], second [m]) of the per-item
    [u32 n] [u32 a, u32 b] * n records that the byte-offset table after
    `header` bytes points at."""
    offsets = np.frombuffer(b, "<u8", n_items + 1, header).astype(np.int64)
    data0 = header + 8 * (n_items + 1)
    if n_items and (offsets[0] != data0 or offsets[-1] != len(b) or np.any(np.diff(offsets) < 4)):
        raise ValueError(f"{path}: inconsistent offset table")
    words = np.frombuffer(b, "<u4", (len(b) - data0) // 4, data0)
    first_word = (offsets[:-1] - data0) // 4          # each record's [u32 n]
    counts = words[first_word].astype(np.int64)
    if np.any(4 + 8 * counts != np.diff(offsets)):
        raise ValueError(f"{path}: a record's length disagrees with its offsets")
    ptr = np.zeros(n_items + 1, np.int64)
    np.cumsum(counts, out=ptr[1:])
    keep = np.ones(words.size, bool)
    keep[first_word] = False                          # drop the [u32 n] words
    pairs = words[keep].reshape(-1, 2)
    return ptr, pairs[:, 0], pairs[:, 1]


def load_term_freq(path: str):
    """Per-document term counts: (doc_ptr [num_docs+1] int64, terms int32
    (vocabulary index), counts uint32), document d owning
    [doc_ptr[d], doc_ptr[d+1])."""
    b = _read(path)
    n_docs = int(np.frombuffer(b, "<u4", 1, 0)[0])
    total = int(np.frombuffer(b, "<u8", 1, 4)[0])
    ptr, vocab, count = _records(b, n_docs, 12, path)
    if int(ptr[-1]) != total:
        raise ValueError(f"{path}: {int(ptr[-1])} entries, header says {total}")
    return ptr, vocab.astype(np.int32), count.astype(np.uint32)


def load_term_freq_num_docs(path: str) -> int:
    """The document count in term_freq.bin's header."""
    with open(path, "rb") as f:
        return int(np.frombuffer(f.read(4), "<u4", 1, 0)[0])


def load_inverted_index(path: str):
    """Term-major postings: (term_ptr [num_vocab+1] int64, post_doc int32,
    post_tf uint16); tf above 65535 is rejected."""
    b = _read(path)
    n_vocab = int(np.frombuffer(b, "<u4", 1, 0)[0])
    total = int(np.frombuffer(b, "<u8", 1, 4)[0])
    ptr, doc, tf = _records(b, n_vocab, 12, path)
    if int(ptr[-1]) != total:
        raise ValueError(f"{path}: {int(ptr[-1])} postings, header says {total}")
    if tf.size and int(tf.max()) > 65535:
        raise ValueError(f"{path}: a term frequency exceeds 65535")
    return ptr, doc.astype(np.int32), tf.astype(np.uint16)
