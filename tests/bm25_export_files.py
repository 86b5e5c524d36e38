"""Writers of the reference's BM25 export files, restated from the format that
rag_test/export_bm25_data.py:13-27 documents (test infrastructure: they make
the fixtures the readers in heteromm_b200/bm25_export.py are checked on)."""
import os
import struct

import numpy as np


def corpus(seed: int, n_docs: int, n_vocab: int, empty_every: int = 0):
    """Per-document {vocab_idx: count} maps, terms ascending; every
    `empty_every`-th document empty."""
    rng = np.random.default_rng(seed)
    docs = []
    for d in range(n_docs):
        m = {}
        if not (empty_every and d % empty_every == 0):
            for t in rng.zipf(1.3, size=int(rng.integers(1, 30))):
                t = int(t) % n_vocab
                m[t] = m.get(t, 0) + int(rng.integers(1, 4))
        docs.append(dict(sorted(m.items())))
    return docs


def doc_major(docs):
    doc_ptr = np.zeros(len(docs) + 1, np.int64)
    doc_ptr[1:] = np.cumsum([len(d) for d in docs])
    terms = np.array([t for d in docs for t in d], np.int32)
    counts = np.array([c for d in docs for c in d.values()], np.uint32)
    return doc_ptr, terms, counts


def term_major(docs, n_vocab):
    """(term_ptr, post_doc, post_tf, doc_len, df): documents ascending within a term."""
    lists = [[] for _ in range(n_vocab)]
    for d, m in enumerate(docs):
        for t, c in m.items():
            lists[t].append((d, c))
    term_ptr = np.zeros(n_vocab + 1, np.int64)
    term_ptr[1:] = np.cumsum([len(x) for x in lists])
    post_doc = np.array([d for x in lists for d, _ in x], np.int32)
    post_tf = np.array([c for x in lists for _, c in x], np.uint16)
    doc_len = np.array([sum(m.values()) for m in docs], np.int32)
    return term_ptr, post_doc, post_tf, doc_len, np.diff(term_ptr).astype(np.uint32)


def _records(f, items):
    header = f.tell()
    offsets, cur = [], header + 8 * (len(items) + 1)
    for it in items:
        offsets.append(cur)
        cur += 4 + 8 * len(it)
    offsets.append(cur)
    f.write(struct.pack(f"<{len(offsets)}Q", *offsets))
    for it in items:
        f.write(struct.pack("<I", len(it)))
        for a, b in it:
            f.write(struct.pack("<II", a, b))


def write_export(out_dir: str, docs, n_vocab: int, token_ids=None):
    os.makedirs(out_dir, exist_ok=True)
    _, _, _, _, df = term_major(docs, n_vocab)
    with open(os.path.join(out_dir, "doc_freq.bin"), "wb") as f:
        f.write(struct.pack("<I", n_vocab))
        f.write(df.astype("<u4").tobytes())
    tok = token_ids if token_ids is not None else list(range(1000, 1000 + n_vocab))
    with open(os.path.join(out_dir, "vocab_mapping.bin"), "wb") as f:
        f.write(struct.pack("<I", n_vocab))
        for v in range(n_vocab):
            f.write(struct.pack("<II", tok[v], v))
    with open(os.path.join(out_dir, "term_freq.bin"), "wb") as f:
        f.write(struct.pack("<I", len(docs)))
        f.write(struct.pack("<Q", sum(len(d) for d in docs)))
        _records(f, [list(d.items()) for d in docs])
    lists = [[] for _ in range(n_vocab)]
    for d, m in enumerate(docs):
        for t, c in m.items():
            lists[t].append((d, c))
    with open(os.path.join(out_dir, "inverted_index.bin"), "wb") as f:
        f.write(struct.pack("<I", n_vocab))
        f.write(struct.pack("<Q", sum(len(x) for x in lists)))
        _records(f, lists)
