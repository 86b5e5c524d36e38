"""Readers of the reference's BM25 export files (heteromm_b200/bm25_export.py)
on files written in that format (tests/bm25_export_files.py): every array
they return, and the errors on damaged files."""
import os

import numpy as np
import pytest

from heteromm_b200 import bm25_export as E

from bm25_export_files import corpus, doc_major, term_major, write_export


@pytest.fixture()
def export(tmp_path):
    docs = corpus(5, 700, 50, empty_every=97)
    write_export(str(tmp_path), docs, 50)
    return str(tmp_path), docs


def test_readers_reproduce_the_arrays(export):
    d, docs = export
    dp, tr, ct = E.load_term_freq(os.path.join(d, "term_freq.bin"))
    dp0, tr0, ct0 = doc_major(docs)
    np.testing.assert_array_equal(dp, dp0)
    np.testing.assert_array_equal(tr, tr0)
    np.testing.assert_array_equal(ct, ct0)
    assert E.load_term_freq_num_docs(os.path.join(d, "term_freq.bin")) == 700
    tp, pd, pt = E.load_inverted_index(os.path.join(d, "inverted_index.bin"))
    tp0, pd0, pt0, _, df0 = term_major(docs, 50)
    np.testing.assert_array_equal(tp, tp0)
    np.testing.assert_array_equal(pd, pd0)
    np.testing.assert_array_equal(pt, pt0)
    np.testing.assert_array_equal(E.load_doc_freq(os.path.join(d, "doc_freq.bin")), df0)
    vm = E.load_vocab_mapping(os.path.join(d, "vocab_mapping.bin"))
    assert vm[1000] == 0 and vm[1049] == 49 and len(vm) == 50


def test_damaged_files_are_rejected(export, tmp_path):
    d, _ = export
    b = open(os.path.join(d, "term_freq.bin"), "rb").read()
    bad = tmp_path / "cut.bin"
    bad.write_bytes(b[:-4])                       # truncated
    with pytest.raises(ValueError):
        E.load_term_freq(str(bad))
    bad.write_bytes(b[:12] + b[20:28] + b[20:])   # offset table shifted
    with pytest.raises(ValueError):
        E.load_term_freq(str(bad))
    b = open(os.path.join(d, "doc_freq.bin"), "rb").read()
    bad.write_bytes(b + b"\0\0\0\0")
    with pytest.raises(ValueError):
        E.load_doc_freq(str(bad))
