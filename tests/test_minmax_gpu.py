"""GPU parity of the min/max page summaries (MinMaxIndexMemory) of the paged
key cache and of the min/max-bound block selector against the oracle
(bit-exact), and of a decode step driven by that selector (attention within
the paged path's fp32 tolerance)."""
import numpy as np
import pytest
import torch

import gen
import heteromm_b200 as hmm
from oracle import oracle as O

from test_paged_gpu import ATOL, RTOL, T, dev_cache, make_cache

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n_seq,L,D,pt,block", [(3, 1000, 128, 16, 64), (2, 333, 64, 16, 24),
                                                (1, 64, 128, 16, 64), (2, 129, 256, 8, 16)])
def test_minmax_summaries_and_selection(cuda, n_seq, L, D, pt, block):
    keys, vals, kp, vp, table = make_cache(500 + L, n_seq, L, D, pt)
    dk, dv, dt = dev_cache(cuda, kp, vp, table)
    mm = hmm.paged_kv_minmax_bf16(dk, dt, L, block).cpu().numpy()
    q = gen.bf16_bits(gen.normal_f32(600 + L, (n_seq, D)))
    nb = (L + block - 1) // block
    for top in (1, 5, nb + 3):
        sel = hmm.block_select_minmax(T(q.view(np.int16), cuda), T(mm, cuda), top).cpu().numpy()
        for s in range(n_seq):
            ref = O.block_minmax_f32(O.bf16_to_f32(keys[s]), block)
            assert np.array_equal(mm[s], ref)
            assert np.array_equal(sel[s], O.block_select_minmax(O.bf16_to_f32(q[s]), ref, top))


def test_minmax_selected_decode(cuda):
    n_seq, L, D, pt, block, top = 4, 4096, 128, 16, 64, 8
    keys, vals, kp, vp, table = make_cache(911, n_seq, L, D, pt)
    dk, dv, dt = dev_cache(cuda, kp, vp, table)
    q = gen.bf16_bits(gen.normal_f32(912, (n_seq, D)))
    dq = T(q.view(np.int16), cuda)
    sel = hmm.block_select_minmax(dq, hmm.paged_kv_minmax_bf16(dk, dt, L, block), top)
    out = hmm.block_sparse_attention_bf16(dq, dk, dv, dt, L, block, sel).cpu().numpy()
    for s in range(n_seq):
        ref = O.block_sparse_attention_f32(O.bf16_to_f32(keys[s]), O.bf16_to_f32(vals[s]),
                                           sel[s].cpu().numpy(), O.bf16_to_f32(q[s]), block)
        np.testing.assert_allclose(out[s], ref, rtol=RTOL, atol=ATOL)
