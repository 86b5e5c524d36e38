"""GPU parity of the int16 indexers (LServe block top-k, SeerAttention token
budget and threshold bitmap) against the oracle: bit-exact."""
import numpy as np
import pytest
import torch

import gen
import heteromm_b200 as hmm
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def inputs(seed, L, nq, D=128, lo=-100, hi=100):
    past = gen.ints(seed, (L, D), lo, hi).astype(np.int16)
    qq = gen.ints(seed + 1, (nq, D), lo, hi).astype(np.int16)
    nk = gen.ints(seed + 2, (nq, D), lo, hi).astype(np.int16)
    return past, qq, nk


def dev(cuda, *arrs):
    return [torch.from_numpy(np.ascontiguousarray(a)).to(cuda) for a in arrs]


CASES = [(1152, 16, -100, 100), (2000, 40, -100, 100), (1500, 9, -32768, 32767),
         (16384, 8, -100, 100), (0, 20, -100, 100)]


@pytest.mark.parametrize("L,nq,lo,hi", CASES)
def test_lserve(cuda, L, nq, lo, hi):
    past, qq, nk = inputs(700 + L, L, nq, lo=lo, hi=hi)
    out = hmm.lserve_topk_i16(*dev(cuda, past, qq, nk), 64, 16).cpu().numpy()
    assert np.array_equal(out, O.lserve_topk_i16(past, qq, nk, 64, 16))


@pytest.mark.parametrize("L,nq,lo,hi", CASES)
def test_seer_budget(cuda, L, nq, lo, hi):
    past, qq, nk = inputs(710 + L, L, nq, lo=lo, hi=hi)
    out = hmm.seer_budget_i16(*dev(cuda, past, qq, nk), 64).cpu().numpy()
    assert np.array_equal(out, O.seer_budget_i16(past, qq, nk, 64))


@pytest.mark.parametrize("L,nq,lo,hi", CASES)
@pytest.mark.parametrize("thr", [100000, 0, -5])
def test_seer_threshold(cuda, L, nq, lo, hi, thr):
    past, qq, nk = inputs(720 + L, L, nq, lo=lo, hi=hi)
    out = hmm.seer_threshold_i16(*dev(cuda, past, qq, nk), thr).cpu().numpy()
    ref = O.seer_threshold_i16(past, qq, nk, thr)
    assert np.array_equal(out.view(np.uint64), ref)


def test_ties_go_to_lowest_position(cuda):
    """Repeated key rows: equal scores must rank by lowest position / block."""
    past, qq, nk = inputs(730, 1300, 12)
    past = past[np.arange(1300) % 37]
    out_b = hmm.seer_budget_i16(*dev(cuda, past, qq, nk), 64).cpu().numpy()
    assert np.array_equal(out_b, O.seer_budget_i16(past, qq, nk, 64))
    out_l = hmm.lserve_topk_i16(*dev(cuda, past, qq, nk), 64, 16).cpu().numpy()
    assert np.array_equal(out_l, O.lserve_topk_i16(past, qq, nk, 64, 16))


@pytest.mark.parametrize("block", [8, 32])
def test_lserve_other_blocks(cuda, block):
    past, qq, nk = inputs(740, 1000, 10)
    out = hmm.lserve_topk_i16(*dev(cuda, past, qq, nk), 20, block).cpu().numpy()
    assert np.array_equal(out, O.lserve_topk_i16(past, qq, nk, 20, block))
