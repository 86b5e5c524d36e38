"""The bounded-wait failure path of the tensor-core kernels, and the
asynchronous shard step.

Every pipeline wait inside tc_score_select_kernel and dsa_scores_kernel is
bounded; a wait that runs out makes its CTA let the copies and MMAs already in
flight complete, exit, and the entry point report HMM_ERR_TIMEOUT.  The test
hook hmm_debug_set_wait_limit_ns(0) makes the first wait that finds its stage
not yet ready give up, so these tests reach that path with no fault and no
hang; the next call with the default limit must then run normally."""
import time

import numpy as np
import pytest
import torch

import gen
import heteromm_b200 as hmm
from heteromm_b200 import _abi
from heteromm_b200.flat import check_status
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def dev(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


@pytest.fixture
def wait_limit_zero():
    _abi.set_wait_limit_ns(0)
    try:
        yield
    finally:
        _abi.set_wait_limit_ns(-1)


def flat_case(cuda, n=1 << 20, nq=16, seed=31):
    mem = gen.bf16_bits(gen.normal_f32(seed, (n, 128)))
    qry = gen.bf16_bits(gen.normal_f32(seed + 1, (nq, 128)))
    return mem, qry, dev(mem.view(np.int16), cuda), dev(qry.view(np.int16), cuda)


def test_flat_tc_timeout_then_clean_call(cuda):
    mem, qry, md, qd = flat_case(cuda)
    k = 100
    _abi.set_wait_limit_ns(0)
    try:
        t0 = time.monotonic()
        with pytest.raises(hmm.HmmError) as e:
            hmm.ip_topk_bf16(md, qd, k, 0)
        torch.cuda.synchronize()
        assert e.value.status == _abi.HMM_ERR_TIMEOUT
        assert time.monotonic() - t0 < 1.5       # gave up at once, far below the 2 s default
    finally:
        _abi.set_wait_limit_ns(-1)
    idx, sc = hmm.ip_topk_bf16(md, qd, k, 0)
    oidx, osc = O.ip_topk_bf16(mem, qry, k, 0)
    assert np.array_equal(idx.cpu().numpy(), oidx)
    assert np.array_equal(sc.cpu().numpy().view(np.uint32), osc.view(np.uint32))


def test_flat_tc_async_timeout_sets_status(cuda, wait_limit_zero):
    _, _, md, qd = flat_case(cuda, n=300000, nq=8, seed=33)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    hmm.ip_topk_bf16(md, qd, 50, 0, status=status)
    with pytest.raises(hmm.HmmError) as e:
        check_status(status)
    assert e.value.status == _abi.HMM_ERR_TIMEOUT


def test_flat_tc_async_equals_sync(cuda):
    """The asynchronous shard step (no host wait; status word checked once
    after several calls) returns the synchronous step's results bit for bit."""
    mem, qry, md, qd = flat_case(cuda, n=2_000_003, nq=256, seed=35)
    k = 100
    ref_i, ref_s = hmm.ip_topk_bf16(md, qd, k, 12345)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    outs = [hmm.ip_topk_bf16(md, qd, k, 12345, status=status) for _ in range(3)]
    check_status(status)
    for i, s in outs:
        assert torch.equal(i, ref_i)
        assert torch.equal(s.view(torch.int32), ref_s.view(torch.int32))
    oidx, osc = O.ip_topk_bf16(mem, qry[:16], k, 12345)   # a query subset against the oracle
    assert np.array_equal(ref_i[:16].cpu().numpy(), oidx)
    assert np.array_equal(ref_s[:16].cpu().numpy().view(np.uint32), osc.view(np.uint32))


def dsa_case(cuda, T=32, H=64, L=2048, seed=41):
    x = gen.normal_f32(seed, (T, H, 128))
    y = gen.normal_f32(seed + 1, (L, 128))
    q = gen.e4m3_bits(x * (448.0 / np.abs(x).max()))
    k = gen.e4m3_bits(y * (448.0 / np.abs(y).max()))
    w = gen.uniform01_f32(seed + 2, (T, H))
    return dev(q, cuda), dev(k, cuda), dev(w, cuda)


def test_dsa_timeout_then_clean_call(cuda):
    q, k, w = dsa_case(cuda)
    pos0, topk = 2048 - 32, 64
    ref_i, ref_s = hmm.dsa_indexer_fp8(q, k, w, pos0, topk)
    _abi.set_wait_limit_ns(0)
    try:
        t0 = time.monotonic()
        with pytest.raises(hmm.HmmError) as e:
            hmm.dsa_indexer_fp8(q, k, w, pos0, topk)
        torch.cuda.synchronize()
        assert e.value.status == _abi.HMM_ERR_TIMEOUT
        assert time.monotonic() - t0 < 1.5
    finally:
        _abi.set_wait_limit_ns(-1)
    i, s = hmm.dsa_indexer_fp8(q, k, w, pos0, topk)
    assert torch.equal(i, ref_i)
    assert torch.equal(s.view(torch.int32), ref_s.view(torch.int32))
