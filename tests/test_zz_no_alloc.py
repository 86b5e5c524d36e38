"""The allocation-free entry point hmm_ip_topk_f32_noalloc.

Some callers cannot allocate device memory - a host reached through an FFI
that only holds device pointers another runtime handed it, or a serving
process whose memory pool owns the device and forbids cudaMalloc while it
runs - so they cannot pass hmm_ip_topk_f32 its workspace.  This entry point
keeps its scratch in a fixed device array inside the library instead.  The
test calls it through the C ABI twice in a row (the second call runs on the
scratch the first one left behind) and checks each result against the
workspace-taking hmm_ip_topk_f32 on the same inputs: indices, scores and
threshold bitmaps must be bit-identical, the tolerance every other test of
this kernel uses.  The file is named to be collected last.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import gen
import heteromm_b200 as hmm
from heteromm_b200 import _abi

THR = float(np.float32(2.0 * np.sqrt(np.float32(128.0))))


def _noalloc(mem, qry, k, thr):
    lib = hmm.load()
    n, d = mem.shape
    nq = qry.shape[0]
    idx = torch.empty((nq, k), dtype=torch.int32, device=mem.device)
    sc = torch.empty((nq, k), dtype=torch.float32, device=mem.device)
    bm = torch.empty((nq, (n + 63) // 64), dtype=torch.int64, device=mem.device)
    st = lib.hmm_ip_topk_f32_noalloc(mem.data_ptr(), n, d, qry.data_ptr(), nq, k,
                                     idx.data_ptr(), sc.data_ptr(), C.c_float(thr),
                                     bm.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert st == 0, hmm.last_error()
    return idx, sc, bm


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point_twice(cuda):
    cases = [((65536, 128), 64, 64, 101), ((3000, 96), 7, 100, 202)]
    for (n, d), nq, k, seed in cases:
        mem = torch.from_numpy(gen.normal_f32(seed, (n, d))).to(cuda)
        qry = torch.from_numpy(gen.normal_f32(seed + 1, (nq, d))).to(cuda)
        got = _noalloc(mem, qry, k, THR)
        want = hmm.ip_topk_f32(mem, qry, k, THR)
        torch.cuda.synchronize()
        assert torch.equal(got[0], want[0])
        assert torch.equal(got[1].view(torch.int32), want[1].view(torch.int32))
        assert torch.equal(got[2], want[2])


def test_noalloc_rejects_oversize_problem():
    """Needs no device: the size check comes before any CUDA call."""
    lib = hmm.load()
    P = C.c_void_p(0x1000)
    need = lib.hmm_ip_topk_f32_workspace_size(1 << 30, 128, 4096, 256)
    assert need > (4 << 20)
    st = lib.hmm_ip_topk_f32_noalloc(P, 1 << 30, 128, P, 4096, 256, P, None, C.c_float(0.0),
                                     None, None)
    assert st == 6 and "fixed" in hmm.last_error()
