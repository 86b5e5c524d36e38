"""GPU parity of the flat score / select kernels against the CPU oracle
(bit-exact scores, indices and bitmaps), called through the C ABI."""
import numpy as np
import pytest
import torch

import gen
import heteromm_b200 as hmm
from oracle import oracle as O

pytestmark = pytest.mark.gpu

THR = float(np.float32(2.0 * np.sqrt(np.float32(128.0))))


def dev(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


@pytest.mark.parametrize("n,d,nq,k", [
    (3000, 128, 4, 64),       # golden shape
    (65536, 128, 64, 64),     # config 1, full size
    (1000, 37, 3, 10),        # dim not a multiple of 4, n not a multiple of 64
    (257, 64, 17, 256),       # k > n/2, a partial query group
    (50, 16, 2, 100),         # k > n
    # the one-CTA path for small memories (n <= 1024 rows, <= 64 queries) and its edges
    (1, 128, 1, 5),           # one row
    (512, 128, 1, 64),        # one (batch, head) of page summaries, one query
    (64, 8, 5, 64),           # k == n, short rows
    (1024, 128, 64, 256),     # largest n, largest query count, largest k
    (1025, 128, 64, 100),     # one row over: the multi-CTA path
    (1024, 128, 65, 10),      # one query over: the multi-CTA path
    (700, 3, 2, 9),           # dim below one vector load
])
def test_ip_topk_f32_matches_oracle(cuda, n, d, nq, k):
    mem = gen.normal_f32(1000 + n, (n, d))
    qry = gen.normal_f32(2000 + n, (nq, d))
    idx, sc, bm = hmm.ip_topk_f32(dev(mem, cuda), dev(qry, cuda), k, THR)
    torch.cuda.synchronize()
    oidx, obm, osc = O.ip_topk_f32(mem, qry, k, THR, want_scores=True)
    assert np.array_equal(idx.cpu().numpy(), oidx)
    assert np.array_equal(bm.cpu().numpy().view(np.uint64), obm)
    kk = min(k, n)
    got = sc.cpu().numpy()
    for q in range(nq):
        assert np.array_equal(got[q, :kk].view(np.uint32), osc[q][oidx[q, :kk]].view(np.uint32))
        assert np.all(np.isneginf(got[q, kk:]))


def test_golden_flat_fixture(cuda):
    import make_golden as mg
    g = np.load(gen.__file__.replace("gen.py", "flat_f32.npz"))
    mem, qry = mg.flat_inputs()
    idx, _, bm = hmm.ip_topk_f32(dev(mem, cuda), dev(qry, cuda), int(g["k"]), float(g["threshold"]))
    assert np.array_equal(idx.cpu().numpy(), g["idx"])
    assert np.array_equal(bm.cpu().numpy().view(np.uint64), g["bitmap"])
    s = hmm.ip_score_f32(dev(mem, cuda), dev(qry, cuda)).cpu().numpy()
    assert np.array_equal(s.view(np.uint32), g["scores"].view(np.uint32))


def test_score_api_bit_exact(cuda):
    mem = gen.normal_f32(11, (4099, 130))
    qry = gen.normal_f32(12, (5, 130))
    s = hmm.ip_score_f32(dev(mem, cuda), dev(qry, cuda)).cpu().numpy()
    assert np.array_equal(s.view(np.uint32), O.ip_score_f32(mem, qry).view(np.uint32))


def test_topk_and_threshold_on_device_scores(cuda):
    import make_golden as mg
    g = np.load(gen.__file__.replace("gen.py", "topk_edge.npz"))
    s = mg.topk_edge_inputs()
    s[5] = np.nan
    for k in (1, 64, 4096):
        idx, sc = hmm.topk_f32(dev(s[None], cuda), k)
        assert np.array_equal(idx.cpu().numpy()[0], O.topk_f32(s, k))
    bm = hmm.threshold_bitmap_f32(dev(s[None], cuda), 0.0).cpu().numpy()[0].view(np.uint64)
    assert np.array_equal(bm, O.threshold_bitmap_f32(s, 0.0))
    assert np.array_equal(hmm.topk_f32(dev(s[None], cuda), 64)[0].cpu().numpy()[0][:0], g["idx64"][:0])


def test_ties_nan_and_signed_zero(cuda):
    mem = np.zeros((300, 8), np.float32)
    mem[::7, 0] = 1.0          # equal scores on every 7th row
    mem[3, 0] = np.nan         # NaN ranks last
    mem[4, 0] = -0.0
    qry = np.ones((1, 8), np.float32)
    idx, sc, bm = hmm.ip_topk_f32(dev(mem, cuda), dev(qry, cuda), 60, 0.0)
    oidx, obm, _ = O.ip_topk_f32(mem, qry, 60, 0.0)
    assert np.array_equal(idx.cpu().numpy(), oidx)
    assert np.array_equal(bm.cpu().numpy().view(np.uint64), obm)


def test_ties_nan_small_bf16(cuda):
    """bf16 rows on the one-CTA path: ties to the lower row, NaN last."""
    mem = np.zeros((200, 128), np.float32)
    mem[::5, 0] = 1.0
    mem[7, 0] = np.nan
    mem = gen.bf16_bits(mem)
    qry = gen.bf16_bits(np.ones((2, 128), np.float32))
    idx, sc = hmm.ip_topk_bf16(dev(mem.view(np.int16), cuda), dev(qry.view(np.int16), cuda), 50, 0)
    oidx, osc = O.ip_topk_bf16(mem, qry, 50, 0)
    assert np.array_equal(idx.cpu().numpy(), oidx)
    assert np.array_equal(sc.cpu().numpy().view(np.uint32), osc.view(np.uint32))


def test_empty_memory(cuda):
    mem = torch.empty((0, 16), dtype=torch.float32, device=cuda)
    qry = torch.ones((2, 16), dtype=torch.float32, device=cuda)
    idx, sc, bm = hmm.ip_topk_f32(mem, qry, 5, 0.0)
    assert (idx.cpu() == -1).all() and torch.isneginf(sc.cpu()).all()
    assert bm.numel() == 0


@pytest.mark.parametrize("n,nq,k,off", [(20000, 16, 100, 0), (7777, 33, 100, 123456789),
                                        (600, 3, 100, 77), (1024, 64, 256, 0)])
def test_ip_topk_bf16_matches_oracle(cuda, n, nq, k, off):
    mem = gen.bf16_bits(gen.normal_f32(31 + n, (n, 128)))
    qry = gen.bf16_bits(gen.normal_f32(32 + n, (nq, 128)))
    idx, sc = hmm.ip_topk_bf16(dev(mem.view(np.int16), cuda), dev(qry.view(np.int16), cuda), k, off)
    oidx, osc = O.ip_topk_bf16(mem, qry, k, off)
    assert np.array_equal(idx.cpu().numpy(), oidx)
    assert np.array_equal(sc.cpu().numpy().view(np.uint32), osc.view(np.uint32))


def test_shard_merge_matches_oracle(cuda):
    n, nq, k, shards = 12000, 8, 100, 4
    mem = gen.bf16_bits(gen.normal_f32(41, (n, 128)))
    qry = gen.bf16_bits(gen.normal_f32(42, (nq, 128)))
    per = n // shards
    cs, ci = [], []
    for s in range(shards):
        i, v = hmm.ip_topk_bf16(dev(mem[s * per:(s + 1) * per].view(np.int16), cuda),
                                dev(qry.view(np.int16), cuda), k, s * per)
        cs.append(v); ci.append(i)
    ms, mi = hmm.shard_merge_topk(torch.stack(cs), torch.stack(ci), k)
    oidx, osc = O.ip_topk_bf16(mem, qry, k, 0)
    assert np.array_equal(mi.cpu().numpy(), oidx)
    assert np.array_equal(ms.cpu().numpy().view(np.uint32), osc.view(np.uint32))
    # and the host merge oracle agrees on the gathered candidates
    os_, oi = O.shard_merge_topk(torch.stack(cs).cpu().numpy(), torch.stack(ci).cpu().numpy(), k)
    assert np.array_equal(oi, oidx)


def test_deterministic_repeat(cuda):
    mem = dev(gen.normal_f32(51, (65536, 128)), cuda)
    qry = dev(gen.normal_f32(52, (64, 128)), cuda)
    a = hmm.ip_topk_f32(mem, qry, 64, THR)
    b = hmm.ip_topk_f32(mem, qry, 64, THR)
    for x, y in zip(a, b):
        assert torch.equal(x, y)


def test_varying_k_across_entry_points(cuda):
    """A small-k top-k call must not shrink the merge kernel's shared-memory
    limit for a later call with a larger k."""
    s = dev(gen.normal_f32(61, (1, 5000)), cuda)
    hmm.topk_f32(s, 64)
    mem = gen.normal_f32(62, (3000, 96))
    qry = gen.normal_f32(63, (7, 96))
    idx, _, _ = hmm.ip_topk_f32(dev(mem, cuda), dev(qry, cuda), 200, THR)
    assert np.array_equal(idx.cpu().numpy(), O.ip_topk_f32(mem, qry, 200, THR)[0])
