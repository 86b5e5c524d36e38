"""Benchmark of the HeteroMM score -> select path on B200.

Workload (default): sharded flat retrieval — 64Mi rows x d=128 bf16 ~N(0,1)
(16 GiB) split by contiguous row ranges over N GPUs, 256 bf16 queries,
fp32-accumulated inner products, per-shard top-100, NCCL all-gather of the
(score, global index) candidates and a final merge to the global top-100.

One step = one pass of the hot path over the whole memory for the batch of
256 queries.  `value` is device-timed whole-job throughput in row-query
pairs per second (rows x queries / step time, max over ranks), with the
memory already resident in HBM.  `e2e` is the same step through the public
API with the queries copied from pinned host memory and the top-100 results
read back to the host inside the timed region.

The default run also measures, after the headline, a sustained loop of the
same step (at least --sustain-s seconds, with its own clock record), checks
16 of the 256 queries bit for bit against the oracle over all 64Mi rows, and
nests one entry per other workload under "configs": the flat fp32 top-k +
threshold at one and at 64 queries (65,536 x 128), the paged-KV block-sparse
decode, BM25 top-10 over 1M documents and the FP8 DSA indexer, each with its
roofline, a CPU baseline on the same workload and a parity sample.

Usage:
  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  python -m torch.distributed.run --nproc-per-node N bench.py --gpus N ...
  python bench.py --config flat|flat_f32|paged|bm25|dsa   # one workload alone
  python bench.py --rows 4194304 --no-cpu-baseline   # smaller case for ncu captures

The roofline is the tensor pipe: 2 x rows x 128 x 256 = 4.40 TFLOP per step
against 16 GiB of HBM reads, i.e. 2.67 ms at the measured burst bf16 rate
versus 2.6 ms at the measured copy bandwidth.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

N_ROWS = 64 * 1024 * 1024
DIM = 128
N_QUERIES = 256
TOP_K = 100
CHUNK = 1 << 20               # rows per generator chunk (seeded independently)
SEED_MEM = 12
SEED_QRY = 13
METRIC = "score+top-k rows/s (row-query pairs per second)"
WORKLOAD = "sharded flat retrieval: 64Mi x 128 bf16 rows, 256 queries, top-100"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


def init_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        from heteromm_b200 import shard as sharding
        # non-blocking communicators: a stalled peer can be abandoned by an abort
        # (heteromm_b200.shard.wait_with_deadline) instead of blocking the host
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local),
                                             pg_options=sharding.nccl_options(nonblocking=True))
    else:
        torch.cuda.set_device(local)
    return rank, world, local


def gen_rows(start: int, count: int, device) -> torch.Tensor:
    """Rows [start, start+count) of the synthetic memory, bf16.  Every 1Mi-row
    chunk has its own seed, so a row's values do not depend on the sharding."""
    out = torch.empty((count, DIM), dtype=torch.bfloat16, device=device)
    g = torch.Generator(device=device)
    r = start
    while r < start + count:
        c0 = r // CHUNK
        c_lo, c_hi = c0 * CHUNK, (c0 + 1) * CHUNK
        lo, hi = max(r, c_lo), min(start + count, c_hi)
        g.manual_seed(SEED_MEM * 1000003 + c0)
        chunk = torch.randn((CHUNK, DIM), generator=g, device=device, dtype=torch.float32)
        out[lo - start:hi - start] = chunk[lo - c_lo:hi - c_lo].to(torch.bfloat16)
        r = hi
    return out


def gen_queries(device) -> torch.Tensor:
    g = torch.Generator(device=device)
    g.manual_seed(SEED_QRY)
    return torch.randn((N_QUERIES, DIM), generator=g, device=device).to(torch.bfloat16)


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        self.out = ""
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out = ""

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in (self.out or "").splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for n, v in zip(names, parts[3:7]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def run_ours(args, rank, world, local):
    import heteromm_b200 as hmm
    from heteromm_b200 import _abi

    from heteromm_b200 import shard as sharding
    from heteromm_b200.flat import check_status
    dev = torch.device("cuda", local)
    hmm.load()
    r0, r1 = sharding.shard_range(N_ROWS, rank, world)
    per = r1 - r0
    shard = gen_rows(r0, per, dev)
    qry = gen_queries(dev)
    shard_i16 = shard.view(torch.int16)
    qry_i16 = qry.view(torch.int16)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    torch.cuda.synchronize()

    stream = torch.cuda.current_stream()

    def step(q_i16):
        # local tensor-core top-k of this rank's rows (no host wait: timeout and
        # pool-overflow flags go to `status`, checked after each loop), NCCL
        # all-gather of the candidates, merge
        return sharding.sharded_ip_topk_bf16(shard_i16, q_i16, TOP_K, r0, status=status)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        step(qry_i16)
    barrier()
    check_status(status)

    # ---- device-resident timing (value) + dominant-kernel timing (roofline)
    # The library brackets each launch of its scoring kernel with CUDA events
    # on the launching stream (hmm_profile_enable); its launch counter gives
    # the number of kernels this library started inside the timed region.
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _abi.profile_read()
    _abi.profile_enable(True)
    with ClockSampler(local) as clk:
        barrier()
        l0 = _abi.kernel_launches()
        ev0.record(stream)
        for i in range(args.steps):
            step(qry_i16)
        ev1.record(stream)
        barrier()
        launches = _abi.kernel_launches() - l0
    _abi.profile_enable(False)
    k_total, k_n = _abi.profile_read()
    check_status(status)
    ms = max_over_ranks(ev0.elapsed_time(ev1)) / args.steps
    kern_ms = max_over_ranks(k_total / args.steps)   # per step, all its launches

    # ---- sustained: the same step back to back for >= sustain_s seconds (the
    # step count is fixed on rank 0 from the timed region and shared), so the
    # clock sampler sees the GPU settle under its power cap
    n_sus = max(args.steps, int(args.sustain_s * 1e3 / max(ms, 1e-3)) + 1)
    if world > 1:
        t = torch.tensor([n_sus], dtype=torch.int64, device=dev)
        torch.distributed.broadcast(t, 0)
        n_sus = int(t.item())
    _abi.profile_enable(True)
    with ClockSampler(local) as clk_sus:
        barrier()
        ev0.record(stream)
        for i in range(n_sus):
            step(qry_i16)
        ev1.record(stream)
        barrier()
    _abi.profile_enable(False)
    ks_total, _ = _abi.profile_read()
    check_status(status)
    sus_ms = max_over_ranks(ev0.elapsed_time(ev1)) / n_sus
    sus_kern_ms = max_over_ranks(ks_total / n_sus)

    # ---- end to end through the public API: pinned host queries in, results
    # out, inside the timed region
    q_host = qry_i16.cpu().pin_memory()
    out_i = torch.empty((N_QUERIES, TOP_K), dtype=torch.int64).pin_memory()
    out_s = torch.empty((N_QUERIES, TOP_K), dtype=torch.float32).pin_memory()
    q_dev = torch.empty_like(qry_i16)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        q_dev.copy_(q_host, non_blocking=True)
        # the user-facing call bounds the exchange by a host deadline: a rank
        # that never contributes ends the call with HMM_ERR_TIMEOUT
        idx, sc = sharding.sharded_ip_topk_bf16(shard_i16, q_dev, TOP_K, r0, status=status,
                                                deadline_s=args.exchange_deadline_s)
        out_i.copy_(idx, non_blocking=True)
        out_s.copy_(sc, non_blocking=True)
    e1.record(stream)
    barrier()
    check_status(status)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1)) / args.steps

    # sanity of the final answer: valid global indices, scores best first
    ok = bool((out_i >= 0).all() and (out_i < N_ROWS).all() and
              (out_s[:, :-1] >= out_s[:, 1:]).all())
    del shard, shard_i16
    torch.cuda.empty_cache()

    result = None
    if rank == 0:
        pk, pk_kind = peaks()
        # algorithmic work of one scoring-kernel launch: 2 x rows x dim FLOP per
        # query over this rank's shard (the scoring pass reads every row once;
        # the short sample pass before it is not counted as algorithmic work)
        flop = 2.0 * per * DIM * N_QUERIES
        achieved = flop / (kern_ms * 1e-3) / 1e12
        peak_t = pk["bf16_tflops"]
        hbm_gbs = (per * DIM * 2 + N_QUERIES * DIM * 2) / (kern_ms * 1e-3) / 1e9
        sus_achieved = flop / (sus_kern_ms * 1e-3) / 1e12
        peak_sus = pk.get("bf16_tflops_sustained", pk["bf16_tflops"])
        value = N_ROWS * N_QUERIES / (ms * 1e-3)
        result = {
            "metric": METRIC,
            "value": value,
            "unit": "rows*queries/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded N(0,1), generated on device per 1Mi-row chunk)",
            "config": {"workload": WORKLOAD, "rows": N_ROWS, "dim": DIM, "queries": N_QUERIES,
                       "top_k": TOP_K, "parallelism": f"row-shard x{world} + NCCL all-gather",
                       "l2": "inputs larger than L2 (shard >= 2 GiB vs 126 MB L2)"},
            "e2e": {"value": N_ROWS * N_QUERIES / (e2e_ms * 1e-3), "unit": "rows*queries/s",
                    "ms_per_step": e2e_ms, "h2d_bytes_per_step": N_QUERIES * DIM * 2,
                    "d2h_bytes_per_step": N_QUERIES * TOP_K * (8 + 4)},
            "gpu_launches": launches,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_t,
                         "unit": "TFLOP/s", "frac": achieved / peak_t,
                         "traffic": traffic_per_launch("tc_score_select_kernel", per),
                         "kernel": "tc_score_select_kernel<0> (the scoring pass)",
                         "kernel_ms": kern_ms,
                         "kernel_launches_per_step": k_n / args.steps,
                         "peak_kind": f"{pk_kind} bf16 burst (cuBLAS 8192^3, best of 10): the "
                                      f"timed region is {ms * args.steps:.0f} ms",
                         "hbm_gbs_achieved": hbm_gbs,
                         "hbm_frac": hbm_gbs / pk["hbm_gbs"]},
            "sustained": {"steps": n_sus, "seconds": sus_ms * n_sus * 1e-3,
                          "ms_per_step": sus_ms,
                          "value": N_ROWS * N_QUERIES / (sus_ms * 1e-3),
                          "kernel_ms": sus_kern_ms, "achieved": sus_achieved,
                          "peak": peak_sus, "unit": "TFLOP/s", "frac": sus_achieved / peak_sus,
                          "peak_kind": f"{pk_kind} bf16 sustained (cuBLAS, 4 s loop)",
                          "clocks": clk_sus.summary()},
            "clocks": clk.summary(),
            "sanity": ok,
        }
    # exact results of a query subset against the oracle over every row
    par = flat_parity(out_i, out_s, world, rank, dev)
    if rank == 0:
        result["parity"] = par
        if world == 1 and not args.no_cpu_baseline:
            result["cpu_baseline"] = cpu_baseline(dev)
    return result


def flat_parity(out_i, out_s, world, rank, dev, n_check: int = 16):
    """Compares the final top-100 of `n_check` of the 256 queries (spread over
    the batch) with the oracle's exact top-100 over all rows, bit for bit.  Rank
    0 regenerates the rows chunk by chunk (the generator is per 1Mi-row chunk,
    so the rows equal every rank's shards), runs the oracle on each 8Mi-row
    piece with its row offset and merges the pieces' candidates."""
    if rank != 0:
        return None
    import numpy as np

    from oracle import oracle as O
    O.set_threads(os.cpu_count() or 1)   # rank 0 alone runs it while the others wait
    pick = np.arange(0, N_QUERIES, N_QUERIES // n_check)
    qh = gen_queries(dev).view(torch.int16).cpu().numpy().view(np.uint16)[pick]
    piece = 8 * CHUNK
    cand_s, cand_i = [], []
    t0 = time.perf_counter()
    for p0 in range(0, N_ROWS, piece):
        cnt = min(piece, N_ROWS - p0)
        rows = gen_rows(p0, cnt, dev).view(torch.int16).cpu().numpy().view(np.uint16)
        i, s = O.ip_topk_bf16(rows, qh, TOP_K, p0)
        cand_i.append(i)
        cand_s.append(s)
    ws, wi = O.shard_merge_topk(np.stack(cand_s), np.stack(cand_i), TOP_K)
    gi = out_i.numpy()[pick]
    gs = out_s.numpy()[pick]
    equal = bool(np.array_equal(gi, wi) and np.array_equal(gs.view(np.uint32), ws.view(np.uint32)))
    return {"checked_queries": int(pick.size), "rows": N_ROWS, "equal": equal,
            "against": "oracle exact top-100 over every row (bit-exact indices and scores)",
            "seconds": time.perf_counter() - t0}


def cpu_baseline(dev, sample_rows: int = 1 << 20, sample_queries: int = 16):
    """The reference's own InnerProductCompute -> TopKRetrieval(100) pipeline
    (oracle/_ref, KernelType::CPU) on a bounded sample: the first 1Mi rows of
    the same memory and 16 of the queries, one query per host thread."""
    from oracle import oracle as O
    rows = gen_rows(0, sample_rows, dev).view(torch.int16).cpu().numpy().view("uint16")
    qry = gen_queries(dev)
    q = qry[:sample_queries].float().cpu().numpy()
    threads = os.cpu_count() or 1
    if O.ref_available():
        mem = O.RefFlatMemory(rows, bf16=True)
        t = time.perf_counter()
        mem.pipeline(q, TOP_K, None, n_threads=threads)
        dt = time.perf_counter() - t
        mem.close()
        kind = "reference"
    else:
        t = time.perf_counter()
        O.ip_topk_bf16(rows, qry[:sample_queries].view(torch.int16).cpu().numpy().view("uint16"),
                       TOP_K)
        dt = time.perf_counter() - t
        kind = "port"
    return {"value": sample_rows * sample_queries / dt, "unit": "rows*queries/s",
            "cores": threads, "kind": kind,
            "sample": f"{sample_rows} rows x {sample_queries} queries of the same memory, "
                      f"top-{TOP_K}, {dt:.2f} s"}


def run_reference(args, rank, world):
    """The reference's own CPU path (oracle/_ref), host cores only; rank 0 runs."""
    if rank != 0:
        return None
    from oracle import oracle as O
    dev = torch.device("cpu")
    sample_rows, sample_queries = 1 << 20, 16
    rows = gen_rows_cpu(sample_rows)
    g = torch.Generator()
    g.manual_seed(SEED_QRY)
    q = torch.randn((sample_queries, DIM), generator=g).to(torch.bfloat16).float().numpy()
    threads = os.cpu_count() or 1
    if O.ref_available():
        mem = O.RefFlatMemory(rows, bf16=True)
        run = lambda: mem.pipeline(q, TOP_K, None, n_threads=threads)  # noqa: E731
        kind = "reference"
    else:
        qb = torch.from_numpy(q).to(torch.bfloat16).view(torch.int16).numpy().view("uint16")
        run = lambda: O.ip_topk_bf16(rows, qb, TOP_K)  # noqa: E731
        kind = "port"
    for _ in range(args.warmup):
        run()
    times = []
    for _ in range(args.steps):
        t = time.perf_counter()
        run()
        times.append(time.perf_counter() - t)
    del dev
    v = sample_rows * sample_queries / statistics.mean(times)
    return {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "rows*queries/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": statistics.mean(times) * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1))",
        "config": {"workload": f"{WORKLOAD}: the reference's CPU pipeline timed on a sample "
                               f"of it ({sample_rows} rows x {sample_queries} queries per step, "
                               f"rate in row-query pairs per second)",
                   "rows": sample_rows, "dim": DIM, "queries": sample_queries,
                   "top_k": TOP_K, "parallelism": f"host threads ({threads}), one query each",
                   "full_workload": {"rows": N_ROWS, "queries": N_QUERIES}},
        "cpu_baseline": {"value": v, "unit": "rows*queries/s", "cores": threads, "kind": kind,
                         "sample": f"{sample_rows} rows x {sample_queries} queries per step"},
        "e2e": {"value": v, "unit": "rows*queries/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def gen_rows_cpu(count: int):
    g = torch.Generator()
    out = torch.empty((count, DIM), dtype=torch.bfloat16)
    for c in range((count + CHUNK - 1) // CHUNK):
        g.manual_seed(SEED_MEM * 1000003 + c)
        n = min(CHUNK, count - c * CHUNK)
        out[c * CHUNK:c * CHUNK + n] = torch.randn((CHUNK, DIM), generator=g)[:n].to(torch.bfloat16)
    return out.view(torch.int16).numpy().view("uint16")


# ---------------------------------------------------------------- config 1
F_ROWS, F_DIM, F_NQ, F_K = 65536, 128, 64, 64
SEED_F_MEM, SEED_F_QRY = 1, 2
L2_FLUSH_BYTES = 256 << 20     # > the 126 MB L2


def run_flat_f32(args, rank, world, local):
    """Flat inner-product top-k + threshold: FlatIndexMemory<float> of 65,536 x
    128 N(0,1) rows, top-64 and the threshold bitmap at 2 sqrt(128) (the
    reference's InnerProductCompute -> TopKRetrieval / ThresholdRetrieval),
    as one call with one query and one call with 64.  The memory (32 MiB)
    fits in L2, so a 256 MB write flushes L2 before every timed call, and each
    call is timed alone by its own CUDA events.  Every rank runs the same
    calls (replicas; the workload is far below one GPU)."""
    import numpy as np

    import heteromm_b200 as hmm
    from heteromm_b200 import _abi
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import gen
    dev = torch.device("cuda", local)
    hmm.load()
    thr = float(np.float32(2.0 * np.sqrt(np.float32(128.0))))
    mem_np = gen.normal_f32(SEED_F_MEM, (F_ROWS, F_DIM))
    q_np = gen.normal_f32(SEED_F_QRY, (F_NQ, F_DIM))
    mem = torch.from_numpy(mem_np).to(dev)
    qall = torch.from_numpy(q_np).to(dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    pk, pk_kind = peaks()
    out = {}
    for nq in (1, F_NQ):
        q = qall[:nq].contiguous()

        def call(qq):
            return hmm.ip_topk_f32(mem, qq, F_K, thr)

        for _ in range(args.warmup):
            call(q)
        torch.cuda.synchronize()
        pairs = []
        with ClockSampler(local) as clk:
            l0 = _abi.kernel_launches()
            for i in range(args.steps):
                flush.fill_(i & 255)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                call(q)
                e1.record(stream)
                pairs.append((e0, e1))
            torch.cuda.synchronize()
            launches = _abi.kernel_launches() - l0
        ms = sum(a.elapsed_time(b) for a, b in pairs) / args.steps
        # end to end: queries from pinned host memory, indices, scores and the
        # threshold bitmap back to pinned host memory, per call
        q_host = q.cpu().pin_memory()
        q_dev = torch.empty_like(q)
        words = (F_ROWS + 63) // 64
        hi = torch.empty((nq, F_K), dtype=torch.int32).pin_memory()
        hs = torch.empty((nq, F_K), dtype=torch.float32).pin_memory()
        hb = torch.empty((nq, words), dtype=torch.int64).pin_memory()
        pairs = []
        for i in range(args.steps):
            flush.fill_(i & 255)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            q_dev.copy_(q_host, non_blocking=True)
            ii, ss, bb = call(q_dev)
            hi.copy_(ii, non_blocking=True)
            hs.copy_(ss, non_blocking=True)
            hb.copy_(bb, non_blocking=True)
            e1.record(stream)
            pairs.append((e0, e1))
        torch.cuda.synchronize()
        e2e_ms = sum(a.elapsed_time(b) for a, b in pairs) / args.steps
        if world > 1:
            t = torch.tensor([ms, e2e_ms], dtype=torch.float64, device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms, e2e_ms = t.tolist()
        if rank != 0:
            continue
        from oracle import oracle as O
        oi, ob, _ = O.ip_topk_f32(mem_np, q_np[:nq], F_K, thr)
        equal = bool(np.array_equal(hi.numpy(), oi) and
                     np.array_equal(hb.numpy().view(np.uint64), ob))
        bytes_alg = F_ROWS * F_DIM * 4 + nq * F_DIM * 4 + nq * F_K * 8 + nq * words * 8
        gbs = bytes_alg / (ms * 1e-3) / 1e9
        clocks = clk.summary()
        sm_mhz = clocks.get("sm_mhz") or pk.get("sm_max_mhz", 1965.0)
        # the reference's arithmetic (a separate fp32 multiply and add per
        # element, no FMA) is two CUDA-core instructions per multiply-add
        instr = 2.0 * F_ROWS * F_DIM * nq
        issue_peak = 148 * 128 * sm_mhz * 1e6
        e = {
            "metric": "flat fp32 score + top-64 + threshold bitmap: row-query pairs per second",
            "value": F_ROWS * nq / (ms * 1e-3), "unit": "rows*queries/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak (replicas)", "dtype": "f32",
            "data": "synthetic (seeded N(0,1))",
            "config": {"workload": f"flat fp32: {F_ROWS} x {F_DIM} rows, {nq} "
                                   f"quer{'y' if nq == 1 else 'ies'} per call, top-{F_K}, "
                                   f"threshold 2*sqrt(128)",
                       "l2": "flushed before every call (256 MB write)",
                       "parallelism": f"replicas x{world}"},
            "e2e": {"value": F_ROWS * nq / (e2e_ms * 1e-3), "unit": "rows*queries/s",
                    "ms_per_step": e2e_ms, "h2d_bytes_per_step": nq * F_DIM * 4,
                    "d2h_bytes_per_step": nq * (F_K * 8 + words * 8)},
            "gpu_launches": launches,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": gbs / pk["hbm_gbs"], "traffic": None,
                         "kernel": ("narrow_ip_topk_kernel<F32In>" if nq <= 4 else
                                    "fused_ip_topk_kernel<F32In>") +
                                   " + the candidate merge (the whole call, timed by events "
                                   "around it)",
                         "kernel_ms": ms, "peak_kind": f"{pk_kind} copy bandwidth",
                         "issue": {"achieved_ginstr_s": instr / (ms * 1e-3) / 1e9,
                                   "peak_ginstr_s": issue_peak / 1e9,
                                   "frac": instr / (ms * 1e-3) / issue_peak,
                                   "note": "exact fp32 multiply + add in the reference's order: "
                                           "2 instructions per multiply-add; peak = 148 SMs x "
                                           "128 lanes x the sampled SM clock (derived)"}},
            "clocks": clocks,
            "parity": {"checked_queries": nq, "equal": equal,
                       "against": "oracle: indices and threshold bitmap bit-exact"},
        }
        if world == 1 and not args.no_cpu_baseline:
            threads = os.cpu_count() or 1
            use = min(threads, nq)
            if O.ref_available():
                rm = O.RefFlatMemory(mem_np)
                reps, t0 = 0, time.perf_counter()
                while time.perf_counter() - t0 < 2.0:
                    rm.pipeline(q_np[:nq], F_K, thr, n_threads=use)
                    reps += 1
                dt = (time.perf_counter() - t0) / reps
                rm.close()
                kind = "reference"
            else:
                reps, t0 = 0, time.perf_counter()
                while time.perf_counter() - t0 < 2.0:
                    O.ip_topk_f32(mem_np, q_np[:nq], F_K, thr)
                    reps += 1
                dt = (time.perf_counter() - t0) / reps
                kind = "port"
            e["cpu_baseline"] = {
                "value": F_ROWS * nq / dt, "unit": "rows*queries/s", "cores": use, "kind": kind,
                "sample": f"the same {nq}-query call: the reference's InnerProductCompute -> "
                          f"TopKRetrieval(64) + ThresholdRetrieval per query "
                          f"(KernelType::CPU, one query per thread), {reps} repetitions, "
                          f"{dt * 1e3:.1f} ms each"}
        out[f"q{nq}"] = e
    return out if rank == 0 else None


# ---------------------------------------------------------------- config 2
P_BATCH, P_HEADS, P_LEN, P_DIM = 8, 32, 32768, 128
P_PAGE, P_BLOCK, P_TOP = 16, 64, 64
SEED_K, SEED_PERM, SEED_Q = 3, 4, 5


def run_paged(args, rank, world, local):
    """Paged-KV block-sparse decode: (batch x heads) sequences of P_LEN bf16
    tokens in 16-token pages (shuffled physical order), fp32 mean summaries of
    64-token blocks, top-64 blocks by q . summary, softmax attention over them.
    Sequences are split across ranks (no exchange)."""
    import heteromm_b200 as hmm
    from heteromm_b200 import _abi
    dev = torch.device("cuda", local)
    hmm.load()
    n_all = args.seqs if args.seqs else P_BATCH * P_HEADS
    per = n_all // world
    pps = P_LEN // P_PAGE
    n_pages = per * pps
    g = torch.Generator(device=dev)
    kp = torch.empty((n_pages, P_PAGE, P_DIM), dtype=torch.bfloat16, device=dev)
    vp = torch.empty_like(kp)
    step_pages = 1 << 16
    for c in range(0, n_pages, step_pages):
        g.manual_seed(SEED_K * 1000003 + rank * 7919 + c)
        kp[c:c + step_pages] = torch.randn(kp[c:c + step_pages].shape, generator=g, device=dev)
        vp[c:c + step_pages] = torch.randn(vp[c:c + step_pages].shape, generator=g, device=dev)
    gc = torch.Generator()
    gc.manual_seed(SEED_PERM + rank)
    table = torch.randperm(n_pages, generator=gc).to(torch.int32).reshape(per, pps).to(dev)
    gc.manual_seed(SEED_Q + rank)
    q = torch.randn((per, P_DIM), generator=gc).to(torch.bfloat16).to(dev)
    k16, v16, q16 = kp.view(torch.int16), vp.view(torch.int16), q.view(torch.int16)
    torch.cuda.synchronize()

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    summ = hmm.paged_kv_summary_bf16(k16, table, P_LEN, P_BLOCK)
    e1.record()
    torch.cuda.synchronize()
    build_ms = e0.elapsed_time(e1)

    # decode loop: no per-step wait; the bounds status is checked after the loop
    status = torch.zeros(1, dtype=torch.int32, device=dev)

    def step(qq):
        return hmm.block_sparse_decode_bf16(qq, summ, k16, v16, table, P_LEN, P_BLOCK, P_TOP,
                                            status=status)

    for _ in range(args.warmup):
        step(q16)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    _abi.profile_read()
    _abi.profile_enable(True)
    stream = torch.cuda.current_stream()
    with ClockSampler(local) as clk:
        l0 = _abi.kernel_launches()
        e0.record(stream)
        for _ in range(args.steps):
            step(q16)
        e1.record(stream)
        torch.cuda.synchronize()
        launches = _abi.kernel_launches() - l0
    _abi.profile_enable(False)
    k_total, k_n = _abi.profile_read()
    ms = e0.elapsed_time(e1) / args.steps
    kern_ms = k_total / args.steps   # per step, all its launches
    from heteromm_b200.paged import check_status
    check_status(status)

    # the min/max-bound selector (MinMaxIndexMemory summaries): built once, then
    # per step the blocks with the largest bound of q.k and attention over them
    e0.record(stream)
    mm = hmm.paged_kv_minmax_bf16(k16, table, P_LEN, P_BLOCK)
    e1.record(stream)
    torch.cuda.synchronize()
    mm_build_ms = e0.elapsed_time(e1)

    def mm_step(qq):
        sel = hmm.block_select_minmax(qq, mm, P_TOP)
        return sel, hmm.block_sparse_attention_bf16(qq, k16, v16, table, P_LEN, P_BLOCK, sel)

    for _ in range(args.warmup):
        mm_step(q16)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.steps):
        mm_step(q16)
    e1.record(stream)
    torch.cuda.synchronize()
    mm_ms = e0.elapsed_time(e1) / args.steps
    del mm

    # end to end: q from pinned host memory, selected blocks + outputs back
    q_host = q16.cpu().pin_memory()
    q_dev = torch.empty_like(q16)
    ob = torch.empty((per, P_TOP), dtype=torch.int32).pin_memory()
    oo = torch.empty((per, P_DIM), dtype=torch.float32).pin_memory()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.steps):
        q_dev.copy_(q_host, non_blocking=True)
        b, o = step(q_dev)
        ob.copy_(b, non_blocking=True)
        oo.copy_(o, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms, kern_ms, e2e_ms], dtype=torch.float64, device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms, kern_ms, e2e_ms = t.tolist()
    if rank != 0:
        return None
    pk, pk_kind = peaks()
    kv_bytes = per * P_TOP * P_BLOCK * P_DIM * 2 * 2          # selected K and V
    summ_bytes = per * (P_LEN // P_BLOCK) * P_DIM * 4
    achieved = kv_bytes / (kern_ms * 1e-3) / 1e9
    res = {
        "metric": "paged-KV block-sparse decode: (batch, head) queries per second",
        "value": n_all / (ms * 1e-3), "unit": "queries/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) K/V, shuffled physical pages)",
        "config": {"workload": f"paged-KV decode: batch {P_BATCH} x {P_HEADS} heads, "
                               f"{P_LEN} tokens x {P_DIM} bf16, page {P_PAGE}, "
                               f"block {P_BLOCK}, top-{P_TOP}",
                   "parallelism": f"(batch, head) split x{world}",
                   "l2": "inputs larger than L2 (604 MB read per step)",
                   "summary_build_ms": build_ms,
                   "step_gbs": (kv_bytes + summ_bytes) / (ms * 1e-3) / 1e9,
                   "minmax_selector": {"summary_build_ms": mm_build_ms, "step_ms": mm_ms,
                                       "note": "blocks by the min/max bound of q.k, then the "
                                               "same attention; bounds read back every step"}},
        "e2e": {"value": n_all / (e2e_ms * 1e-3), "unit": "queries/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": per * P_DIM * 2,
                "d2h_bytes_per_step": per * (P_TOP * 4 + P_DIM * 4)},
        "gpu_launches": launches,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"],
                     "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                     "traffic": traffic_per_launch("bsa_page_kernel", per),
                     "kernel": "bsa_page_kernel<128,16>", "kernel_ms": kern_ms,
                     "kernel_launches_per_step": k_n / args.steps, "peak_kind": f"{pk_kind} copy bandwidth"},
        "clocks": clk.summary(),
    }
    # parity and CPU baseline: the reference's own decode of 8 of this rank's
    # sequences (blocks exact, outputs within the attention tolerance); timed
    # as the CPU baseline on one GPU
    from oracle import oracle as O
    import numpy as np
    n_s = 8
    tb = table.long()
    t_total = 0.0
    blocks_equal, out_close = True, True
    for s_i in range(n_s):
        keys = kp[tb[s_i]].float().reshape(P_LEN, P_DIM).cpu().numpy()
        vals = vp[tb[s_i]].float().reshape(P_LEN, P_DIM).cpu().numpy()
        qq = q[s_i].float().cpu().numpy()
        t = time.perf_counter()
        rb, ro = O.ref_paged_decode_f32(keys, vals, qq, P_BLOCK, P_TOP)
        t_total += time.perf_counter() - t
        # the last end-to-end step's results for this sequence
        blocks_equal &= bool(np.array_equal(ob[s_i].numpy(), rb))
        out_close &= bool(np.allclose(oo[s_i].numpy(), ro, rtol=2e-5, atol=2e-6))
    res["parity"] = {"checked_sequences": n_s, "blocks_equal": blocks_equal,
                     "outputs_within_tolerance": out_close, "equal": blocks_equal and out_close,
                     "against": "the reference's own PagedKVIndexBuilder + "
                                "InnerProductCompute + TopKRetrieval + BlockSparseAttention "
                                "(blocks exact, outputs rtol 2e-5 atol 2e-6)"}
    if world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = {"value": n_s / t_total, "unit": "queries/s", "cores": 1,
                               "kind": "reference",
                               "sample": f"{n_s} sequences: the reference's "
                                         f"PagedKVIndexBuilder + InnerProductCompute + "
                                         f"TopKRetrieval + BlockSparseAttention per sequence "
                                         f"(summary build included), {t_total:.2f} s"}
    return res


# ---------------------------------------------------------------- config 3
B_DOCS, B_VOCAB, B_MEAN, B_NQ, B_QLEN, B_K = 1_000_000, 30522, 60.0, 1024, 8, 10
SEED_CORPUS, SEED_BQ = 6, 8


def bm25_csr_build(tp, pd, tf, dl, dev, n_docs):
    """The index's CSR rebuilt from per-document term counts (the reference's
    term_freq.bin layout): on the device by hmm_bm25_csr_from_docs (inputs
    resident, CUDA events, checked against the original CSR), and on the host
    as a NumPy stable sort by term, for comparison."""
    import numpy as np

    from heteromm_b200.bm25 import csr_from_docs
    n_terms = tp.size - 1
    term = np.repeat(np.arange(n_terms, dtype=np.int32), np.diff(tp))
    order = np.argsort(pd, kind="stable")              # document major
    terms_dm = term[order]
    counts_dm = tf[order].astype(np.uint32)
    doc_ptr = np.zeros(n_docs + 1, np.int64)
    doc_ptr[1:] = np.cumsum(np.bincount(pd, minlength=n_docs))
    t0 = time.perf_counter()
    o2 = np.argsort(terms_dm, kind="stable")
    h_doc = np.repeat(np.arange(n_docs, dtype=np.int32), np.diff(doc_ptr))[o2]
    h_tf = counts_dm[o2].astype(np.uint16)
    h_ptr = np.zeros(n_terms + 1, np.int64)
    h_ptr[1:] = np.cumsum(np.bincount(terms_dm, minlength=n_terms))
    host_s = time.perf_counter() - t0
    d = [torch.from_numpy(a).to(dev) for a in (doc_ptr, terms_dm, counts_dm.view(np.int32))]
    out = csr_from_docs(*d, n_terms, dev)   # warm-up
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 3
    e0.record()
    for _ in range(reps):
        out = csr_from_docs(*d, n_terms, dev)
    e1.record()
    torch.cuda.synchronize()
    ok = (np.array_equal(out[0].cpu().numpy(), tp) and np.array_equal(out[1].cpu().numpy(), pd)
          and np.array_equal(out[2].cpu().numpy().view(np.uint16), tf)
          and np.array_equal(out[3].cpu().numpy(), dl) and np.array_equal(h_ptr, tp)
          and np.array_equal(h_doc, pd) and np.array_equal(h_tf, tf))
    return {"entries": int(doc_ptr[-1]), "device_ms": e0.elapsed_time(e1) / reps,
            "host_numpy_s": host_s, "equal": bool(ok)}


def run_bm25(args, rank, world, local):
    """BM25 top-10 over a 1M-doc CSR index (Zipf(1.1) terms over 30,522,
    Poisson(60) lengths), 1,024 queries of 8 distinct Zipf terms.  Queries are
    split across ranks (every rank holds the whole index; no exchange)."""
    import heteromm_b200 as hmm
    from heteromm_b200 import _abi
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import gen
    dev = torch.device("cuda", local)
    hmm.load()
    n_docs = args.docs if args.docs else B_DOCS
    tp, pd, tf, dl = gen.bm25_corpus(SEED_CORPUS, n_docs, B_VOCAB, B_MEAN)
    n_q = args.queries if args.queries else B_NQ
    qall = gen.bm25_queries(SEED_BQ, n_q, B_QLEN, B_VOCAB)
    per = n_q // world
    q_np = qall[rank * per:(rank + 1) * per]
    t0 = time.perf_counter()
    index = hmm.BM25Index(tp, pd, tf, dl, dev)
    torch.cuda.synchronize()
    build_s = time.perf_counter() - t0
    csr_build = bm25_csr_build(tp, pd, tf, dl, dev, n_docs) if rank == 0 else None
    q = torch.from_numpy(q_np).to(dev)
    for _ in range(args.warmup):
        index.topk(q, B_K)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _abi.profile_read()
    _abi.profile_enable(True)
    with ClockSampler(local) as clk:
        l0 = _abi.kernel_launches()
        e0.record(stream)
        for _ in range(args.steps):
            index.topk(q, B_K)
        e1.record(stream)
        torch.cuda.synchronize()
        launches = _abi.kernel_launches() - l0
    _abi.profile_enable(False)
    k_total, k_n = _abi.profile_read()
    ms = e0.elapsed_time(e1) / args.steps
    kern_ms = k_total / args.steps   # per step, all its launches
    q_host = torch.from_numpy(q_np).pin_memory()
    q_dev = torch.empty_like(q)
    oi = torch.empty((per, B_K), dtype=torch.int32).pin_memory()
    osc = torch.empty((per, B_K), dtype=torch.float64).pin_memory()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.steps):
        q_dev.copy_(q_host, non_blocking=True)
        i, sc = index.topk(q_dev, B_K)
        oi.copy_(i, non_blocking=True)
        osc.copy_(sc, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms, kern_ms, e2e_ms], dtype=torch.float64, device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms, kern_ms, e2e_ms = t.tolist()
    if rank != 0:
        return None
    pk, pk_kind = peaks()
    df = tp[1:] - tp[:-1]
    post = int(df[q_np].sum())      # postings scored per step (all query terms distinct)
    # algorithmic bytes: the postings each query reads, in the index the kernel
    # scores from (an int32 doc id + an fp64 impact each).  Queries run fastest
    # in the grid, so a doc range's index slice is read from DRAM about once per
    # launch and served to the queries in flight by L2: the bound is L2 bandwidth
    bytes_alg = post * 12
    achieved = bytes_alg / (kern_ms * 1e-3) / 1e9
    l2_gbs = l2_read_peak(dev)
    idx_bytes = int(tp[-1]) * 12     # the whole index, the DRAM reads of one launch at least
    res = {
        "metric": "BM25 top-10 queries per second", "value": n_q / (ms * 1e-3),
        "unit": "queries/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f64",
        "data": "synthetic (seeded Zipf/Poisson corpus standing in for a BeIR-style corpus)",
        "config": {"workload": f"BM25: {n_docs} docs, vocab {B_VOCAB}, {tp[-1]} postings, "
                               f"{n_q} queries x {B_QLEN} terms, top-{B_K}",
                   "parallelism": f"query split x{world}",
                   "postings_per_step": post, "index_prepare_s": build_s,
                   "csr_from_docs": csr_build,
                   "l2": "inputs larger than L2 (postings read per step > 126 MB)"},
        "e2e": {"value": n_q / (e2e_ms * 1e-3), "unit": "queries/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": per * B_QLEN * 4,
                "d2h_bytes_per_step": per * B_K * (4 + 8)},
        "gpu_launches": launches,
        "roofline": {"bound": "l2", "achieved": achieved, "peak": l2_gbs,
                     "unit": "GB/s", "frac": achieved / l2_gbs,
                     "kernel": "bm25_range_kernel", "kernel_ms": kern_ms,
                     "kernel_launches_per_step": k_n / args.steps,
                     "algorithmic": "postings read per query x 12 B (int32 doc id + fp64 impact)",
                     "peak_kind": "measured here: L2-resident torch sums (64 MiB) and copies "
                                  "(2 x 40 MiB), 40 back to back, best of 5",
                     "hbm": {"index_bytes": idx_bytes,
                             "achieved": idx_bytes / (kern_ms * 1e-3) / 1e9,
                             "peak": pk["hbm_gbs"], "peak_kind": f"{pk_kind} copy bandwidth",
                             "note": "DRAM reads the index about once per launch"},
                     "traffic": traffic_per_launch("bm25_range_kernel", per)},
        "clocks": clk.summary(),
    }
    # parity: a spread subset of this rank's queries against the oracle (exact
    # fp64 scores, ascending term order), from the last end-to-end step
    import numpy as np

    from oracle import oracle as O
    pick = np.arange(0, per, max(1, per // 64))
    t = time.perf_counter()
    wi, wsc = O.bm25_topk(tp, pd, tf, dl, q_np[pick], B_K)
    dt = time.perf_counter() - t
    equal = bool(np.array_equal(oi.numpy()[pick], wi) and
                 np.array_equal(osc.numpy()[pick].view(np.uint64), wsc.view(np.uint64)))
    res["parity"] = {"checked_queries": int(pick.size), "equal": equal,
                     "against": "oracle: doc ids and fp64 scores bit-exact"}
    if world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = {"value": pick.size / dt, "unit": "queries/s",
                               "cores": os.cpu_count() or 1, "kind": "port",
                               "sample": f"{pick.size} of the queries on the same {n_docs}-doc "
                                         f"index: the oracle's restatement of the reference's "
                                         f"BM25 CPU kernel over the CSR postings (OpenMP over "
                                         f"queries), {dt:.2f} s.  The reference's own kernel "
                                         f"scans every document's term map per query term; "
                                         f"`--config bm25 --ref-bm25` times it on this corpus"}
        if args.ref_bm25:
            idx = O.RefBM25(tp, pd, tf, n_docs)
            n_cq = 2
            t = time.perf_counter()
            for i in range(n_cq):
                idx.query(qall[i])
            dt = time.perf_counter() - t
            idx.close()
            res["cpu_baseline_reference"] = {
                "value": n_cq / dt, "unit": "queries/s", "cores": 1, "kind": "reference",
                "sample": f"{n_cq} queries on the same {n_docs}-doc corpus with the reference's "
                          f"own BM25IndexMemory + FusedBM25Retrieval CPU kernel, {dt:.2f} s"}
    return res


# ---------------------------------------------------------------- config 4
D_TOKENS, D_HEADS, D_KEYS, D_DIM, D_TOPK = 4096, 64, 131072, 128, 2048
SEED_DQ, SEED_DK, SEED_DW = 9, 10, 11


def l2_read_peak(dev) -> float:
    """Bandwidth of L2-resident buffers on this GPU, GB/s: the best of (a) 40
    back-to-back torch sums over a 64 MiB fp32 tensor (reads) and (b) 40
    back-to-back copies between two 40 MiB tensors (reads + writes), each timed
    as one group with events, best of 5 groups.  Half of the 126 MB L2 or less
    is in use, so the buffers stay resident after the warm-up.  The
    denominator for a kernel whose operands are served by L2."""
    x = torch.ones(16 << 20, dtype=torch.float32, device=dev)
    a = torch.ones(10 << 20, dtype=torch.float32, device=dev)
    b = torch.empty_like(a)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def best_of(op, nbytes):
        for _ in range(5):
            op()
        torch.cuda.synchronize()
        best = float("inf")
        for _ in range(5):
            e0.record()
            for _ in range(40):
                op()
            e1.record()
            torch.cuda.synchronize()
            best = min(best, e0.elapsed_time(e1) / 40)
        return nbytes / (best * 1e-3) / 1e9

    reads = best_of(lambda: x.sum(), x.numel() * 4)
    copies = best_of(lambda: b.copy_(a), 2 * a.numel() * 4)
    del x, a, b
    return max(reads, copies)


def fp8_gemm_peak(dev, seconds: float = 1.0) -> float:
    """Dense FP8 (e4m3) GEMM throughput of cuBLAS on this GPU (torch._scaled_mm,
    8192^3, back to back for about `seconds`), TFLOP/s: the measured FP8
    denominator for the tensor roofline."""
    n = 8192
    a = torch.randn((n, n), device=dev).to(torch.float8_e4m3fn)
    b = torch.randn((n, n), device=dev).to(torch.float8_e4m3fn).t()
    one = torch.ones((), device=dev)
    torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 0
    e0.record()
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        for _ in range(10):
            torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
        reps += 10
        torch.cuda.synchronize()
    e1.record()
    torch.cuda.synchronize()
    return 2.0 * n ** 3 * reps / (e0.elapsed_time(e1) * 1e-3) / 1e12


def run_dsa(args, rank, world, local):
    """DSA lightning-indexer prefill: 4,096 query tokens x 64 heads x 128 e4m3
    against 131,072 e4m3 keys, weights U(0,1), causal (token t at position
    131,072 - 4,096 + t), top-2,048 keys per token.  Query tokens are split
    across ranks (no exchange)."""
    import heteromm_b200 as hmm
    from heteromm_b200 import _abi
    dev = torch.device("cuda", local)
    hmm.load()
    T = (args.tokens if args.tokens else D_TOKENS) // world
    t0 = rank * T
    pos0 = D_KEYS - D_TOKENS + t0
    g = torch.Generator(device=dev)
    g.manual_seed(SEED_DQ * 1000003 + rank)
    x = torch.randn((T, D_HEADS, D_DIM), generator=g, device=dev)
    q = (x * (448.0 / x.abs().max())).to(torch.float8_e4m3fn).view(torch.uint8)
    g.manual_seed(SEED_DK)
    y = torch.randn((D_KEYS, D_DIM), generator=g, device=dev)
    k = (y * (448.0 / y.abs().max())).to(torch.float8_e4m3fn).view(torch.uint8)
    g.manual_seed(SEED_DW * 1000003 + rank)
    w = torch.rand((T, D_HEADS), generator=g, device=dev)
    del x, y

    def step(qq):
        return hmm.dsa_indexer_fp8(qq, k, w, pos0, D_TOPK)

    for _ in range(args.warmup):
        step(q)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _abi.profile_read()
    _abi.profile_enable(True)
    with ClockSampler(local) as clk:
        l0 = _abi.kernel_launches()
        e0.record(stream)
        for _ in range(args.steps):
            step(q)
        e1.record(stream)
        torch.cuda.synchronize()
        launches = _abi.kernel_launches() - l0
    _abi.profile_enable(False)
    k_total, k_n = _abi.profile_read()
    ms = e0.elapsed_time(e1) / args.steps
    kern_ms = k_total / args.steps   # per step, all its launches
    # end to end through the public host-to-host call: q and w uploaded, indices
    # and scores read back, in token slices whose transfers overlap the indexer
    q_host = q.cpu().pin_memory()
    w_host = w.cpu().pin_memory()
    chunks = args.dsa_chunks or None
    # warm-up in the timed loop's own pattern (the previous call's pinned
    # results stay alive while the next call runs, so two sets get allocated)
    for _ in range(max(2, args.warmup)):
        h_idx, h_sc = hmm.dsa_indexer_fp8_host(q_host, k, w_host, pos0, D_TOPK, chunks=chunks)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.steps):
        h_idx, h_sc = hmm.dsa_indexer_fp8_host(q_host, k, w_host, pos0, D_TOPK, chunks=chunks)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms, kern_ms, e2e_ms], dtype=torch.float64, device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms, kern_ms, e2e_ms = t.tolist()
    if rank != 0:
        return None
    n_tok = T * world
    vis = sum(min(D_KEYS, pos0 + t + 1) for t in range(T))     # this rank's (token, key) pairs
    flop = 2.0 * D_HEADS * D_DIM * vis
    achieved = flop / (kern_ms * 1e-3) / 1e12
    peak = fp8_gemm_peak(dev)
    res = {
        "metric": "DSA indexer query tokens per second", "value": n_tok / (ms * 1e-3),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "e4m3",
        "data": "synthetic (seeded N(0,1) scaled to the e4m3 range, w ~ U(0,1))",
        "config": {"workload": f"DSA indexer: {n_tok} tokens x {D_HEADS} heads x {D_DIM} e4m3, "
                               f"{D_KEYS} keys, causal, top-{D_TOPK}",
                   "parallelism": f"token split x{world}",
                   "l2": "keys (16 MiB) re-read per token group, hit bitmap (T x 16 KiB) "
                         "and candidate lists larger than L2"},
        "e2e": {"value": n_tok / (e2e_ms * 1e-3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": T * D_HEADS * D_DIM + T * D_HEADS * 4,
                "d2h_bytes_per_step": T * D_TOPK * (4 + 4), "token_slices": args.dsa_chunks or "waves"},
        "gpu_launches": launches,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": traffic_per_launch("dsa_scores_kernel", T),
                     "kernel": "dsa_scores_kernel",
                     "kernel_ms": kern_ms, "kernel_launches_per_step": k_n / args.steps,
                     "peak_kind": "measured here: cuBLAS e4m3 GEMM 8192^3 (torch._scaled_mm), "
                                  "1 s back to back"},
        "clocks": clk.summary(),
    }
    # parity: the first, a middle and the last tokens of this rank against the
    # oracle's exact ranking (indices in order, and scores), from the last
    # end-to-end call
    import numpy as np

    from oracle import oracle as O
    runs = [(0, min(8, T))] + ([(max(8, T - 8), T)] if T > 8 else [])   # first and last tokens
    pick = np.concatenate([np.arange(a0, a1) for a0, a1 in runs])
    ks = k.cpu().numpy()
    t = time.perf_counter()
    parts = [O.dsa_indexer_fp8(q[a0:a1].cpu().numpy(), ks, w[a0:a1].cpu().numpy(), pos0 + a0,
                               D_TOPK) for a0, a1 in runs]
    dt = time.perf_counter() - t
    wi = np.concatenate([p_[0] for p_ in parts])
    wsc = np.concatenate([p_[1] for p_ in parts])
    gi, gs = h_idx.numpy()[pick], h_sc.numpy()[pick]
    res["parity"] = {"checked_tokens": int(pick.size),
                     "tokens_equal": int(sum(np.array_equal(gi[j], wi[j]) for j in range(pick.size))),
                     "equal": bool(np.array_equal(gi, wi) and
                                   np.array_equal(gs.view(np.uint32), wsc.view(np.uint32))),
                     "against": "oracle: exact e4m3 dots, fp32 head sum in head order; "
                                "indices best first (ties to the lowest key) and scores bit-exact"}
    if world == 1 and not args.no_cpu_baseline:
        n_s = int(pick.size)
        res["cpu_baseline"] = {"value": n_s / dt, "unit": "tokens/s",
                               "cores": os.cpu_count() or 1, "kind": "port",
                               "sample": f"{n_s} query tokens against all {D_KEYS} keys, exact "
                                         f"scores + top-{D_TOPK} (oracle restatement, OpenMP "
                                         f"over tokens), {dt:.2f} s"}
    return res


def traffic_per_launch(kernel: str, units: int):
    """DRAM bytes (read + write) of one launch of `kernel` from its committed
    ncu capture, scaled from the capture's units (rows, sequences) to `units`:
    each kernel streams every unit once, so its traffic grows in proportion."""
    p = os.path.join(ROOT, "profiles", f"{kernel}.traffic.json")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        d = json.load(f)
    return d["dram_bytes_per_launch"] * units / d["units"]


def main():
    global N_ROWS, WORKLOAD
    # stdout carries the JSON line alone: anything the libraries print (NCCL's
    # version banner, for one) goes to stderr
    json_out = os.fdopen(os.dup(1), "w")
    sys.stdout.flush()
    os.dup2(2, 1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--config", choices=["all", "flat", "flat_f32", "paged", "bm25", "dsa"],
                    default="all",
                    help="all (default): the sharded flat retrieval benchmark, then every other "
                         "workload nested under 'configs'; flat: the sharded flat retrieval "
                         "alone; flat_f32: fp32 top-k + threshold at 1 and 64 queries; paged: "
                         "the paged-KV block-sparse decode step; bm25: BM25 top-10 over a CSR "
                         "index; dsa: the FP8 DSA indexer")
    ap.add_argument("--sustain-s", type=float, default=2.0,
                    help="flat: seconds of the sustained loop after the timed steps")
    ap.add_argument("--exchange-deadline-s", type=float, default=30.0,
                    help="flat, N > 1: host deadline of the candidate exchange in the "
                         "end-to-end calls")
    ap.add_argument("--ref-bm25", action="store_true",
                    help="bm25: also time the reference's own BM25 CPU kernel on the corpus "
                         "(its index takes minutes to build on the host)")
    ap.add_argument("--dsa-chunks", type=int, default=0,
                    help="token slices of the DSA end-to-end call (0: whole waves of the "
                         "scoring kernel; transfers overlap the work)")
    ap.add_argument("--tokens", type=int, default=0,
                    help="dsa: number of query tokens (default 4,096; fewer are for profiler "
                         "captures only)")
    ap.add_argument("--queries", type=int, default=0,
                    help="bm25: number of queries (default 1,024; fewer are for profiler "
                         "captures only)")
    ap.add_argument("--docs", type=int, default=0,
                    help="bm25: number of documents (default 1M; fewer are for profiler "
                         "captures only)")
    ap.add_argument("--seqs", type=int, default=0,
                    help="paged: number of (batch, head) sequences (default 8 x 32; fewer "
                         "are for profiler captures only)")
    ap.add_argument("--rows", type=int, default=N_ROWS,
                    help="total rows (default 64Mi, the benchmark workload; smaller "
                         "values are for profiler captures only)")
    args = ap.parse_args()
    if args.rows != N_ROWS:
        N_ROWS = args.rows
        WORKLOAD = f"profiling case: {N_ROWS} x 128 bf16 rows, 256 queries, top-100"
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        res = run_reference(args, rank, world)
    else:
        rank, world, local = init_dist()
        runners = {"flat": run_ours, "flat_f32": run_flat_f32, "paged": run_paged,
                   "bm25": run_bm25, "dsa": run_dsa}
        if args.config == "all":
            res = run_ours(args, rank, world, local)
            nested = {}
            for name in ("flat_f32", "paged", "bm25", "dsa"):
                torch.cuda.empty_cache()
                if world > 1:
                    torch.distributed.barrier()
                r = runners[name](args, rank, world, local)
                if rank == 0:
                    nested[name] = r
            if rank == 0:
                res["configs"] = nested
        else:
            res = runners[args.config](args, rank, world, local)
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
    if rank == 0 and res is not None:
        print(json.dumps(res), file=json_out, flush=True)


if __name__ == "__main__":
    main()
