// flat_tc.cu — tcgen05 (5th-gen tensor core) scoring of a bf16 row shard with
// exact top-k selection: the sharded flat-retrieval hot path (inner product
// of reference steps/example_kernel/inner_product_compute.cpp:11-31 fused
// with the top-k of topk_retrieval.cpp:13-31), bit-exact to the reference's
// sequential fp32 arithmetic.
//
// Tensor cores sum in their own order, so their scores are approximations.
// The kernel uses them only to decide which (row, query) pairs can matter:
//   s~ = tensor-core score of row r for query q (fp32 accumulate in TMEM)
//   |s~ - s| <= EPS * max_j|a_rj| * sum_j|b_qj| + 2^-118   (s = the reference's
//   score; the 2^-118 covers products below fp32's normal range, and a bound
//   past 2^100, where partial sums may overflow, lets every pair through)
// A pair is rescored exactly - the reference's separate fp32 multiply and add
// in ascending j over the row (read back from L2, where it was just streamed)
// - only when its upper bound s~ + margin reaches the query's current
// threshold.  Exact (score, row) composites that beat the threshold enter a
// per-query candidate pool in global memory; each time a pool reaches a
// power-of-two fill mark, the warp that filled it computes the pool's k-th
// best composite and raises the query's threshold (a k-th best of a subset
// never exceeds the k-th best of the whole memory, so no true top-k row is
// ever dropped).  A final merge takes the exact top-k of each pool.
//
// The starting threshold comes from a short sample pass of the same kernel
// over SAMPLE_TPC tiles per cluster spread over the shard: each epilogue
// thread keeps the SAMPLE_M largest lower bounds s~ - margin of its query, and
// the k-th largest of them all (distinct rows, each bound <= its row's exact
// score) is <= the shard's k-th best score.  The scoring pass then covers
// every row with empty pools, and its first tiles already filter as tightly
// as the k-th best of the sample allows.
//
// The queries are the MMA's M side and the rows its N side, so each epilogue
// thread owns one query and compares its scores against one threshold held in
// a register; a pair of SMs (a cluster of two CTAs) shares each tile, so each
// SM's tensor core reads half of the row operand.  The kernel's thread roles
// are listed at the kernel.  Every mbarrier wait is bounded; a wait that gives
// up sets a status word and both CTAs of the pair drain and exit.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "hmm_common.cuh"
#include "sm100_ptx.cuh"

namespace hmm {

// from flat_topk.cu: the exact CUDA-core path (small shards, full pools)
hmm_status_t flat_bf16_exact(const uint16_t* mem, int64_t n, int64_t dim, const uint16_t* qry,
                             int64_t nq, int64_t k, int64_t row_offset, int64_t* out_idx,
                             float* out_scores, void* ws, size_t ws_bytes, cudaStream_t st);
size_t flat_bf16_exact_ws_bytes(int64_t n, int64_t nq, int64_t k);
hmm_status_t launch_pool_merge(const uint64_t* pool, int64_t cap, const int* counts, int nq,
                               int k, int64_t row_offset, int64_t* out_idx, float* out_scores,
                               cudaStream_t st);

namespace {

using namespace sm100;

constexpr int TC_DIM = 128;                    // row width handled (MMA K total)
constexpr int TC_NMAX = 256;                   // queries per pass: 128 per CTA of the pair
constexpr int PQ = 128;                        // queries per CTA (the pair's MMA M is 256)
constexpr int PR = 128;                        // rows per CTA and tile (the pair's MMA N is 256)
constexpr int STAGES = 5;
constexpr int ROW_BOX = PR * 128;              // 128 rows x 64 bf16 columns = 16 KiB
constexpr int ROW_STAGE = 2 * ROW_BOX;         // 32 KiB per CTA and tile
constexpr int Q_BOX = PQ * 128;                // 128 queries x 64 columns = 16 KiB
constexpr int Q_BYTES = 2 * Q_BOX;             // 32 KiB
constexpr int N_EPI_WARPS = 8;                 // two epilogue warpgroups (row halves)
constexpr int N_RB_WARPS = 2;                  // row-bound warps (two rows per lane)
constexpr int NTHREADS = 32 * (8 + N_EPI_WARPS);    // + TMA, MMA, 4 rescorers, 2 row-bound warps
constexpr int RING = 128;                       // pairs per epilogue warp awaiting rescoring
constexpr int N_RESCORERS = 4;                  // warps 2, 3, 6 and 7 (warp 3 of the first
                                                // CTA issues MMAs instead)
constexpr int RPR_MAX = 3;                      // rings per rescorer: 8 over 3 or 4 of them
constexpr int TMEM_COLS = 512;                  // two accumulators of 256 fp32 columns
constexpr float EPS = 1.0f / 1024.0f;          // >= 25x the worst-case summation gap
constexpr int TC_MIN_ROWS = 8192;              // smaller shards take the exact CUDA-core path
#ifndef HMM_SAMPLE_TPC
#define HMM_SAMPLE_TPC 4
#endif
constexpr int SAMPLE_TPC = HMM_SAMPLE_TPC;      // sample-pass pair tiles per cluster
constexpr int SAMPLE_M = 4;                     // lower bounds kept per (query, CTA)
constexpr int MAX_CTAS = 512;                   // grid bound (sample_lb sizing)
constexpr int POOL_CAP = 8192;
constexpr int KMAX_TC = 128;
#ifndef HMM_RAISE_STEP
#define HMM_RAISE_STEP 128
#endif
#ifndef HMM_RAISE_WINDOW
#define HMM_RAISE_WINDOW 512
#endif
constexpr int RAISE_STEP = HMM_RAISE_STEP;      // appends between threshold raises
constexpr int RAISE_WINDOW = HMM_RAISE_WINDOW;  // newest pool entries a raise selects over
constexpr int MR_RING = 8;                      // tiles of row bounds in flight
static_assert(MR_RING >= STAGES + 2, "a row-bound slot is rewritten only after both epilogues read it");
static_assert(N_RB_WARPS == 2, "the epilogue reads two row-bound slots per half");
constexpr uint64_t REFRESH_NS = 2000;          // cadence of the rescorers' shared-threshold refresh
constexpr uint64_t DRAIN_NS = 1000000;         // abort path: all of a producer's stage drains together

struct __align__(8) Ctrl {
    uint64_t full[STAGES];          // this CTA's rows of tile i landed (TMA tx); in the first
                                    // CTA also the peer's (its forwarder arrives)
    uint64_t empty[STAGES];         // ... consumed: row-bound threads + one epilogue thread
                                    // that has seen the tile's accumulator
    uint64_t acc_full[2];           // accumulator written (pair MMA commit)
    uint64_t acc_empty[2];          // first CTA only: drained by the epilogue warps of both CTAs
    uint64_t q_full;                // this CTA's queries landed (first CTA: and the peer's)
    uint32_t tmem_base;
    int abort;
    int issued;                     // first CTA: tiles whose MMAs are all issued (turn counter)
    // max|a| over the rows of (tile, half, row-bound warp) as (tile + 1) << 32 |
    // float bits: one 8-byte store carries the value and the tile it is for
    uint64_t mr[MR_RING][2][N_RB_WARPS];
    uint64_t tau[TC_NMAX];          // CTA copy of each of its queries' threshold composites
    uint64_t ring[N_EPI_WARPS][RING];    // (shard row << 8) | query, epilogue -> rescorer
    int ring_head[N_EPI_WARPS];          // consumed (rescorer)
    int ring_tail[N_EPI_WARPS];          // published (epilogue warp)
    int epi_done[N_EPI_WARPS];           // the epilogue warp has published its last pair
    unsigned hist[N_RESCORERS][256];
};

constexpr size_t TC_SMEM = 1024 /* alignment slack */ + Q_BYTES + STAGES * ROW_STAGE + sizeof(Ctrl);
static_assert(TC_SMEM <= 227 * 1024, "shared memory per CTA");

struct TcArgs {
    int64_t n_rows;
    int64_t row_begin;
    int n_tiles;             // 256-row pair tiles over [row_begin, n_rows)
    int sample_tiles;        // sample pass only: tiles spread evenly over the n_tiles
    uint64_t* sample_lb;     // sample pass only: [nq][gridDim.x * SAMPLE_M] lower-bound keys
    int nq;
    int k;
    int pool_cap;
    int wm0;                 // first fill mark that triggers a threshold raise
    const uint16_t* qry;     // [nq][128]
    const uint16_t* mem;     // [n_rows][128], for rescoring
    uint64_t* tau_global;    // [nq]
    uint64_t* pool;          // [nq][pool_cap]
    int* pool_cnt;           // [nq]
    int* status;             // [0] timeout flag, [1] pool overflow flag,
                             // [2] pairs rescored, [3] threshold raises
    uint64_t wait_ns;        // limit of every bounded wait (wait_limit_ns())
};

// EPS * M_h * L1_q (rounded up) plus 2^-118: products and partial sums below
// fp32's normal range may be flushed or rounded differently by the tensor core,
// at most 2^-126 each over 128 of them.
__device__ __forceinline__ float tc_margin(float mh, float l1) {
    return __fadd_ru(__fmul_ru(EPS, __fmul_ru(mh, l1)), 0x1p-118f);
}

__device__ __forceinline__ float tau_score(uint64_t t) {
    return t == 0ull ? -INFINITY : cand_score(t);
}

// max of three, NaN if any input is NaN.
__device__ __forceinline__ float max3_nan(float a, float b, float c) {
    float d;
    asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// s + a * b with the product rounded first (no contraction into an FMA).
__device__ __forceinline__ float mac_rn(float s, float a, float b) {
    return __fadd_rn(s, __fmul_rn(a, b));
}

__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// The reference's fp32 dot product of a memory row and a query, j
// ascending, each product rounded before it is added (a fused multiply-add
// would differ where a bf16 x bf16 product overflows fp32 or falls below its
// normal range), both read from global memory (the row was just streamed and
// is in L2; the queries are small and stay cached).
__device__ __forceinline__ float exact_dot_rows(const uint16_t* __restrict__ row,
                                                const uint16_t* __restrict__ qrow) {
    float s = 0.0f;
    const uint4* rp = reinterpret_cast<const uint4*>(row);
    const uint4* qp = reinterpret_cast<const uint4*>(qrow);
#pragma unroll
    for (int c = 0; c < 16; ++c) {
        const uint4 a = __ldg(rp + c);
        const uint4 b = __ldg(qp + c);
        s = mac_rn(s, bf_lo(a.x), bf_lo(b.x)); s = mac_rn(s, bf_hi(a.x), bf_hi(b.x));
        s = mac_rn(s, bf_lo(a.y), bf_lo(b.y)); s = mac_rn(s, bf_hi(a.y), bf_hi(b.y));
        s = mac_rn(s, bf_lo(a.z), bf_lo(b.z)); s = mac_rn(s, bf_hi(a.z), bf_hi(b.z));
        s = mac_rn(s, bf_lo(a.w), bf_lo(b.w)); s = mac_rn(s, bf_hi(a.w), bf_hi(b.w));
    }
    return s;
}

// The same dot product with the query read from the CTA's staged MMA operand
// (query ql of the CTA: two 64-column boxes of 128 queries, 128-byte rows,
// 16-byte chunk c of row ql at chunk position c ^ (ql & 7)); only the row
// comes from global memory, so all of its 16 loads are in flight together.
__device__ __forceinline__ float exact_dot_staged_q(const uint16_t* __restrict__ row,
                                                    const unsigned char* Qs, int ql) {
    uint4 a[16];
    const uint4* rp = reinterpret_cast<const uint4*>(row);
#pragma unroll
    for (int c = 0; c < 16; ++c) a[c] = __ldg(rp + c);
    float s = 0.0f;
#pragma unroll
    for (int c = 0; c < 16; ++c) {
        const uint4 b = *reinterpret_cast<const uint4*>(Qs + (c >> 3) * Q_BOX + ql * 128 +
                                                        (((c & 7) ^ (ql & 7)) << 4));
        s = mac_rn(s, bf_lo(a[c].x), bf_lo(b.x)); s = mac_rn(s, bf_hi(a[c].x), bf_hi(b.x));
        s = mac_rn(s, bf_lo(a[c].y), bf_lo(b.y)); s = mac_rn(s, bf_hi(a[c].y), bf_hi(b.y));
        s = mac_rn(s, bf_lo(a[c].z), bf_lo(b.z)); s = mac_rn(s, bf_hi(a[c].z), bf_hi(b.z));
        s = mac_rn(s, bf_lo(a[c].w), bf_lo(b.w)); s = mac_rn(s, bf_hi(a[c].w), bf_hi(b.w));
    }
    return s;
}

__device__ __forceinline__ uint32_t max_u16x2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("max.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t min_u16x2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("min.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
// Per half: the operand of larger magnitude, with the xor of both signs; a NaN
// operand gives NaN.  Its magnitude is max(|a|, |b|) whatever the signs.
__device__ __forceinline__ uint32_t absmax_bf16x2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("max.NaN.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// max_j |a_rj| over rows r and r + 32 of a staged 128-row tile, as fp32 bits.
// Magnitude bit patterns order as unsigned integers; NaN counts as +inf (so a
// NaN makes the bound infinite instead of hiding the other values).
__device__ __forceinline__ uint32_t rows_absmax_bits(const unsigned char* Rs, int r) {
    uint32_t m[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
        const int row = r + 32 * rr;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint4* p = reinterpret_cast<const uint4*>(Rs + h * ROW_BOX + row * 128);
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const uint4 a = p[c ^ (row & 7)];   // a quarter-warp's lanes hit distinct banks
                m[0] = absmax_bf16x2(m[0], a.x);
                m[1] = absmax_bf16x2(m[1], a.y);
                m[2] = absmax_bf16x2(m[2], a.z);
                m[3] = absmax_bf16x2(m[3], a.w);
            }
        }
    }
    const uint32_t v = min_u16x2(max_u16x2(max_u16x2(m[0] & 0x7fff7fffu, m[1] & 0x7fff7fffu),
                                           max_u16x2(m[2] & 0x7fff7fffu, m[3] & 0x7fff7fffu)),
                                 0x7f807f80u);
    return max(v & 0xffffu, v >> 16) << 16;
}

// Every lane polls (so each observes the phase itself); the warp proceeds
// only if all lanes saw it, keeping the warp converged either way.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          uint64_t limit) {
    const bool ok = mbar_wait_bounded(bar, parity, abort, limit);
    return __all_sync(0xffffffffu, ok);
}

// Gives up in both CTAs of the pair: the peer's waits see its flag at once.
__device__ __forceinline__ void set_abort(Ctrl* ctl, int* status, uint32_t peer) {
    atomicExch(&ctl->abort, 1);
    st_cluster_u32(mapa_shared(smem_u32(&ctl->abort), peer), 1u);
    atomicExch(&status[0], 1);
}

__device__ __forceinline__ int ld_volatile(const int* p) { return *reinterpret_cast<const volatile int*>(p); }
__device__ __forceinline__ void st_volatile(int* p, int v) { *reinterpret_cast<volatile int*>(p) = v; }

// k-th best of M <= RAISE_WINDOW pool keys (one warp), as the radix select of
// warp_select_threshold but over keys loaded into registers once: all of a
// lane's loads are in flight together (L2, bypassing L1, so that entries other
// SMs appended since an earlier read are seen), and the byte passes then touch
// only registers and the shared histogram.  Slots reserved but not yet
// written read as 0, below every real key: the result can only be lower, so it
// stays a lower bound of the window's k-th best.  Returns 0 for k >= M.
__device__ __forceinline__ uint64_t warp_kth_window(const uint64_t* __restrict__ keys, int M,
                                                    int k, unsigned* hist) {
    constexpr int PER_LANE = RAISE_WINDOW / 32;
    const int lane = threadIdx.x & 31;
    if (k >= M) return 0ull;
    uint64_t r[PER_LANE];
#pragma unroll
    for (int j = 0; j < PER_LANE; ++j) {
        const int i = lane + 32 * j;
        r[j] = i < M ? __ldcg(keys + i) : 0ull;
    }
    uint64_t prefix = 0, mask = 0;
    unsigned need = (unsigned)k;
    for (int shift = 56; shift >= 0; shift -= 8) {
        for (int b = lane; b < 256; b += 32) hist[b] = 0;
        __syncwarp();
#pragma unroll
        for (int j = 0; j < PER_LANE; ++j)
            if ((r[j] & mask) == prefix) atomicAdd(&hist[(r[j] >> shift) & 255], 1u);
        __syncwarp();
        // lane l owns bins 255-8l down to 248-8l (descending key order)
        unsigned c[8], s = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) { c[j] = hist[255 - 8 * lane - j]; s += c[j]; }
        unsigned incl = s;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        const unsigned excl = incl - s;
        const unsigned ball = __ballot_sync(0xffffffffu, excl < need && need <= incl);
        const int src = __ffs(ball) - 1;
        unsigned bucket = 0, before = 0, cnt = 0;
        if (lane == src) {
            unsigned acc = excl;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (cnt == 0 && acc + c[j] >= need) {
                    bucket = 255 - 8 * lane - j; before = acc; cnt = c[j];
                }
                acc += c[j];
            }
        }
        bucket = __shfl_sync(0xffffffffu, bucket, src);
        before = __shfl_sync(0xffffffffu, before, src);
        cnt = __shfl_sync(0xffffffffu, cnt, src);
        need -= before;
        prefix |= (uint64_t)bucket << shift;
        mask |= (uint64_t)0xff << shift;
        __syncwarp();
        // every key of this bucket is among the k best: the bucket's prefix
        // (lower bytes 0) is <= the k-th best and exactly k keys exceed it
        if (cnt == need) break;
    }
    return prefix;
}
static_assert(RAISE_WINDOW % 32 == 0 && RAISE_WINDOW <= 1024, "window keys held in registers");

// Rescores one batch of up to 32 queued pairs exactly (lane = pair) and
// appends the ones that beat their query's threshold to the pools; raises
// thresholds at fill marks from the newest RAISE_WINDOW pool entries.
// The pairs are the CTA's own queries (q0 .. q0 + 127), read from its staged
// query operand Qs.
__device__ __noinline__ void rescore_batch(Ctrl* ctl, unsigned* hist, uint64_t e, bool valid,
                                           int m, const TcArgs& a, const unsigned char* Qs,
                                           int q0) {
    const int lane = threadIdx.x & 31;
    if (lane == 0) atomicAdd(&a.status[2], m);
    int q = 0, raise = 0;
    const int64_t row = (int64_t)(e >> 8);
    if (valid && row < a.n_rows && (int)(e & 255u) < a.nq) {
        q = (int)(e & 255u);
        const int ql = q - q0;
        const float s = (unsigned)ql < (unsigned)PQ
                            ? exact_dot_staged_q(a.mem + row * TC_DIM, Qs, ql)
                            : exact_dot_rows(a.mem + row * TC_DIM, a.qry + (int64_t)q * TC_DIM);
        const uint64_t E = make_cand(f32_key(s), (uint32_t)row);
        if (E > ctl->tau[q]) {
            const int pos = atomicAdd(&a.pool_cnt[q], 1);
            if (pos < a.pool_cap) {
                a.pool[(int64_t)q * a.pool_cap + pos] = E;
                const int w = pos + 1;
                if (w >= a.wm0 && (w % RAISE_STEP) == 0) raise = w;
            } else {
                atomicExch(&a.status[1], 1);
            }
        }
    }
    unsigned mk = __ballot_sync(0xffffffffu, raise != 0);
    while (mk) {
        const int src = __ffs(mk) - 1;
        mk &= mk - 1;
        const int W = __shfl_sync(0xffffffffu, raise, src);
        const int qq = __shfl_sync(0xffffffffu, q, src);
        const uint64_t T =
            warp_kth_window(a.pool + (int64_t)qq * a.pool_cap + (W > RAISE_WINDOW ? W - RAISE_WINDOW : 0),
                            W > RAISE_WINDOW ? RAISE_WINDOW : W, a.k, hist);
        if (lane == 0) atomicAdd(&a.status[3], 1);
        if (lane == 0 && T != 0ull) {
            atomicMax(reinterpret_cast<unsigned long long*>(&a.tau_global[qq]),
                      (unsigned long long)T);
            atomicMax(reinterpret_cast<unsigned long long*>(&ctl->tau[qq]), (unsigned long long)T);
        }
        __syncwarp();
    }
    __syncwarp();
}

// One cluster of two CTAs per pair of SMs; the pair scores 256-row tiles
// against all 256 queries with one tcgen05.mma.cta_group::2 of M = 256
// queries (128 resident in each CTA) x N = 256 rows (128 staged in each CTA)
// per K = 16 slice, so each SM's tensor core reads half of the row operand
// it would read alone.  D lands in TMEM as query (lane) x row (column).
// Roles in each CTA (16 warps, so that each SM sub-partition holds four
// warps of up to 128 registers):
//   warp 0      TMA producer: the CTA's 128 queries once, then its 128 rows of
//               each tile (two 64-column boxes, 128-byte swizzle), 5 stages
//   warps 1, 3  first CTA: MMA issuers (one lane each; even and odd tiles),
//               8 pair MMAs per tile into one of two accumulators of 256 fp32
//               columns, committed to both CTAs' accumulator barriers;
//   warp 1      second CTA: forwards each landing of its queries and rows
//               onto the first CTA's barriers
//   warp 2      TMEM allocator (both CTAs), then a rescorer
//   warps 4-5   row bounds: max|a| over the CTA's 128 rows of a landed tile,
//               stored with the tile number into both CTAs (one 8-byte store
//               each, polled by the epilogue)
//   warps 8-15  epilogue, two warpgroups: warpgroup h reads the columns of
//               the rows staged by CTA h; thread = query (TMEM lane), with its
//               own threshold less its error bound in a register; a 3-input
//               max tree per 32 columns; pairs that reach it are published to
//               the warp's ring
//   warps 2, 3, 6, 7  rescorers (first CTA: 2, 6, 7): exact rescoring of the rings' pairs, pools,
//               threshold raises, and the refresh of thresholds that other
//               clusters raised
// A pair (row r, query q) can beat q's threshold t only if its exact score
// s >= score(t); |s~ - s| <= EPS * max_j|a_rj| * sum_j|b_qj| <= EPS * M_h * L1_q
// (M_h = max over the tile half's rows), so the epilogue passes every pair
// with s~ >= score(t) - EPS * M_h * L1_q (rounded down); NaN passes.
//
// SAMPLE = true is the sample pass that precedes the scoring pass: the same
// pipeline over sample_tiles pair tiles spread evenly over the shard, with no
// rescoring.  Each epilogue thread keeps the SAMPLE_M largest lower bounds
// s~ - EPS * M_h * L1_q (rounded down) of its query over the rows it sees
// and writes them to sample_lb; every bound is <= the exact score of a
// distinct row, so the k-th largest of all of them is <= the k-th best exact
// score of the shard (sample_tau_kernel turns it into the starting threshold).
template <bool SAMPLE>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NTHREADS, 1)
tc_score_select_kernel(const __grid_constant__ CUtensorMap tmR,
                       const __grid_constant__ CUtensorMap tmQ, const TcArgs a) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // 1024-byte aligned base, derived by pointer arithmetic so that the
    // compiler keeps every access below in the shared address space; both
    // CTAs get the same offsets, which the pair MMAs rely on
    unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    unsigned char* Qs = smem;
    unsigned char* Rs = Qs + Q_BYTES;
    Ctrl* ctl = reinterpret_cast<Ctrl*>(Rs + STAGES * ROW_STAGE);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t crank = cluster_ctarank();   // 0: issues the pair's MMAs
    const uint32_t peer = crank ^ 1u;
    const int cl = (int)blockIdx.x >> 1, ncl = (int)gridDim.x >> 1;
    const int v_tiles = SAMPLE ? a.sample_tiles : a.n_tiles;
    const int my_tiles = cl < v_tiles ? (v_tiles - 1 - cl) / ncl + 1 : 0;
    // pair tile of this cluster's i-th iteration (the sample pass spreads its
    // tiles evenly over the shard)
    auto tile_of = [&](int i) -> int64_t {
        const int j = cl + i * ncl;
        return SAMPLE ? (int64_t)j * a.n_tiles / a.sample_tiles : (int64_t)j;
    };
    const int q0 = (int)crank * PQ;             // this CTA's first query
    volatile int* abort = &ctl->abort;

    if (threadIdx.x == 0) {
        const uint32_t landings = crank == 0 ? 2 : 1;   // own copy (+ the peer's, forwarded)
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&ctl->full[s], landings);
            mbar_init(&ctl->empty[s], 32 * N_RB_WARPS + 1);   // row-bound threads + an epilogue thread
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&ctl->acc_full[b], 1);
            mbar_init(&ctl->acc_empty[b], 2 * N_EPI_WARPS);   // every epilogue warp of the pair
        }
        mbar_init(&ctl->q_full, landings);
        ctl->abort = 0;
        ctl->issued = 0;
        for (int e = 0; e < N_EPI_WARPS; ++e) {
            ctl->ring_head[e] = 0;
            ctl->ring_tail[e] = 0;
            ctl->epi_done[e] = 0;
        }
        fence_barrier_init();
    }
    for (int q = threadIdx.x; q < TC_NMAX; q += NTHREADS)
        ctl->tau[q] = q < a.nq ? a.tau_global[q] : ~0ull;
    for (int e = threadIdx.x; e < MR_RING * 2 * N_RB_WARPS; e += NTHREADS)
        (&ctl->mr[0][0][0])[e] = 0ull;   // tag 0: no tile
    if (warp == 2) {
        tmem_alloc_pair(&ctl->tmem_base, TMEM_COLS);
        tmem_relinquish_pair();
    }
    // both CTAs' barriers and slots initialised and TMEM allocated before any
    // remote arrive, remote store or pair MMA
    tc_fence_before();
    cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem = ctl->tmem_base;

    if (warp == 0) {
        // ------------------------------------------------------ TMA producer
        if (lane == 0) {
            prefetch_tmap(&tmR);
            prefetch_tmap(&tmQ);
            mbar_expect_tx(&ctl->q_full, Q_BYTES);
            tma_load_2d(Qs, &tmQ, &ctl->q_full, 0, q0);
            tma_load_2d(Qs + Q_BOX, &tmQ, &ctl->q_full, 64, q0);
        }
        int issued = 0;
        for (int i = 0; i < my_tiles; ++i) {
            const int s = i % STAGES;
            if (!warp_wait(&ctl->empty[s], ((i / STAGES) & 1) ^ 1, abort, a.wait_ns)) {
                if (lane == 0) set_abort(ctl, a.status, peer);
                break;
            }
            if (lane == 0) {
                const int y = (int)(a.row_begin + (tile_of(i) * 2 + crank) * PR);
                mbar_expect_tx(&ctl->full[s], ROW_STAGE);
                tma_load_2d(Rs + s * ROW_STAGE, &tmR, &ctl->full[s], 0, y);
                tma_load_2d(Rs + s * ROW_STAGE + ROW_BOX, &tmR, &ctl->full[s], 64, y);
            }
            __syncwarp();
            issued = i + 1;
        }
        if (!*abort) {
            // tail: the MMA commits that release the last stages arrive before
            // the CTA exits (nothing may arrive on a CTA that has exited)
            for (int i = max(0, issued - STAGES); i < issued; ++i)
                if (!warp_wait(&ctl->empty[i % STAGES], (i / STAGES) & 1, abort, a.wait_ns)) {
                    if (lane == 0) set_abort(ctl, a.status, peer);
                    break;
                }
        }
        if (*abort) {
            // drain: the latest arming of each stage must land before exit.  In
            // the first CTA a stage's phase also counts the peer's forwarded
            // landing, which a forwarder that gave up never sends, so all the
            // stages share one budget (a copy lands within microseconds; the
            // budget is a thousand times that) instead of one each
            const uint64_t t_end = globaltimer_ns() + DRAIN_NS;
            auto left = [&]() -> uint64_t {
                const uint64_t now = globaltimer_ns();
                return now < t_end ? t_end - now : 0ull;
            };
            for (int i = max(0, issued - STAGES); i < issued; ++i)
                mbar_wait_drain(&ctl->full[i % STAGES], (i / STAGES) & 1, left());
            mbar_wait_drain(&ctl->q_full, 0, left());
            // the pair MMAs already issued commit to this CTA's barriers after
            // they complete; their arrivals land well within this pause, before
            // the CTA can exit
            const uint64_t t0 = globaltimer_ns();
            while (globaltimer_ns() - t0 < 50000ull) __nanosleep(1000);
        }
    } else if (warp == 1 || (warp == 3 && crank == 0)) {
        // ------------------------------------------ MMA issuers (first CTA)
        // Two threads, lane 0 of warps 1 and 3: warp 1 issues the even tiles
        // (accumulator 0), warp 3 the odd ones (accumulator 1).  A pair MMA
        // holds its issuing thread for about its own execution time, so while
        // one thread waits for its next tile's barriers and commits, the
        // other keeps the tensor core busy.  They take turns (ctl->issued):
        // a tile's MMAs enter the tensor core's queue whole and in tile
        // order, so no tile waits behind half of the next one.  A commit
        // tracks only its own thread's MMAs; the two threads share no
        // accumulator and no stage phase.
        if (crank == 0 && lane == 0) {
            const int par = warp == 1 ? 0 : 1;
            const uint32_t idesc = idesc_f16(2 * PQ, 2 * PR, 1);
            const uint32_t qa = smem_u32(Qs);
            const uint32_t d = tmem + (uint32_t)(par * 2 * PR);
            const uint32_t f_loc = smem_u32(&ctl->acc_full[par]);
            const uint32_t f_peer = mapa_shared(f_loc, 1);
            int last = -1;
            bool ok = mbar_wait_bounded(&ctl->q_full, 0, abort, a.wait_ns);   // both CTAs' queries
            for (int i = par; ok && i < my_tiles; i += 2) {
                const int s = i % STAGES;
                // both CTAs' rows of tile i landed; both epilogues released the accumulator
                if (!mbar_wait_bounded(&ctl->full[s], (i / STAGES) & 1, abort, a.wait_ns) ||
                    !mbar_wait_bounded(&ctl->acc_empty[par], ((i >> 1) & 1) ^ 1, abort, a.wait_ns)) {
                    ok = false;
                    break;
                }
                // this thread's turn: the other has issued every MMA of tile i - 1
                if (ld_volatile(&ctl->issued) != i) {
                    const uint64_t t0 = globaltimer_ns();
                    while (ld_volatile(&ctl->issued) != i) {
                        if (*abort || globaltimer_ns() - t0 >= a.wait_ns) { ok = false; break; }
                    }
                    if (!ok) break;
                }
                tc_fence_after();
                const uint32_t ra = smem_u32(Rs + s * ROW_STAGE);
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks)
                        mma_f16_pair(d, desc_k_sw128(qa + h * Q_BOX + ks * 32),
                                     desc_k_sw128(ra + h * ROW_BOX + ks * 32), idesc,
                                     (h | ks) != 0);
                st_volatile(&ctl->issued, i + 1);   // the other thread's turn
                // the accumulator of both CTAs (each epilogue then releases its
                // CTA's stage: the MMAs that read it have completed)
                mma_commit_pair(f_loc);
                mma_commit_pair(f_peer);
                last = i;
            }
            // tail: both CTAs' epilogues have released this thread's last
            // accumulator (their arrivals on this CTA's barrier have landed)
            if (ok && last >= 0)
                ok = mbar_wait_bounded(&ctl->acc_empty[par], (last >> 1) & 1, abort, a.wait_ns);
            if (!ok) set_abort(ctl, a.status, peer);
            if (*abort && last >= 0)   // the MMAs issued must finish before TMEM is freed
                mbar_wait_drain(&ctl->acc_full[par], (last >> 1) & 1);
        } else if (crank != 0) {
            // ------------------------- forwarder (second CTA): each landing of
            // this CTA's queries and rows, onto the first CTA's barriers
            bool ok = warp_wait(&ctl->q_full, 0, abort, a.wait_ns);
            if (ok && lane == 0) mbar_arrive_remote(mapa_shared(smem_u32(&ctl->q_full), 0));
            for (int i = 0; ok && i < my_tiles; ++i) {
                const int s = i % STAGES;
                ok = warp_wait(&ctl->full[s], (i / STAGES) & 1, abort, a.wait_ns);
                if (ok && lane == 0) mbar_arrive_remote(mapa_shared(smem_u32(&ctl->full[s]), 0));
            }
            if (!ok && lane == 0) set_abort(ctl, a.status, peer);
        }
    } else if (warp >= 4 && warp < 4 + N_RB_WARPS) {
        // ---------------------------------------------------- row-bound warps
        const int w4 = warp - 4;
        const int r = w4 * 64 + lane;   // and r + 32
        bool ok = true;
        for (int i = 0; ok && i < my_tiles; ++i) {
            const int s = i % STAGES;
            if (!warp_wait(&ctl->full[s], (i / STAGES) & 1, abort, a.wait_ns)) {
                ok = false;
                break;
            }
            const uint32_t m = rows_absmax_bits(Rs + s * ROW_STAGE, r);   // rows past the end are 0
            mbar_arrive(&ctl->empty[s]);                                 // smem reads of this tile done
            const uint32_t wm = __reduce_max_sync(0xffffffffu, m);      // >= 0: int order = float order
            if (lane == 0) {
                const uint64_t v = ((uint64_t)(uint32_t)(i + 1) << 32) | wm;
                uint64_t* slot = &ctl->mr[i % MR_RING][crank][w4];
                *reinterpret_cast<volatile uint64_t*>(slot) = v;
                st_cluster_u64(mapa_shared(smem_u32(slot), peer), v);
            }
            __syncwarp();
        }
        if (!ok && lane == 0) set_abort(ctl, a.status, peer);
    } else if (warp >= 8 && warp < 16) {
        // --------------------------------------------------------- epilogue
        const int ew = warp - 8;            // 0..7
        const int hh = ew >> 2;             // row half: the columns of CTA hh's rows
        const int sub = warp & 3;           // TMEM lanes 32*sub .. +31
        const int q = q0 + sub * 32 + lane; // query of this thread
        const bool qvalid = q < a.nq;
        float l1 = 0.0f;                    // sum_j |b_qj|, rounded up
        if (qvalid) {
            const uint4* qp = reinterpret_cast<const uint4*>(a.qry + (int64_t)q * TC_DIM);
#pragma unroll 4
            for (int c = 0; c < 16; ++c) {
                const uint4 v = __ldg(qp + c);
                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int t = 0; t < 4; ++t)
                    l1 = __fadd_ru(__fadd_ru(l1, fabsf(bf_lo(w[t]))), fabsf(bf_hi(w[t])));
            }
        }
        if constexpr (SAMPLE) {
            // the SAMPLE_M largest lower bounds of this query over the rows of
            // this cluster's sample tiles in row half hh, in descending order
            float lbs[SAMPLE_M];
#pragma unroll
            for (int j = 0; j < SAMPLE_M; ++j) lbs[j] = -INFINITY;
            for (int i = 0; i < my_tiles; ++i) {
                const int b = i & 1, e = i % MR_RING;
                if (!warp_wait(&ctl->acc_full[b], (i >> 1) & 1, abort, a.wait_ns)) {
                    if (lane == 0) set_abort(ctl, a.status, peer);
                    break;
                }
                tc_fence_after();
                if (ew == 0 && lane == 0) mbar_arrive(&ctl->empty[i % STAGES]);
                uint64_t v0 = 0, v1 = 0;
                {
                    const uint32_t tag = (uint32_t)(i + 1);
                    const volatile uint64_t* sl = &ctl->mr[e][hh][0];
                    bool ready = false;
                    uint64_t t0 = 0;
                    for (int it = 0;; ++it) {
                        if (lane == 0) { v0 = sl[0]; v1 = sl[1]; }
                        v0 = __shfl_sync(0xffffffffu, v0, 0);
                        v1 = __shfl_sync(0xffffffffu, v1, 0);
                        if ((uint32_t)(v0 >> 32) == tag && (uint32_t)(v1 >> 32) == tag) { ready = true; break; }
                        if (it == 0) t0 = globaltimer_ns();
                        if (*abort || globaltimer_ns() - t0 >= a.wait_ns) break;
                        __nanosleep(32);
                    }
                    if (!ready) {
                        if (lane == 0) set_abort(ctl, a.status, peer);
                        break;
                    }
                }
                const float mh = fmaxf(__uint_as_float((uint32_t)v0), __uint_as_float((uint32_t)v1));
                const float marg = tc_margin(mh, l1);
                // |partial sums| <= M_h * L1_q <= 2^110: neither order overflows,
                // so the error bound holds (a larger or NaN bound is skipped)
                const bool use = qvalid && marg <= 0x1p100f;
                const uint32_t tbase =
                    tmem + (uint32_t)(b * 2 * PR + hh * PR) + ((uint32_t)(sub * 32) << 16);
                const int64_t half_row0 = a.row_begin + (tile_of(i) * 2 + hh) * PR;
#pragma unroll 1
                for (int c = 0; c < PR / 32; ++c) {
                    uint32_t v[32];
                    tmem_ld_x32(tbase + (uint32_t)(c * 32), v);
                    tmem_wait_ld();
                    const int64_t rem = a.n_rows - (half_row0 + c * 32);   // rows past the end
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const float sv = __uint_as_float(v[j]);
                        if (use && j < rem && fabsf(sv) <= 3.0e38f) {
                            const float lb = __fsub_rd(sv, marg);
                            if (lb > lbs[SAMPLE_M - 1]) {
                                lbs[SAMPLE_M - 1] = lb;
#pragma unroll
                                for (int t = SAMPLE_M - 1; t > 0; --t)
                                    if (lbs[t] > lbs[t - 1]) {
                                        const float x = lbs[t]; lbs[t] = lbs[t - 1]; lbs[t - 1] = x;
                                    }
                            }
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_remote(mapa_shared(smem_u32(&ctl->acc_empty[b]), 0));
            }
            // written whatever happened: the bounds of the tiles seen are valid
            if (qvalid) {
                uint64_t* out = a.sample_lb + (int64_t)q * (gridDim.x * SAMPLE_M) +
                                ((int64_t)cl * 2 + hh) * SAMPLE_M;
#pragma unroll
                for (int j = 0; j < SAMPLE_M; ++j)
                    out[j] = lbs[j] > -INFINITY ? (uint64_t)f32_key(lbs[j]) << 32 : 0ull;
            }
        }
        int tail = 0;        // pairs this warp has queued in its ring (warp-uniform)
        int published = 0;   // of those, pairs whose tail the rescorers can see
        bool ring_ok = true;
        for (int i = 0; !SAMPLE && i < my_tiles; ++i) {
            const int b = i & 1, e = i % MR_RING;
            // ---- accumulator ready -> the maxima of the four 32-column chunks
            if (!warp_wait(&ctl->acc_full[b], (i >> 1) & 1, abort, a.wait_ns)) {
                if (lane == 0) set_abort(ctl, a.status, peer);
                break;
            }
            tc_fence_after();
            // the MMAs that read this CTA's rows of tile i have completed
            if (ew == 0 && lane == 0) mbar_arrive(&ctl->empty[i % STAGES]);
            const uint32_t tbase =
                tmem + (uint32_t)(b * 2 * PR + hh * PR) + ((uint32_t)(sub * 32) << 16);
            static_assert(PR / 32 == 4, "four 32-column chunks per row half");
            float cm0 = 0.0f, cm1 = 0.0f, cm2 = 0.0f, cm3 = 0.0f;   // chunk maxima
#pragma unroll 1
            for (int c = 0; c < PR / 32; c += 2) {
                uint32_t v[64];   // two chunks per tcgen05.wait::ld
                tmem_ld_x32(tbase + (uint32_t)(c * 32), v);
                tmem_ld_x32(tbase + (uint32_t)(c * 32 + 32), v + 32);
                tmem_wait_ld();
                float mx2[2];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint32_t* w = v + 32 * h;
                    float m[11];
#pragma unroll
                    for (int j = 0; j < 10; ++j)
                        m[j] = max3_nan(__uint_as_float(w[3 * j]), __uint_as_float(w[3 * j + 1]),
                                        __uint_as_float(w[3 * j + 2]));
                    m[10] = max3_nan(__uint_as_float(w[30]), __uint_as_float(w[31]), __uint_as_float(w[31]));
                    const float m0 = max3_nan(m[0], m[1], m[2]), m1 = max3_nan(m[3], m[4], m[5]);
                    const float m2 = max3_nan(m[6], m[7], m[8]), m3 = max3_nan(m[9], m[10], m[10]);
                    mx2[h] = max3_nan(max3_nan(m0, m1, m2), m3, m3);
                }
                if (c == 0) { cm0 = mx2[0]; cm1 = mx2[1]; } else { cm2 = mx2[0]; cm3 = mx2[1]; }
            }
            // ---- then the tile half's row bounds (both row-bound warps of CTA
            // hh; tagged with the tile, polled, bounded): by now they are
            // normally there, so their latency hides behind the filter
            uint64_t v0 = 0, v1 = 0;
            {
                const uint32_t tag = (uint32_t)(i + 1);
                const volatile uint64_t* sl = &ctl->mr[e][hh][0];
                bool ready = false;
                uint64_t t0 = 0;
                for (int it = 0;; ++it) {
                    if (lane == 0) { v0 = sl[0]; v1 = sl[1]; }
                    v0 = __shfl_sync(0xffffffffu, v0, 0);
                    v1 = __shfl_sync(0xffffffffu, v1, 0);
                    if ((uint32_t)(v0 >> 32) == tag && (uint32_t)(v1 >> 32) == tag) { ready = true; break; }
                    if (it == 0) t0 = globaltimer_ns();
                    if (*abort || globaltimer_ns() - t0 >= a.wait_ns) break;
                    __nanosleep(32);
                }
                if (!ready) {
                    if (lane == 0) set_abort(ctl, a.status, peer);
                    break;
                }
            }
            const float mh = fmaxf(__uint_as_float((uint32_t)v0), __uint_as_float((uint32_t)v1));
            const float ts = tau_score(*reinterpret_cast<volatile uint64_t*>(&ctl->tau[q]));
            const float marg = tc_margin(mh, l1);
            // a margin past 2^100 means partial sums may overflow, where the
            // bound does not hold: then every pair passes (-inf included)
            const float theta =
                !qvalid ? INFINITY : (marg <= 0x1p100f ? __fsub_rd(ts, marg) : -INFINITY);
            // warp-uniform: chunks where some pair reaches theta (NaN passes)
            unsigned hitmask = (__any_sync(0xffffffffu, !(cm0 < theta)) ? 1u : 0u) |
                               (__any_sync(0xffffffffu, !(cm1 < theta)) ? 2u : 0u) |
                               (__any_sync(0xffffffffu, !(cm2 < theta)) ? 4u : 0u) |
                               (__any_sync(0xffffffffu, !(cm3 < theta)) ? 8u : 0u);
            // rare: re-read the hit chunks into per-chunk bit masks, release the
            // accumulator, and only then queue the (row, query) pairs, so that
            // queueing never holds up the next MMAs
            const int64_t half_row0 = a.row_begin + (tile_of(i) * 2 + hh) * PR;
            uint32_t hb0 = 0, hb1 = 0, hb2 = 0, hb3 = 0;
            for (unsigned hm = hitmask; hm != 0u; hm &= hm - 1u) {
                const int c = __ffs(hm) - 1;
                uint32_t bits = 0;
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {   // 16 columns at a time: fewer live registers
                    uint32_t v[16];
                    tmem_ld_x16(tbase + (uint32_t)(c * 32 + hf * 16), v);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        bits |= (uint32_t)(!(__uint_as_float(v[j]) < theta)) << (hf * 16 + j);
                }
                const int64_t rem = a.n_rows - (half_row0 + c * 32);   // rows past the end never pass
                bits &= rem >= 32 ? 0xffffffffu : (rem <= 0 ? 0u : (1u << rem) - 1u);
                if (!qvalid) bits = 0u;   // padded queries (a NaN row passes the compare)
                if (c == 0) hb0 = bits; else if (c == 1) hb1 = bits; else if (c == 2) hb2 = bits; else hb3 = bits;
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(mapa_shared(smem_u32(&ctl->acc_empty[b]), 0));
            for (int c = 0; hitmask != 0u && ring_ok && c < PR / 32; ++c) {
                if (!((hitmask >> c) & 1u)) continue;
                uint32_t bits = c == 0 ? hb0 : c == 1 ? hb1 : c == 2 ? hb2 : hb3;
                while (ring_ok && __any_sync(0xffffffffu, bits != 0)) {
                    const bool has = bits != 0;
                    const int j = has ? __ffs(bits) - 1 : 0;
                    bits &= bits - 1;
                    const unsigned mk = __ballot_sync(0xffffffffu, has);
                    const int n = __popc(mk);
                    // room in the ring: the rescorers free slots as they go (bounded
                    // wait; what is queued so far is published first, or the
                    // rescorers could not see it to free anything)
                    if (tail + n - ld_volatile(&ctl->ring_head[ew]) > RING) {
                        __syncwarp();
                        if (lane == 0) {
                            __threadfence_block();
                            st_volatile(&ctl->ring_tail[ew], tail);
                        }
                        published = tail;
                        const uint64_t t0 = globaltimer_ns();
                        while (tail + n - ld_volatile(&ctl->ring_head[ew]) > RING) {
                            if (*abort || globaltimer_ns() - t0 >= a.wait_ns) {
                                ring_ok = false;
                                break;
                            }
                            __nanosleep(64);
                        }
                        ring_ok = __all_sync(0xffffffffu, ring_ok);
                        if (!ring_ok) break;
                    }
                    if (has)
                        ctl->ring[ew][(tail + __popc(mk & ((1u << lane) - 1u))) % RING] =
                            ((uint64_t)(half_row0 + c * 32 + j) << 8) | (uint64_t)q;
                    tail += n;   // published once per tile, below
                }
            }
            if (tail != published) {   // this tile's pairs
                if (lane == 0) {
                    __threadfence_block();
                    st_volatile(&ctl->ring_tail[ew], tail);
                }
                published = tail;
            }
            if (!ring_ok) {
                if (lane == 0) set_abort(ctl, a.status, peer);
                break;
            }
        }
        __syncwarp();
        if (lane == 0) {
            __threadfence_block();
            st_volatile(&ctl->epi_done[ew], 1);   // after its last published pair
        }
    } else if (!SAMPLE && (warp == 2 || warp == 3 || warp == 6 || warp == 7)) {
        // ------------------------------------------------------- rescorers
        // Exact rescoring of the epilogue warps' pairs, off the accumulator
        // path.  The first CTA has three rescorers (warp 3 issues MMAs there),
        // the second four; rescorer c drains rings c, c + nres, ... gathering up
        // to 32 pairs across them into one batch (lane = pair), so that sparse
        // hits do not pay a batch's memory latency each.
        const int nres = crank == 0 ? 3 : 4;
        const int c = warp == 2 ? 0 : warp == 3 ? 3 : warp - 5;   // warps 6, 7 -> 1, 2
        const int nr = (N_EPI_WARPS - c + nres - 1) / nres;       // rings of this rescorer
        int head[RPR_MAX];   // warp-uniform
#pragma unroll
        for (int e4 = 0; e4 < RPR_MAX; ++e4) head[e4] = 0;
        uint64_t last = globaltimer_ns();
        uint64_t refreshed = 0;
        // the rescorers read this CTA's queries from Qs: wait for their landing
        // here (its phase 0 completes once and for all)
        const bool q_ok = warp_wait(&ctl->q_full, 0, abort, a.wait_ns);
        if (!q_ok && lane == 0) set_abort(ctl, a.status, peer);
        for (; q_ok;) {
            // thresholds raised by other clusters (shared through tau_global),
            // copied here every REFRESH_NS: rescorer c refreshes the CTA's query
            // blocks of 32 numbered c, c + nres, ...
            const uint64_t now = globaltimer_ns();
            if (now - refreshed > REFRESH_NS) {
                refreshed = now;
                for (int j = c; j < PQ / 32; j += nres) {
                    const int q = q0 + j * 32 + lane;
                    if (q < a.nq) {
                        const uint64_t t = *reinterpret_cast<volatile uint64_t*>(&a.tau_global[q]);
                        if (t > ctl->tau[q])
                            atomicMax(reinterpret_cast<unsigned long long*>(&ctl->tau[q]),
                                      (unsigned long long)t);
                    }
                }
            }
            int avail[RPR_MAX];
            int total = 0;
#pragma unroll
            for (int e4 = 0; e4 < RPR_MAX; ++e4) {
                // one lane's read, shared: every lane sees the same count
                avail[e4] = e4 < nr ? __shfl_sync(0xffffffffu,
                                                  ld_volatile(&ctl->ring_tail[c + e4 * nres]), 0) -
                                          head[e4]
                                    : 0;
                total += avail[e4];
            }
            __threadfence_block();   // the entries published before those tails
            bool progress = false;
            if (total > 0) {
                const int m = min(total, 32);
                // lane l takes the l-th pending pair in ring order
                int off = lane, er = 0;
#pragma unroll
                for (int e4 = 0; e4 < RPR_MAX - 1; ++e4)
                    if (er == e4 && off >= avail[e4]) {
                        off -= avail[e4];
                        er = e4 + 1;
                    }
                const bool valid = lane < m;
                uint64_t entry = 0ull;
#pragma unroll
                for (int e4 = 0; e4 < RPR_MAX; ++e4)
                    if (valid && er == e4) entry = ctl->ring[c + e4 * nres][(head[e4] + off) % RING];
                __syncwarp();
                int rem = m;
#pragma unroll
                for (int e4 = 0; e4 < RPR_MAX; ++e4) {
                    const int take = min(avail[e4], rem);
                    rem -= take;
                    if (take > 0) {
                        head[e4] += take;
                        if (lane == 0) {
                            __threadfence_block();
                            st_volatile(&ctl->ring_head[c + e4 * nres], head[e4]);   // slots read: free them
                        }
                    }
                }
                rescore_batch(ctl, ctl->hist[c], entry, valid, m, a, Qs, q0);
                progress = true;
            }
            if (progress) {
                last = globaltimer_ns();
                continue;
            }
            // idle: done once every producer has finished and its ring is empty
            bool done = true;
#pragma unroll
            for (int e4 = 0; e4 < RPR_MAX; ++e4) {
                if (e4 >= nr) continue;
                const int e = c + e4 * nres;
                const bool fin = ld_volatile(&ctl->epi_done[e]) != 0;
                __threadfence_block();
                done = done && fin && ld_volatile(&ctl->ring_tail[e]) == head[e4];
            }
            if (__all_sync(0xffffffffu, done)) break;
            if (*abort) break;
            if (globaltimer_ns() - last >= a.wait_ns) {
                if (lane == 0) set_abort(ctl, a.status, peer);
                break;
            }
            __nanosleep(256);
        }
    }

    // every role of both CTAs has finished (each loop above is bounded) before
    // either CTA frees the TMEM or exits: the pair's MMAs, commits, remote
    // arrivals and stores all target both CTAs
    tc_fence_before();
    cluster_sync_all();
    tc_fence_after();
    if (warp == 2) tmem_dealloc_pair(tmem, TMEM_COLS);
}


// Starting threshold of each query from the sample pass's lower bounds
// (keys << 32, 0 = none): the k-th largest x of them bounds the shard's k-th
// best exact score from below, and (key(x) << 32) is below the composite of
// every row scoring >= x, so at least k composites exceed it.  Empties the
// query's pool.  One block of 256 threads per query.
__global__ void __launch_bounds__(256) sample_tau_kernel(const uint64_t* __restrict__ lb,
                                                         int n_lb, int k,
                                                         uint64_t* __restrict__ tau,
                                                         int* __restrict__ cnt) {
    __shared__ unsigned sm[300];
    const int q = blockIdx.x;
    const uint64_t T = block_select_threshold(lb + (int64_t)q * n_lb, n_lb, k, sm);
    if (threadIdx.x == 0) {
        tau[q] = T & 0xffffffff00000000ull;
        cnt[q] = 0;
    }
}

// Folds one pass's status words into a caller-owned device status word
// (asynchronous form): bit 2 = a bounded wait gave up, bit 3 = a candidate
// pool filled up (the pass's results are incomplete).
__global__ void status_fold_kernel(const int* __restrict__ status, int32_t* __restrict__ dev_status) {
    if (threadIdx.x == 0) {
        int bits = 0;
        if (status[0]) bits |= HMM_STATUS_TIMEOUT;
        if (status[1]) bits |= HMM_STATUS_POOL_OVERFLOW;
        if (bits) atomicOr(dev_status, bits);
    }
}

// ----------------------------------------------------------- host helpers

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// Row-major bf16 matrix [rows][128] as a 2-D tensor map with a
// {64 columns, box_rows rows} box and the 128-byte swizzle.
hmm_status_t make_tmap_bf16(CUtensorMap* m, const void* base, int64_t rows, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return set_error(HMM_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[2] = {(cuuint64_t)TC_DIM, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)TC_DIM * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                          strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(HMM_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return HMM_OK;
}

struct TcLayout {
    size_t pool, cnt, tau, status, sample_lb, total;
};

TcLayout tc_layout(int64_t nq_pass) {
    TcLayout L;
    auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
    size_t o = 0;
    L.pool = o; o += up(sizeof(uint64_t) * nq_pass * POOL_CAP);
    L.cnt = o; o += up(sizeof(int) * nq_pass);
    L.tau = o; o += up(sizeof(uint64_t) * nq_pass);
    L.status = o; o += up(sizeof(int) * 4);
    L.sample_lb = o; o += up(sizeof(uint64_t) * nq_pass * MAX_CTAS * SAMPLE_M);
    L.total = o;
    return L;
}

}  // namespace

bool tc_path_applies(int64_t n, int64_t dim, int64_t nq, int64_t k, const void* mem,
                     const void* qry) {
    return dim == TC_DIM && k >= 1 && k <= KMAX_TC && nq >= 1 && n > TC_MIN_ROWS &&
           (reinterpret_cast<uintptr_t>(mem) % 16) == 0 &&
           (reinterpret_cast<uintptr_t>(qry) % 16) == 0;
}

size_t tc_ws_bytes(int64_t n, int64_t nq, int64_t k) {
    (void)n; (void)k;
    return tc_layout(std::min<int64_t>(nq, TC_NMAX)).total + 256;
}

// Scores one shard on tensor cores and returns its exact top-k (int64 rows
// + row_offset, fp32 scores), query passes of at most 256.  With dev_status
// null the call reads each pass's status back (waiting for the stream) and
// recomputes a pass whose pool filled up on the exact CUDA-core path; with
// dev_status set it never waits, and ORs HMM_STATUS_TIMEOUT /
// HMM_STATUS_POOL_OVERFLOW into *dev_status instead.
hmm_status_t flat_bf16_tc(const uint16_t* mem, int64_t n, const uint16_t* qry, int64_t nq,
                          int64_t k, int64_t row_offset, int64_t* out_idx, float* out_scores,
                          void* ws, size_t ws_bytes, cudaStream_t st, int32_t* dev_status) {
    // tile coordinates (up to n + 255) stay int32
    HMM_REQUIRE(n < (int64_t(1) << 31) - 512, "n_rows must be < 2^31 - 512");
    HMM_CUDA_TRY(cudaFuncSetAttribute(tc_score_select_kernel<false>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TC_SMEM));
    HMM_CUDA_TRY(cudaFuncSetAttribute(tc_score_select_kernel<true>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TC_SMEM));
    CUtensorMap tmR;
    hmm_status_t s = make_tmap_bf16(&tmR, mem, n, PR);
    if (s != HMM_OK) return s;
    const int sms = device_sm_count();
    for (int64_t q0 = 0; q0 < nq; q0 += TC_NMAX) {
        const int nqp_pass = (int)std::min<int64_t>(TC_NMAX, nq - q0);
        const TcLayout L = tc_layout(nqp_pass);
        if (ws_bytes < L.total)
            return set_error(HMM_ERR_OOM, "workspace too small: %zu < %zu", ws_bytes, L.total);
        unsigned char* w = static_cast<unsigned char*>(ws);
        uint64_t* pool = reinterpret_cast<uint64_t*>(w + L.pool);
        int* cnt = reinterpret_cast<int*>(w + L.cnt);
        uint64_t* tau = reinterpret_cast<uint64_t*>(w + L.tau);
        int* status = reinterpret_cast<int*>(w + L.status);
        uint64_t* sample_lb = reinterpret_cast<uint64_t*>(w + L.sample_lb);
        const uint16_t* qp = qry + q0 * TC_DIM;

        // empty pool slots read as 0 (below every key) in threshold raises
        HMM_CUDA_TRY(cudaMemsetAsync(pool, 0, sizeof(uint64_t) * nqp_pass * POOL_CAP, st));
        HMM_CUDA_TRY(cudaMemsetAsync(status, 0, sizeof(int) * 4, st));

        CUtensorMap tmQ;
        s = make_tmap_bf16(&tmQ, qp, nqp_pass, PQ);
        if (s != HMM_OK) return s;
        {
            TcArgs a;
            a.n_rows = n;
            a.row_begin = 0;
            a.n_tiles = (int)((n + 2 * PR - 1) / (2 * PR));
            a.sample_tiles = 0;
            a.sample_lb = sample_lb;
            a.nq = nqp_pass;
            a.k = (int)k;
            a.pool_cap = POOL_CAP;
            a.wm0 = std::max(256, next_pow2(2 * (int)k));
            a.qry = qp;
            a.mem = mem;
            a.tau_global = tau;
            a.pool = pool;
            a.pool_cnt = cnt;
            a.status = status;
            a.wait_ns = wait_limit_ns();
            // clusters of two CTAs, one per pair of SMs
            const int ncl_max = std::max(1, std::min(sms, MAX_CTAS) / 2);

            // 1. sample pass: SAMPLE_TPC tiles per cluster spread over the shard
            //    (all of them for small shards) -> lower bounds -> starting
            //    thresholds, pools emptied
            a.sample_tiles = std::min(a.n_tiles, SAMPLE_TPC * ncl_max);
            const int grid_s = 2 * std::min(ncl_max, a.sample_tiles);
            tc_score_select_kernel<true><<<grid_s, NTHREADS, TC_SMEM, st>>>(tmR, tmQ, a);
            s = check_launch("tc_score_select_kernel<sample>");
            if (s != HMM_OK) return s;
            sample_tau_kernel<<<nqp_pass, 256, 0, st>>>(sample_lb, grid_s * SAMPLE_M, (int)k, tau,
                                                        cnt);
            s = check_launch("sample_tau_kernel");
            if (s != HMM_OK) return s;

            // 2. one scoring pass over every row, appending to the pools; the
            //    rescorers raise and share the thresholds as candidates arrive
            a.sample_tiles = 0;
            const int grid = 2 * std::min(ncl_max, a.n_tiles);
            const ProfileMark pm = profile_begin(st);
            tc_score_select_kernel<false><<<grid, NTHREADS, TC_SMEM, st>>>(tmR, tmQ, a);
            s = check_launch("tc_score_select_kernel");
            profile_end(pm, st);
            if (s != HMM_OK) return s;
        }

        s = launch_pool_merge(pool, POOL_CAP, cnt, nqp_pass, (int)k, row_offset,
                              out_idx + q0 * k, out_scores + q0 * k, st);
        if (s != HMM_OK) return s;

        if (dev_status) {
            status_fold_kernel<<<1, 32, 0, st>>>(status, dev_status);
            s = check_launch("status_fold_kernel");
            if (s != HMM_OK) return s;
            continue;
        }
        // The kernel reports a bounded wait that gave up (status[0]) and a
        // query whose candidate pool filled up (status[1]; only inputs whose
        // row order makes the running k-th best climb for thousands of rows,
        // e.g. rows sorted by score, get there).  A full pool means dropped
        // candidates, so that pass is recomputed on the exact CUDA-core path,
        // which needs no pool and fits the same workspace.
        int host_status[4] = {0, 0, 0, 0};
        HMM_CUDA_TRY(cudaMemcpyAsync(host_status, status, sizeof(host_status),
                                     cudaMemcpyDeviceToHost, st));
        HMM_CUDA_TRY(cudaStreamSynchronize(st));
        if (host_status[0] != 0)
            return set_error(HMM_ERR_TIMEOUT,
                             "tc_score_select_kernel: a bounded pipeline wait gave up; the "
                             "outputs of queries [%lld, %lld) are invalid",
                             (long long)q0, (long long)(q0 + nqp_pass));
        if (host_status[1] != 0) {
            s = flat_bf16_exact(mem, n, TC_DIM, qp, nqp_pass, k, row_offset, out_idx + q0 * k,
                                out_scores + q0 * k, ws, ws_bytes, st);
            if (s != HMM_OK) return s;
        }
    }
    return HMM_OK;
}

}  // namespace hmm
