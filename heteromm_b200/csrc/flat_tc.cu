// flat_tc.cu — tcgen05 (5th-gen tensor core) scoring of a bf16 row shard with
// exact top-k selection: the sharded flat-retrieval hot path (inner product
// of reference steps/example_kernel/inner_product_compute.cpp:11-31 fused
// with the top-k of topk_retrieval.cpp:13-31), bit-exact to the reference's
// sequential fp32 arithmetic.
//
// Tensor cores sum in their own order, so their scores are approximations.
// The kernel uses them only to decide which (row, query) pairs can matter:
//   s~ = tensor-core score of row r for query q (fp32 accumulate in TMEM)
//   |s~ - s| <= EPS * max_j|a_rj| * sum_j|b_qj|   (s = the reference's score)
// A pair is rescored exactly - fp32 multiply-add in ascending j from the row
// tile still resident in shared memory, which rounds exactly as the
// reference's separate multiply and add because bf16 products are exact in
// fp32 - only when its upper bound s~ + margin reaches the query's current
// threshold.  Exact (score, row) composites that beat the threshold enter a
// per-query candidate pool in global memory; each time a pool reaches a
// power-of-two fill mark, the warp that filled it computes the pool's k-th
// best composite and raises the query's threshold (a k-th best of a subset
// never exceeds the k-th best of the whole memory, so no true top-k row is
// ever dropped).  A final merge takes the exact top-k of each pool.
//
// The threshold is seeded with the exact top-k of the first SEED_ROWS rows
// (CUDA-core kernel of flat_topk.cu), so the first tiles already filter.
//
// The thresholds themselves are folded into the tensor-core accumulator: a
// ninth K = 16 MMA per tile adds -t'_q (t'_q = the query's threshold score
// rounded down to bf16), so the epilogue only needs a 3-input max tree over
// each row's folded scores against one per-row margin.  The kernel's thread
// roles are listed at the kernel.  Every mbarrier wait is bounded; a wait that
// gives up sets a status word and the CTA drains and exits.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "hmm_common.cuh"
#include "sm100_ptx.cuh"

namespace hmm {

// from flat_topk.cu: the exact CUDA-core path (seed sample and small shards)
hmm_status_t flat_bf16_exact(const uint16_t* mem, int64_t n, int64_t dim, const uint16_t* qry,
                             int64_t nq, int64_t k, int64_t row_offset, int64_t* out_idx,
                             float* out_scores, void* ws, size_t ws_bytes, cudaStream_t st);
size_t flat_bf16_exact_ws_bytes(int64_t n, int64_t nq, int64_t k);
hmm_status_t launch_pool_merge(const uint64_t* pool, int64_t cap, const int* counts, int nq,
                               int k, int64_t row_offset, int64_t* out_idx, float* out_scores,
                               cudaStream_t st);

namespace {

using namespace sm100;

constexpr int TC_M = 128;                      // rows per tile (MMA M)
constexpr int TC_NMAX = 256;                   // queries per pass (MMA N)
constexpr int TC_DIM = 128;                    // row width handled (MMA K total)
constexpr int STAGES = 4;
constexpr int A_BOX = TC_M * 128;              // 64 bf16 columns x 128 rows = 16 KiB
constexpr int A_STAGE = 2 * A_BOX;             // 32 KiB per tile
constexpr int Q_BOX = TC_NMAX * 128;           // 256 queries x 64 columns = 32 KiB
constexpr int Q_BYTES = 2 * Q_BOX;             // 64 KiB
constexpr int FA_BYTES = TC_M * 32;            // threshold-fold A operand: 128 rows x 16 bf16
constexpr int FB_BYTES = TC_NMAX * 32;         // threshold-fold B operand: 256 rows x 16 bf16
constexpr int N_EPI_WARPS = 8;                 // two epilogue warpgroups (query halves)
constexpr int NTHREADS = 32 * (10 + N_EPI_WARPS);   // + TMA, MMA, 4 rescorers, 4 row-bound warps
constexpr int RING = 128;                       // pairs per epilogue warp awaiting rescoring
constexpr int N_RESCORERS = 4;                  // warps 2, 3, 16 and 17
constexpr int RPR = N_EPI_WARPS / N_RESCORERS;  // rings per rescorer
constexpr int TMEM_COLS = 512;
constexpr float EPS = 1.0f / 1024.0f;          // >= 25x the worst-case summation gap
#ifndef HMM_SEED_ROWS
#define HMM_SEED_ROWS 8192
#endif
constexpr int SEED_ROWS = HMM_SEED_ROWS;
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
constexpr int MR_RING = 8;                     // tiles of row bounds in flight (>= STAGES + 2)
constexpr uint64_t REFRESH_NS = 2000;          // cadence of the rescorers' shared-threshold refresh

struct __align__(8) Ctrl {
    uint64_t a_full[STAGES];        // tile landed (TMA tx)
    uint64_t a_empty[STAGES];       // tile consumed: row-bound threads + MMA commit
    uint64_t acc_full[2];           // accumulator written (MMA commit)
    uint64_t acc_empty[2];          // accumulator drained by its epilogue warpgroup
    uint64_t b_full;                // queries landed
    uint64_t mr_full[MR_RING];      // row bounds of tile i published
    uint32_t tmem_base;
    int abort;
    float l1max;                    // max over queries of sum_j |b_qj|
    float tmax;                     // max |folded threshold| ever written to the fold operand
    uint64_t tau[TC_NMAX];          // CTA copy of each query's threshold composite
    uint64_t ring[N_EPI_WARPS][RING];    // (shard row << 8) | query, epilogue -> rescorer
    int ring_head[N_EPI_WARPS];          // consumed (rescorer)
    int ring_tail[N_EPI_WARPS];          // published (epilogue warp)
    int epi_done[N_EPI_WARPS];           // the epilogue warp has published its last pair
    unsigned hist[N_RESCORERS][256];
    float mrow[MR_RING][TC_M];      // EPS * max|a_r| per row of tile i
};

constexpr size_t TC_SMEM =
    1024 /* alignment slack */ + Q_BYTES + STAGES * A_STAGE + FA_BYTES + FB_BYTES + sizeof(Ctrl);

struct TcArgs {
    int64_t n_rows;
    int64_t row_begin;
    int n_tiles;             // 128-row tiles over [row_begin, n_rows)
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

__device__ __forceinline__ float tau_score(uint64_t t) {
    return t == 0ull ? -INFINITY : cand_score(t);
}

// max of three, NaN if any input is NaN.
__device__ __forceinline__ float max3_nan(float a, float b, float c) {
    float d;
    asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// Largest bf16 value <= x (round toward -inf), as fp32.
__device__ __forceinline__ float bf16_floor(float x) {
    const uint32_t u = __float_as_uint(x);
    uint32_t hi = u & 0xffff0000u;                         // truncation: toward 0
    if ((u & 0xffffu) != 0u && (u & 0x80000000u)) hi += 0x10000u;   // negative: away from 0
    return __uint_as_float(hi);
}

// The folded threshold t' = t_hi + t_lo <= t (the score part of threshold
// composite T) as two bf16: t_hi = bf16_floor(t), t_lo = bf16_floor(t - t_hi)
// (t - t_hi is exact in fp32), so t - t' < 2^-16 |t|.  Returns the packed
// bf16x2 (-t_hi, -t_lo) for K columns 0 and 1 of the fold B operand, and
// |t_hi| + |t_lo| in *mag (an empty threshold folds to +inf: nothing is filtered).
__device__ __forceinline__ uint32_t neg_fold_pair(uint64_t T, float* mag) {
    const float t = tau_score(T);
    if (!(t > -INFINITY)) { *mag = 0.0f; return 0x7f80u; }   // (+inf, +0)
    const float th = bf16_floor(t);
    const float tl = bf16_floor(t - th);
    *mag = fabsf(th) + fabsf(tl);
    return ((__float_as_uint(th) ^ 0x80000000u) >> 16) | ((__float_as_uint(tl) ^ 0x80000000u) & 0xffff0000u);
}

// Writes query q's folded threshold into the fold B operand (row q, K
// columns 0-1 as one 4-byte store, so a concurrent MMA sees the old or the
// new pair, both <= the current threshold; 32-byte swizzle: 16-byte chunk c
// of row q sits at c ^ ((q >> 2) & 1)).  The fold bound tmax is raised
// first, so no MMA can read a fold that the epilogue's margin does not cover.
__device__ __forceinline__ void write_fold(unsigned char* FB, Ctrl* ctl, int q, uint64_t T) {
    float mag;
    const uint32_t bits = neg_fold_pair(T, &mag);
    atomicMax(reinterpret_cast<int*>(&ctl->tmax), __float_as_int(__fmul_ru(mag, 1.0f + 1.0f / 1024.0f)));
    __threadfence_block();
    *reinterpret_cast<uint32_t*>(FB + q * 32 + ((((q >> 2) & 1)) << 4)) = bits;
    fence_proxy_async_smem();
}

// The reference's fp32 dot product of a memory row and a query, j
// ascending, both read from global memory (the row was just streamed and is
// in L2; the queries are small and stay cached).
__device__ __forceinline__ float exact_dot_rows(const uint16_t* __restrict__ row,
                                                const uint16_t* __restrict__ qrow) {
    float s = 0.0f;
    const uint4* rp = reinterpret_cast<const uint4*>(row);
    const uint4* qp = reinterpret_cast<const uint4*>(qrow);
#pragma unroll
    for (int c = 0; c < 16; ++c) {
        const uint4 a = __ldg(rp + c);
        const uint4 b = __ldg(qp + c);
        s = fmaf(bf_lo(a.x), bf_lo(b.x), s); s = fmaf(bf_hi(a.x), bf_hi(b.x), s);
        s = fmaf(bf_lo(a.y), bf_lo(b.y), s); s = fmaf(bf_hi(a.y), bf_hi(b.y), s);
        s = fmaf(bf_lo(a.z), bf_lo(b.z), s); s = fmaf(bf_hi(a.z), bf_hi(b.z), s);
        s = fmaf(bf_lo(a.w), bf_lo(b.w), s); s = fmaf(bf_hi(a.w), bf_hi(b.w), s);
    }
    return s;
}

// max_j |a_rj| over row r of a tile (chunk order is irrelevant).
__device__ __forceinline__ float row_absmax(const unsigned char* As, int r) {
    __nv_bfloat162 m = __floats2bfloat162_rn(0.0f, 0.0f);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint4* p = reinterpret_cast<const uint4*>(As + h * A_BOX + r * 128);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            uint4 a = p[c ^ (r & 7)];   // lanes of a quarter-warp hit distinct banks
            a.x &= 0x7fff7fffu; a.y &= 0x7fff7fffu; a.z &= 0x7fff7fffu; a.w &= 0x7fff7fffu;
            m = __hmax2(m, *reinterpret_cast<__nv_bfloat162*>(&a.x));
            m = __hmax2(m, *reinterpret_cast<__nv_bfloat162*>(&a.y));
            m = __hmax2(m, *reinterpret_cast<__nv_bfloat162*>(&a.z));
            m = __hmax2(m, *reinterpret_cast<__nv_bfloat162*>(&a.w));
        }
    }
    return fmaxf(__low2float(m), __high2float(m));
}

// Every lane polls (so each observes the phase itself); the warp proceeds
// only if all lanes saw it, keeping the warp converged either way.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          uint64_t limit) {
    const bool ok = mbar_wait_bounded(bar, parity, abort, limit);
    return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ void set_abort(Ctrl* ctl, int* status) {
    atomicExch(&ctl->abort, 1);
    atomicExch(&status[0], 1);
}

// Raises query q's CTA threshold to T (if higher) and refolds it.
__device__ __forceinline__ void raise_tau(Ctrl* ctl, unsigned char* FB, int q, uint64_t T) {
    const unsigned long long old =
        atomicMax(reinterpret_cast<unsigned long long*>(&ctl->tau[q]), (unsigned long long)T);
    if (T > old) write_fold(FB, ctl, q, T);
}

// Rescores one batch of up to 32 queued pairs exactly (lane = pair) and
// appends the ones that beat their query's threshold to the pools; raises
// thresholds at fill marks from the newest RAISE_WINDOW pool entries.
__device__ __noinline__ void rescore_batch(Ctrl* ctl, unsigned char* FB, unsigned* hist,
                                           uint64_t e, bool valid, int m, const TcArgs& a) {
    const int lane = threadIdx.x & 31;
    if (lane == 0) atomicAdd(&a.status[2], m);
    int q = 0, raise = 0;
    if (valid) {
        const int64_t row = (int64_t)(e >> 8);
        q = (int)(e & 255u);
        const float s = exact_dot_rows(a.mem + row * TC_DIM, a.qry + (int64_t)q * TC_DIM);
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
            warp_select_threshold(a.pool + (int64_t)qq * a.pool_cap + (W > RAISE_WINDOW ? W - RAISE_WINDOW : 0),
                                  W > RAISE_WINDOW ? RAISE_WINDOW : W, a.k, hist);
        if (lane == 0) atomicAdd(&a.status[3], 1);
        if (lane == 0 && T != 0ull) {
            atomicMax(reinterpret_cast<unsigned long long*>(&a.tau_global[qq]),
                      (unsigned long long)T);
            raise_tau(ctl, FB, qq, T);
        }
        __syncwarp();
    }
    __syncwarp();
}

__device__ __forceinline__ int ld_volatile(const int* p) { return *reinterpret_cast<const volatile int*>(p); }
__device__ __forceinline__ void st_volatile(int* p, int v) { *reinterpret_cast<volatile int*>(p) = v; }

// One persistent CTA per SM.  Roles (18 warps):
//   warp 0      TMA producer: the 256 queries once, then 128-row x 128-col bf16
//               tiles (two 64-column boxes, 128-byte swizzle) into a 4-stage ring
//   warp 1      MMA issuer: per tile, 8 x tcgen05.mma (M = 128 rows, N = 256
//               queries, K = 16) plus one K = 16 MMA that adds -t'_q (each
//               query's threshold, folded as a bf16 rounded down) into the same
//               TMEM accumulator (two accumulators of 256 fp32 columns)
//   warp 2      TMEM allocator, then (with warps 3, 16, 17) exact rescoring of
//               the pairs the epilogue publishes to per-warp rings, and the
//               refolding of thresholds that other CTAs raised
//   warps 4-7   row bounds: EPS * max|a_r| for each row of a landed tile; with
//               the MMA commit they free the tile's stage
//   warps 8-15  epilogue, two warpgroups on every tile, each over half of the
//               256 query columns (measured faster than one warpgroup per
//               tile): thread = row (TMEM lane); a 3-input max tree over the
//               row's 128 folded scores s~ - t'_q against the row's margin;
//               pairs that reach it are published to the warp's ring for the
//               rescorer warps, so rescoring never delays the accumulator release
__global__ void __launch_bounds__(NTHREADS, 1)
tc_score_select_kernel(const __grid_constant__ CUtensorMap tmA,
                       const __grid_constant__ CUtensorMap tmB, const TcArgs a) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // 1024-byte aligned base, derived by pointer arithmetic so that the
    // compiler keeps every access below in the shared address space
    unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    unsigned char* Qs = smem;
    unsigned char* As = Qs + Q_BYTES;
    unsigned char* FA = As + STAGES * A_STAGE;     // 1024-aligned
    unsigned char* FB = FA + FA_BYTES;
    Ctrl* ctl = reinterpret_cast<Ctrl*>(FB + FB_BYTES);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x;
    const int my_tiles = (int)blockIdx.x < a.n_tiles ? (a.n_tiles - 1 - (int)blockIdx.x) / G + 1 : 0;
    volatile int* abort = &ctl->abort;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&ctl->a_full[s], 1);
            mbar_init(&ctl->a_empty[s], TC_M + 1);   // row-bound threads + the MMA commit
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&ctl->acc_full[b], 1);
            mbar_init(&ctl->acc_empty[b], N_EPI_WARPS);   // every epilogue warp
        }
        mbar_init(&ctl->b_full, 1);
        for (int e = 0; e < MR_RING; ++e) mbar_init(&ctl->mr_full[e], 4);
        ctl->abort = 0;
        for (int e = 0; e < N_EPI_WARPS; ++e) {
            ctl->ring_head[e] = 0;
            ctl->ring_tail[e] = 0;
            ctl->epi_done[e] = 0;
        }
        ctl->l1max = 0.0f;
        ctl->tmax = 0.0f;
        fence_barrier_init();
    }
    // fold operands: A' = 1 in K column 0, B' = -t'_q in K column 0, zero elsewhere
    for (int i = threadIdx.x; i < (FA_BYTES + FB_BYTES) / 4; i += NTHREADS)
        reinterpret_cast<uint32_t*>(FA)[i] = 0u;
    __syncthreads();
    for (int r = threadIdx.x; r < TC_M; r += NTHREADS)   // (1.0, 1.0) in K columns 0-1
        *reinterpret_cast<uint32_t*>(FA + r * 32 + (((r >> 2) & 1) << 4)) = 0x3f803f80u;
    for (int q = threadIdx.x; q < TC_NMAX; q += NTHREADS) {
        float l1 = 0.0f;
        uint64_t t = ~0ull;   // padded queries: never selected (fold = -inf below)
        if (q < a.nq) {
            const uint16_t* p = a.qry + (int64_t)q * TC_DIM;
            for (int j = 0; j < TC_DIM; ++j) l1 += fabsf(bf16_bits_to_f32(p[j]));
            l1 *= 1.0f + 1.0f / 256.0f;   // covers the rounding of this sum
            t = a.tau_global[q];
            atomicMax(reinterpret_cast<int*>(&ctl->l1max), __float_as_int(l1));   // l1 >= 0
        }
        ctl->tau[q] = t;
        float mag = 0.0f;
        const uint32_t bits = q < a.nq ? neg_fold_pair(t, &mag) : 0xff80u;   // (-inf, +0)
        *reinterpret_cast<uint32_t*>(FB + q * 32 + (((q >> 2) & 1) << 4)) = bits;
        atomicMax(reinterpret_cast<int*>(&ctl->tmax), __float_as_int(__fmul_ru(mag, 1.0f + 1.0f / 1024.0f)));
    }
    fence_proxy_async_smem();
    if (warp == 2) {
        tmem_alloc(&ctl->tmem_base, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ctl->tmem_base;

    if (warp == 0) {
        // ------------------------------------------------------ TMA producer
        if (lane == 0) {
            prefetch_tmap(&tmA);
            prefetch_tmap(&tmB);
            mbar_expect_tx(&ctl->b_full, Q_BYTES);
            tma_load_2d(Qs, &tmB, &ctl->b_full, 0, 0);
            tma_load_2d(Qs + Q_BOX, &tmB, &ctl->b_full, 64, 0);
        }
        int issued = 0;
        for (int i = 0; i < my_tiles; ++i) {
            const int s = i % STAGES;
            if (!warp_wait(&ctl->a_empty[s], ((i / STAGES) & 1) ^ 1, abort, a.wait_ns)) {
                if (lane == 0) set_abort(ctl, a.status);
                break;
            }
            if (lane == 0) {
                const int y = (int)(a.row_begin + (int64_t)((int)blockIdx.x + i * G) * TC_M);
                mbar_expect_tx(&ctl->a_full[s], A_STAGE);
                tma_load_2d(As + s * A_STAGE, &tmA, &ctl->a_full[s], 0, y);
                tma_load_2d(As + s * A_STAGE + A_BOX, &tmA, &ctl->a_full[s], 64, y);
            }
            __syncwarp();
            issued = i + 1;
        }
        if (*abort) {
            // drain: the latest arming of each stage must land before exit
            for (int i = max(0, issued - STAGES); i < issued; ++i)
                mbar_wait_drain(&ctl->a_full[i % STAGES], (i / STAGES) & 1);
            mbar_wait_drain(&ctl->b_full, 0);
        }
    } else if (warp == 1) {
        // -------------------------------------------------------- MMA issuer
        const uint32_t idesc = idesc_f16(TC_M, TC_NMAX, 1);
        int last = -1;
        bool ok = warp_wait(&ctl->b_full, 0, abort, a.wait_ns);
        if (!ok && lane == 0) set_abort(ctl, a.status);
        for (int i = 0; ok && i < my_tiles; ++i) {
            const int s = i % STAGES, b = i & 1;
            if (!warp_wait(&ctl->a_full[s], (i / STAGES) & 1, abort, a.wait_ns) ||
                !warp_wait(&ctl->acc_empty[b], ((i >> 1) & 1) ^ 1, abort, a.wait_ns)) {
                if (lane == 0) set_abort(ctl, a.status);
                break;
            }
            tc_fence_after();
            if (lane == 0) {
                const uint32_t a0 = smem_u32(As + s * A_STAGE), q0 = smem_u32(Qs);
                const uint32_t d = tmem + (uint32_t)(b * TC_NMAX);
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks)
                        mma_f16(d, desc_k_sw128(a0 + h * A_BOX + ks * 32),
                                desc_k_sw128(q0 + h * Q_BOX + ks * 32), idesc, (h | ks) != 0);
                // fold: D[r][q] += 1 * (-t'_q)
                mma_f16(d, desc_k_sw32(smem_u32(FA)), desc_k_sw32(smem_u32(FB)), idesc, 1u);
                mma_commit(&ctl->acc_full[b]);
                mma_commit(&ctl->a_empty[s]);
            }
            __syncwarp();
            last = i;
        }
        if (*abort && last >= 0)   // the MMAs issued must finish before TMEM is freed
            mbar_wait_drain(&ctl->acc_full[last & 1], (last >> 1) & 1);
    } else if (warp >= 4 && warp < 8) {
        // ---------------------------------------------------- row-bound warps
        const int r = (warp - 4) * 32 + lane;
        for (int i = 0; i < my_tiles; ++i) {
            const int s = i % STAGES;
            if (!warp_wait(&ctl->a_full[s], (i / STAGES) & 1, abort, a.wait_ns)) {
                if (lane == 0) set_abort(ctl, a.status);
                break;
            }
            const int64_t row = a.row_begin + (int64_t)((int)blockIdx.x + i * G) * TC_M + r;
            const float e = row < a.n_rows ? __fmul_ru(EPS, row_absmax(As + s * A_STAGE, r)) : 0.0f;
            mbar_arrive(&ctl->a_empty[s]);       // smem reads of this tile are done
            ctl->mrow[i % MR_RING][r] = e;
            __syncwarp();
            if (lane == 0) mbar_arrive(&ctl->mr_full[i % MR_RING]);
        }
    } else if (warp >= 8 && warp < 16) {
        // --------------------------------------------------------- epilogue
        const int ew = warp - 8;            // 0..7
        const int g = ew >> 2;              // warpgroup: query columns 128g .. 128g + 127
        const int sub = warp & 3;           // TMEM lanes 32*sub .. +31
        const int r = sub * 32 + lane;      // tile row of this thread
        const int nchunks = min((a.nq + 31) / 32, 4 * g + 4);
        int tail = 0;        // pairs this warp has queued in its ring (warp-uniform)
        int published = 0;   // of those, pairs whose tail the rescorers can see
        bool ring_ok = true;
        for (int i = 0; i < my_tiles; ++i) {
            const int b = i & 1;
            // ---- off the critical path: the tile's row bounds are published
            if (!warp_wait(&ctl->mr_full[i % MR_RING], (i / MR_RING) & 1, abort, a.wait_ns)) {
                if (lane == 0) set_abort(ctl, a.status);
                break;
            }
            const int64_t tile_row0 = a.row_begin + (int64_t)((int)blockIdx.x + i * G) * TC_M;
            const bool valid = tile_row0 + r < a.n_rows;
            const float er = ctl->mrow[i % MR_RING][r];

            // ---- critical path: accumulator ready -> filter -> release
            if (!warp_wait(&ctl->acc_full[b], (i >> 1) & 1, abort, a.wait_ns)) {
                if (lane == 0) set_abort(ctl, a.status);
                break;
            }
            tc_fence_after();
            // |s~ - t' - (s - t')| <= EPS * (max|a_r| * sum|b_q| + |t'|) for every
            // query; a pair can beat its threshold only if s~ - t' >= -margin
            const float margin = __fmaf_ru(er, ctl->l1max, __fmul_ru(EPS, ctl->tmax));
            const float neg = valid ? -margin : INFINITY;   // rows past the end never pass
            const uint32_t tbase = tmem + (uint32_t)(b * TC_NMAX) + ((uint32_t)(sub * 32) << 16);
            // filter: one 32-column chunk per tcgen05.wait::ld (measured faster than
            // two), kept free of the rare hit path, which would slow every chunk
            unsigned hitmask = 0;   // warp-uniform: chunks where some pair reaches -margin
#pragma unroll 1
            for (int c = 4 * g; c < nchunks; ++c) {
                uint32_t v[32];
                tmem_ld_x32(tbase + (uint32_t)(c * 32), v);
                tmem_wait_ld();
                float m[11];
#pragma unroll
                for (int j = 0; j < 10; ++j)
                    m[j] = max3_nan(__uint_as_float(v[3 * j]), __uint_as_float(v[3 * j + 1]),
                                    __uint_as_float(v[3 * j + 2]));
                m[10] = max3_nan(__uint_as_float(v[30]), __uint_as_float(v[31]), __uint_as_float(v[31]));
                const float m0 = max3_nan(m[0], m[1], m[2]), m1 = max3_nan(m[3], m[4], m[5]);
                const float m2 = max3_nan(m[6], m[7], m[8]), m3 = max3_nan(m[9], m[10], m[10]);
                const float mx = max3_nan(max3_nan(m0, m1, m2), m3, m3);
                if (__any_sync(0xffffffffu, !(mx < neg))) hitmask |= 1u << c;   // NaN passes
            }
            // rare: re-read the hit chunks and queue their (row, query) pairs
            while (hitmask != 0u && ring_ok) {
                const int c = __ffs(hitmask) - 1;
                hitmask &= hitmask - 1u;
                uint32_t v[32];
                tmem_ld_x32(tbase + (uint32_t)(c * 32), v);
                tmem_wait_ld();
                uint32_t bits = 0;
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    bits |= (uint32_t)(!(__uint_as_float(v[j]) < neg)) << j;
                const int rem = a.nq - c * 32;
                bits &= rem >= 32 ? 0xffffffffu : (1u << rem) - 1u;
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
                            ((uint64_t)(tile_row0 + r) << 8) | (uint64_t)(c * 32 + j);
                    tail += n;   // published once per tile, below
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ctl->acc_empty[b]);
            if (tail != published) {   // this tile's pairs
                if (lane == 0) {
                    __threadfence_block();
                    st_volatile(&ctl->ring_tail[ew], tail);
                }
                published = tail;
            }
            if (!ring_ok) {
                if (lane == 0) set_abort(ctl, a.status);
                break;
            }
        }
        __syncwarp();
        if (lane == 0) {
            __threadfence_block();
            st_volatile(&ctl->epi_done[ew], 1);   // after its last published pair
        }
    } else if (warp == 2 || warp == 3 || warp >= 16) {
        // ------------------------------------------------------- rescorers
        // Exact rescoring of the epilogue warps' pairs, off the accumulator
        // path: rescorer c drains the rings of epilogue warps RPR*c .. RPR*c + RPR-1,
        // gathering up to 32 pairs across them into one batch (lane = pair), so
        // that sparse hits do not pay a batch's memory latency each.
        const int c = warp < 16 ? warp - 2 : warp - 14;
        int head[RPR];   // warp-uniform
#pragma unroll
        for (int e4 = 0; e4 < RPR; ++e4) head[e4] = 0;
        uint64_t last = globaltimer_ns();
        uint64_t refreshed = 0;
        for (;;) {
            // thresholds raised by other CTAs (shared through tau_global), refolded
            // here every REFRESH_NS so that the epilogue never waits on them
            const uint64_t now = globaltimer_ns();
            if (now - refreshed > REFRESH_NS) {
                refreshed = now;
#pragma unroll
                for (int j = 0; j < TC_NMAX / (32 * N_RESCORERS); ++j) {
                    const int q = c * (TC_NMAX / N_RESCORERS) + j * 32 + lane;
                    if (q < a.nq) {
                        const uint64_t t = *reinterpret_cast<volatile uint64_t*>(&a.tau_global[q]);
                        if (t > ctl->tau[q]) raise_tau(ctl, FB, q, t);
                    }
                }
            }
            int avail[RPR];
            int total = 0;
#pragma unroll
            for (int e4 = 0; e4 < RPR; ++e4) {
                // one lane's read, shared: every lane sees the same count
                avail[e4] = __shfl_sync(0xffffffffu, ld_volatile(&ctl->ring_tail[c * RPR + e4]), 0) -
                            head[e4];
                total += avail[e4];
            }
            __threadfence_block();   // the entries published before those tails
            bool progress = false;
            if (total > 0) {
                const int m = min(total, 32);
                // lane l takes the l-th pending pair in ring order
                int off = lane, er = 0;
#pragma unroll
                for (int e4 = 0; e4 < RPR - 1; ++e4)
                    if (er == e4 && off >= avail[e4]) {
                        off -= avail[e4];
                        er = e4 + 1;
                    }
                const bool valid = lane < m;
                uint64_t entry = 0ull;
#pragma unroll
                for (int e4 = 0; e4 < RPR; ++e4)
                    if (valid && er == e4) entry = ctl->ring[c * RPR + e4][(head[e4] + off) % RING];
                __syncwarp();
                int rem = m;
#pragma unroll
                for (int e4 = 0; e4 < RPR; ++e4) {
                    const int take = min(avail[e4], rem);
                    rem -= take;
                    if (take > 0) {
                        head[e4] += take;
                        if (lane == 0) {
                            __threadfence_block();
                            st_volatile(&ctl->ring_head[c * RPR + e4], head[e4]);   // slots read: free them
                        }
                    }
                }
                rescore_batch(ctl, FB, ctl->hist[c], entry, valid, m, a);
                progress = true;
            }
            if (progress) {
                last = globaltimer_ns();
                continue;
            }
            // idle: done once every producer has finished and its ring is empty
            bool done = true;
#pragma unroll
            for (int e4 = 0; e4 < RPR; ++e4) {
                const int e = c * RPR + e4;
                const bool fin = ld_volatile(&ctl->epi_done[e]) != 0;
                __threadfence_block();
                done = done && fin && ld_volatile(&ctl->ring_tail[e]) == head[e4];
            }
            if (__all_sync(0xffffffffu, done)) break;
            if (*abort) break;
            if (globaltimer_ns() - last >= a.wait_ns) {
                if (lane == 0) set_abort(ctl, a.status);
                break;
            }
            __nanosleep(256);
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 2) tmem_dealloc(tmem, TMEM_COLS);
}

// Seeds each query's pool with the exact top-k of the sample rows and sets
// its starting threshold to the k-th of them.
__global__ void seed_pool_kernel(const int64_t* __restrict__ seed_idx,
                                 const float* __restrict__ seed_sc, int nq, int k,
                                 uint64_t* __restrict__ pool, int pool_cap, int* __restrict__ cnt,
                                 uint64_t* __restrict__ tau) {
    const int q = blockIdx.x;
    __shared__ int m;
    if (threadIdx.x == 0) m = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
        const int64_t r = seed_idx[(int64_t)q * k + i];
        if (r >= 0) {
            pool[(int64_t)q * pool_cap + i] = make_cand(f32_key(seed_sc[(int64_t)q * k + i]),
                                                        (uint32_t)r);
            atomicAdd(&m, 1);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        cnt[q] = m;
        tau[q] = m == k ? pool[(int64_t)q * pool_cap + k - 1] : 0ull;
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
    size_t pool, cnt, tau, status, seed_idx, seed_sc, seed_ws, total;
};

TcLayout tc_layout(int64_t n, int64_t nq_pass, int64_t k) {
    TcLayout L;
    auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
    size_t o = 0;
    L.pool = o; o += up(sizeof(uint64_t) * nq_pass * POOL_CAP);
    L.cnt = o; o += up(sizeof(int) * nq_pass);
    L.tau = o; o += up(sizeof(uint64_t) * nq_pass);
    L.status = o; o += up(sizeof(int) * 4);
    L.seed_idx = o; o += up(sizeof(int64_t) * nq_pass * k);
    L.seed_sc = o; o += up(sizeof(float) * nq_pass * k);
    L.seed_ws = o; o += up(flat_bf16_exact_ws_bytes(std::min<int64_t>(n, SEED_ROWS), nq_pass, k));
    L.total = o;
    return L;
}

}  // namespace

bool tc_path_applies(int64_t n, int64_t dim, int64_t nq, int64_t k, const void* mem,
                     const void* qry) {
    return dim == TC_DIM && k >= 1 && k <= KMAX_TC && nq >= 1 && n > SEED_ROWS &&
           (reinterpret_cast<uintptr_t>(mem) % 16) == 0 &&
           (reinterpret_cast<uintptr_t>(qry) % 16) == 0;
}

size_t tc_ws_bytes(int64_t n, int64_t nq, int64_t k) {
    return tc_layout(n, std::min<int64_t>(nq, TC_NMAX), k).total + 256;
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
    HMM_REQUIRE(n < (int64_t(1) << 31), "n_rows must be < 2^31");
    HMM_CUDA_TRY(cudaFuncSetAttribute(tc_score_select_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TC_SMEM));
    const int64_t seed = std::min<int64_t>(n, SEED_ROWS);
    CUtensorMap tmA;
    hmm_status_t s = make_tmap_bf16(&tmA, mem, n, TC_M);
    if (s != HMM_OK) return s;
    const int sms = device_sm_count();
    for (int64_t q0 = 0; q0 < nq; q0 += TC_NMAX) {
        const int nqp_pass = (int)std::min<int64_t>(TC_NMAX, nq - q0);
        const TcLayout L = tc_layout(n, nqp_pass, k);
        if (ws_bytes < L.total)
            return set_error(HMM_ERR_OOM, "workspace too small: %zu < %zu", ws_bytes, L.total);
        unsigned char* w = static_cast<unsigned char*>(ws);
        uint64_t* pool = reinterpret_cast<uint64_t*>(w + L.pool);
        int* cnt = reinterpret_cast<int*>(w + L.cnt);
        uint64_t* tau = reinterpret_cast<uint64_t*>(w + L.tau);
        int* status = reinterpret_cast<int*>(w + L.status);
        int64_t* seed_idx = reinterpret_cast<int64_t*>(w + L.seed_idx);
        float* seed_sc = reinterpret_cast<float*>(w + L.seed_sc);
        const uint16_t* qp = qry + q0 * TC_DIM;

        HMM_CUDA_TRY(cudaMemsetAsync(pool, 0, sizeof(uint64_t) * nqp_pass * POOL_CAP, st));
        HMM_CUDA_TRY(cudaMemsetAsync(status, 0, sizeof(int) * 4, st));
        s = flat_bf16_exact(mem, seed, TC_DIM, qp, nqp_pass, k, 0, seed_idx, seed_sc,
                            w + L.seed_ws, L.total - L.seed_ws, st);
        if (s != HMM_OK) return s;
        seed_pool_kernel<<<nqp_pass, 128, 0, st>>>(seed_idx, seed_sc, nqp_pass, (int)k, pool,
                                                    POOL_CAP, cnt, tau);
        s = check_launch("seed_pool_kernel");
        if (s != HMM_OK) return s;

        CUtensorMap tmB;
        s = make_tmap_bf16(&tmB, qp, nqp_pass, TC_NMAX);
        if (s != HMM_OK) return s;
        // One tensor-core pass over rows [seed, n), appending to the pools.  The
        // pools start from the seed's exact top-k, and the rescorers refresh the
        // shared threshold as candidates arrive, so one pass keeps hits sparse;
        // passes over growing row prefixes, each reseeded from the exact top-k
        // of the last, measured no faster at 8Mi-64Mi rows (slower below 32Mi).
        {
            TcArgs a;
            a.n_rows = n;
            a.row_begin = seed;
            a.n_tiles = (int)((n - seed + TC_M - 1) / TC_M);
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
            const int grid = std::max(1, std::min(sms, a.n_tiles));
            const ProfileMark pm = profile_begin(st);
            tc_score_select_kernel<<<grid, NTHREADS, TC_SMEM, st>>>(tmA, tmB, a);
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
