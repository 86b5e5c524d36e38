// flat_topk.cu — exact inner-product scoring fused with top-k and threshold
// selection on CUDA cores (reference steps/example_kernel/
// inner_product_compute.cpp:11-31, topk_retrieval.cpp:13-31,
// threshold_retrieval.cpp:11-32), plus the stand-alone top-k / threshold
// kernels on device-resident scores and the candidate merges.
//
// Layout in HBM: memory rows [n][dim] row-major (fp32 or bf16), queries
// [nq][dim].  One CTA owns QG=16 queries and a contiguous range of rows,
// which it streams through shared memory in tiles of RT=256 rows x KC=64
// columns.  Each thread keeps a 4-row x 4-query register tile; a dot product
// accumulates column-ascending exactly as the reference (fp32: separate
// multiply and add, both round-to-nearest; bf16: the product is exact in fp32
// so a fused multiply-add rounds identically).  After each row tile the CTA
// writes the threshold-bitmap words straight from warp ballots, and appends
// the (score, row) composites that beat its running per-query threshold to a
// shared-memory candidate buffer.  A full buffer is cut back to its top k with
// a warp radix select, which also raises the threshold.  Scores never leave
// the SM; each CTA emits k candidates per query, and one CTA per query
// merges them (block radix select + bitonic sort).
#include <algorithm>
#include <mutex>

#include "hmm_common.cuh"

namespace hmm {
namespace {

constexpr int NT = 256;     // threads per CTA
constexpr int QG = 16;      // queries per CTA
constexpr int RT = 256;     // rows per tile
constexpr int KC = 64;      // columns per shared-memory chunk
constexpr int SROW = KC + 4;  // padded row stride (floats): conflict-free float4 reads
constexpr int CAP = 512;    // candidate slots per query
constexpr int KMAX_FUSED = CAP - RT;  // largest k the fused kernel keeps
constexpr int NWARPS = NT / 32;

struct F32In {
    using T = float;
    static constexpr int VEC = 4;   // elements per 16-byte load
    __device__ static float widen1(const float* p) { return *p; }
    __device__ static float mac(float acc, float a, float b) { return __fadd_rn(acc, __fmul_rn(a, b)); }
};

struct BF16In {
    using T = uint16_t;
    static constexpr int VEC = 8;
    __device__ static float widen1(const uint16_t* p) { return bf16_bits_to_f32(*p); }
    // the product rounded before it is added, as the reference does: a bf16 x bf16
    // product is exact in fp32 only inside its normal range, so a fused
    // multiply-add would differ where a product overflows or underflows
    __device__ static float mac(float acc, float a, float b) { return __fadd_rn(acc, __fmul_rn(a, b)); }
};

size_t fused_smem_bytes(int dim) {
    const int dimp = (dim + 3) & ~3;
    return sizeof(float) * (size_t)(RT * SROW + QG * dimp) + sizeof(uint64_t) * (QG * CAP + QG) +
           sizeof(int) * QG + sizeof(unsigned) * NWARPS * 256;
}

struct Plan {
    int64_t rows_per_part;
    int n_parts;
    int n_qgroups;
};

// One CTA per SM (the kernel's shared memory allows no more): the CTAs of
// all query groups together form one wave.
Plan plan_fused(int64_t n, int64_t nq) {
    Plan p;
    p.n_qgroups = (int)((nq + QG - 1) / QG);
    const int64_t tiles = std::max<int64_t>(1, (n + RT - 1) / RT);
    const int64_t target = std::max<int64_t>(1, (int64_t)device_sm_count() / p.n_qgroups);
    const int64_t tiles_per_part = (tiles + target - 1) / target;
    p.rows_per_part = tiles_per_part * RT;
    p.n_parts = (int)((tiles + tiles_per_part - 1) / tiles_per_part);
    return p;
}

// Loads chunk [c0, c0+w) of rows [t0, t0+RT) into srow, widened to fp32 and
// zero padded to a multiple of 4 columns.  Zero padding leaves every sum
// unchanged: s + (+-0) == s for the +0-initialised accumulations used here.
template <typename In>
__device__ __forceinline__ void load_rows(float* srow, const typename In::T* __restrict__ mem,
                                          int64_t t0, int64_t r_end, int dim, int c0, int w,
                                          bool vec_ok) {
    const int wp = (w + 3) & ~3;
    if (vec_ok && (w % In::VEC) == 0) {
        const int per_row = w / In::VEC;
        // every load of this thread issued before any store: one memory round
        // trip per chunk instead of one per vector
        constexpr int MAXV = RT * (KC / In::VEC) / NT;
        uint4 v[MAXV];
#pragma unroll
        for (int u = 0; u < MAXV; ++u) {
            const int idx = threadIdx.x + u * NT;
            const int r = idx / per_row, j = (idx % per_row) * In::VEC;
            const int64_t row = t0 + r;
            v[u] = (idx < RT * per_row && row < r_end)
                       ? __ldg(reinterpret_cast<const uint4*>(mem + row * dim + c0 + j))
                       : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < MAXV; ++u) {
            const int idx = threadIdx.x + u * NT;
            if (idx >= RT * per_row) break;
            const int r = idx / per_row, j = (idx % per_row) * In::VEC;
            float* dst = srow + r * SROW + j;
            if constexpr (In::VEC == 4) {
                *reinterpret_cast<uint4*>(dst) = v[u];
            } else {
                float4 lo, hi;
                lo.x = __uint_as_float(v[u].x << 16); lo.y = __uint_as_float(v[u].x & 0xffff0000u);
                lo.z = __uint_as_float(v[u].y << 16); lo.w = __uint_as_float(v[u].y & 0xffff0000u);
                hi.x = __uint_as_float(v[u].z << 16); hi.y = __uint_as_float(v[u].z & 0xffff0000u);
                hi.z = __uint_as_float(v[u].w << 16); hi.w = __uint_as_float(v[u].w & 0xffff0000u);
                *reinterpret_cast<float4*>(dst) = lo;
                *reinterpret_cast<float4*>(dst + 4) = hi;
            }
        }
    } else {
        for (int idx = threadIdx.x; idx < RT * wp; idx += NT) {
            const int r = idx / wp, j = idx % wp;
            const int64_t row = t0 + r;
            srow[r * SROW + j] = (row < r_end && j < w) ? In::widen1(mem + row * dim + c0 + j) : 0.0f;
        }
    }
}

// Cuts query ql's candidate buffer back to its best k and raises its threshold.
__device__ __forceinline__ void compact_query(uint64_t* cbuf, int* scnt, uint64_t* sthr, int ql,
                                              int k, unsigned* hist) {
    const int m = scnt[ql];
    const uint64_t T = warp_select_threshold(cbuf + ql * CAP, m, k, hist);
    const int kept = warp_compact_ge(cbuf + ql * CAP, m, T);
    if ((threadIdx.x & 31) == 0) {
        scnt[ql] = kept;
        if (kept >= k) sthr[ql] = T;
    }
    __syncwarp();
}

// grid (n_parts, n_qgroups), NT threads.  cand [nq][n_parts][k] composites.
template <typename In>
__global__ void __launch_bounds__(NT, 1)
fused_ip_topk_kernel(const typename In::T* __restrict__ mem, int64_t n, int dim,
                     const typename In::T* __restrict__ qry, int nq, int k,
                     int64_t rows_per_part, float thr, uint32_t* __restrict__ bitmap32,
                     float* __restrict__ scores_out, uint64_t* __restrict__ cand, bool vec_ok) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int dimp = (dim + 3) & ~3;
    float* srow = reinterpret_cast<float*>(smem_raw);
    float* sq = srow + RT * SROW;
    uint64_t* cbuf = reinterpret_cast<uint64_t*>(sq + QG * dimp);
    uint64_t* sthr = cbuf + QG * CAP;
    int* scnt = reinterpret_cast<int*>(sthr + QG);
    unsigned* shist = reinterpret_cast<unsigned*>(scnt + QG);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int rg = tid & 63;          // rows rg + 64*i
    const int qg = tid >> 6;          // queries 4*qg .. 4*qg+3
    const int part = blockIdx.x;
    const int q0 = blockIdx.y * QG;
    const int64_t r_begin = (int64_t)part * rows_per_part;
    const int64_t r_end = min(n, r_begin + rows_per_part);
    const int64_t words32 = 2 * ((n + 63) / 64);

    for (int i = tid; i < QG * dimp; i += NT) {
        const int q = i / dimp, j = i % dimp;
        sq[i] = (q0 + q < nq && j < dim) ? In::widen1(qry + (int64_t)(q0 + q) * dim + j) : 0.0f;
    }
    if (tid < QG) { scnt[tid] = 0; sthr[tid] = 0ull; }

    for (int64_t t0 = r_begin; t0 < r_end; t0 += RT) {
        float acc[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;

        for (int c0 = 0; c0 < dim; c0 += KC) {
            const int w = min(KC, dim - c0);
            __syncthreads();
            load_rows<In>(srow, mem, t0, r_end, dim, c0, w, vec_ok);
            __syncthreads();
            const int wp = (w + 3) & ~3;
            for (int kk = 0; kk < wp; kk += 4) {
                float4 a[4], b[4];
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    a[i] = *reinterpret_cast<const float4*>(srow + (rg + 64 * i) * SROW + kk);
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    b[j] = *reinterpret_cast<const float4*>(sq + (4 * qg + j) * dimp + c0 + kk);
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        acc[i][j] = In::mac(acc[i][j], a[i].x, b[j].x);
                        acc[i][j] = In::mac(acc[i][j], a[i].y, b[j].y);
                        acc[i][j] = In::mac(acc[i][j], a[i].z, b[j].z);
                        acc[i][j] = In::mac(acc[i][j], a[i].w, b[j].w);
                    }
            }
        }

        // ---- tile epilogue: scores, threshold bitmap, candidates
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int64_t row = t0 + rg + 64 * i;
            const bool rv = row < r_end;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int ql = 4 * qg + j;
                const int q = q0 + ql;
                const bool v = rv && q < nq;
                const float s = acc[i][j];
                if (scores_out && v) scores_out[(int64_t)q * n + row] = s;
                if (bitmap32) {
                    const unsigned bits = __ballot_sync(0xffffffffu, v && s >= thr);
                    const int64_t w32 = ((t0 + 64 * i) >> 5) + (rg >> 5);
                    if (lane == 0 && q < nq && w32 < words32)
                        bitmap32[(int64_t)q * words32 + w32] = bits;
                }
                if (v && cand) {
                    const uint64_t c = make_cand(f32_key(s), (uint32_t)row);
                    if (c > sthr[ql]) {
                        const int pos = atomicAdd(&scnt[ql], 1);
                        cbuf[ql * CAP + pos] = c;
                    }
                }
            }
        }
        if (cand) {
            __syncthreads();
            for (int ql = warp; ql < QG; ql += NWARPS)
                if (scnt[ql] > CAP - RT) compact_query(cbuf, scnt, sthr, ql, k, shist + warp * 256);
            __syncthreads();
        }
    }
    if (!cand) return;

    // ---- final: top-k of each query's buffer -> cand
    const int n_parts = gridDim.x;
    for (int ql = warp; ql < QG; ql += NWARPS) {
        const int q = q0 + ql;
        if (q >= nq) continue;
        compact_query(cbuf, scnt, sthr, ql, k, shist + warp * 256);
        const int m = scnt[ql];
        uint64_t* dst = cand + ((int64_t)q * n_parts + part) * k;
        for (int i = lane; i < k; i += 32) dst[i] = i < m ? cbuf[ql * CAP + i] : 0ull;
    }
}

// Top-k over device scores: CTA (part, q) turns scores[q][part*P .. +P) into
// composites and keeps its best k.  cand [nq][n_parts][k].
constexpr int TOPK_P = 4096;
constexpr int TOPK_KMAX = 4096;

__global__ void __launch_bounds__(256)
scores_topk_partition_kernel(const float* __restrict__ scores, int64_t n, int k,
                             uint64_t* __restrict__ cand) {
    __shared__ uint64_t keys[TOPK_P];
    __shared__ unsigned sm[300];
    __shared__ int cnt;
    const int part = blockIdx.x, q = blockIdx.y;
    const int64_t r0 = (int64_t)part * TOPK_P;
    const int m = (int)(n - r0 < TOPK_P ? n - r0 : TOPK_P);
    const float* src = scores + (int64_t)q * n + r0;
    for (int i = threadIdx.x; i < m; i += 256) keys[i] = make_cand(f32_key(src[i]), (uint32_t)(r0 + i));
    if (threadIdx.x == 0) cnt = 0;
    __syncthreads();
    const int kk = min(k, m);
    const uint64_t T = block_select_threshold(keys, m, kk, sm);
    __syncthreads();
    uint64_t* dst = cand + ((int64_t)q * gridDim.x + part) * k;
    // keys are unique and nonzero: exactly kk of them are >= T
    for (int i = threadIdx.x; i < m; i += 256) {
        if (keys[i] >= T) dst[atomicAdd(&cnt, 1)] = keys[i];
    }
    for (int i = kk + threadIdx.x; i < k; i += 256) dst[i] = 0ull;
}

// First level of the candidate merge when the partitions left too many for
// one CTA per query: CTA (g, q) keeps the best k of cand[q][g*span ..
// g*span + span) (unsorted; empty slots 0) in out[q][g][0..k).
constexpr int MERGE_GROUP = 16;        // partitions per first-level CTA
constexpr int MERGE_ONE_CTA = 4096;    // candidates per query one merge CTA takes directly

__global__ void __launch_bounds__(256)
merge_groups_kernel(const uint64_t* __restrict__ cand, int64_t M, int64_t span, int k,
                    uint64_t* __restrict__ out) {
    __shared__ unsigned sm[300];
    __shared__ int cnt;
    const int g = blockIdx.x, q = blockIdx.y;
    const int64_t b0 = (int64_t)g * span;
    const int64_t m = min(span, M - b0);
    const uint64_t* src = cand + (int64_t)q * M + b0;
    uint64_t* dst = out + ((int64_t)q * gridDim.x + g) * k;
    const uint64_t T = block_select_threshold(src, m, k, sm);
    if (threadIdx.x == 0) cnt = 0;
    __syncthreads();
    for (int64_t i = threadIdx.x; i < m; i += 256) {
        const uint64_t c = src[i];
        if (c > T) dst[atomicAdd(&cnt, 1)] = c;
    }
    __syncthreads();
    // keys equal to T: one real key (T > 0) or any number of empty slots (T == 0)
    if (threadIdx.x == 0 && T != 0ull && cnt < k) dst[cnt++] = T;
    __syncthreads();
    for (int i = cnt + threadIdx.x; i < k; i += 256) dst[i] = 0ull;
}

// One CTA per query: best k of cand[q][0..M) -> sorted outputs.
template <typename IdxT>
__global__ void __launch_bounds__(256)
merge_candidates_kernel(const uint64_t* __restrict__ cand, int64_t M, int k, int64_t row_offset,
                        IdxT* __restrict__ out_idx, float* __restrict__ out_scores,
                        const int* __restrict__ counts) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    uint64_t* best = reinterpret_cast<uint64_t*>(smem_raw);
    __shared__ unsigned sm[300];
    __shared__ int cnt;
    const int q = blockIdx.x;
    const uint64_t* src = cand + (int64_t)q * M;
    if (counts && (int64_t)counts[q] < M) M = counts[q];   // per-query fill (pools)
    const int kp = next_pow2(k);
    const uint64_t T = block_select_threshold(src, M, k, sm);
    if (threadIdx.x == 0) cnt = 0;
    for (int i = threadIdx.x; i < kp; i += 256) best[i] = 0ull;
    __syncthreads();
    for (int64_t i = threadIdx.x; i < M; i += 256) {
        const uint64_t c = src[i];
        if (c > T) best[atomicAdd(&cnt, 1)] = c;
    }
    __syncthreads();
    // keys equal to T: one real key (T > 0) or any number of empty slots (T == 0)
    if (threadIdx.x == 0 && T != 0ull && cnt < k) best[cnt++] = T;
    __syncthreads();
    block_bitonic_sort_desc(best, kp);
    for (int i = threadIdx.x; i < k; i += 256) {
        const uint64_t c = best[i];
        const bool ok = c != 0ull;
        out_idx[(int64_t)q * k + i] = ok ? (IdxT)((int64_t)cand_row(c) + row_offset) : (IdxT)-1;
        if (out_scores) out_scores[(int64_t)q * k + i] = ok ? cand_score(c) : -INFINITY;
    }
}

// The merge kernel's dynamic shared memory grows with k; its limit is set
// once to the largest k any entry point accepts, never to one call's need,
// so that launches with different k (on any path) stay within it.
constexpr int MERGE_KMAX = 4096;
template <typename IdxT>
hmm_status_t prepare_merge_kernel() {
    HMM_CUDA_TRY(cudaFuncSetAttribute(merge_candidates_kernel<IdxT>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)(sizeof(uint64_t) * MERGE_KMAX)));
    return HMM_OK;
}

// bit i%64 of word i/64 = scores[i] >= thr.  One warp per 64-score word.
__global__ void threshold_bitmap_kernel(const float* __restrict__ scores, int64_t n, int nq,
                                        float thr, uint64_t* __restrict__ bitmap) {
    const int64_t words = (n + 63) / 64;
    const int lane = threadIdx.x & 31;
    const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (gw >= words * nq) return;
    const int64_t q = gw / words, w = gw % words;
    const float* s = scores + q * n;
    const int64_t i0 = w * 64 + lane, i1 = i0 + 32;
    const unsigned lo = __ballot_sync(0xffffffffu, i0 < n && s[i0] >= thr);
    const unsigned hi = __ballot_sync(0xffffffffu, i1 < n && s[i1] >= thr);
    if (lane == 0) bitmap[q * words + w] = ((uint64_t)hi << 32) | lo;
}

// Shard merge: one CTA per query sorts the n_shards*k gathered (score,
// global index) candidates by (score desc, index asc) in shared memory and
// keeps the first k.  Empty slots (index -1) sort last.
constexpr int MERGE_MAX = 8192;

__device__ __forceinline__ bool pair_better(uint32_t ka, int64_t ia, uint32_t kb, int64_t ib) {
    return ka > kb || (ka == kb && ia < ib);
}

__global__ void __launch_bounds__(256)
shard_merge_kernel(const float* __restrict__ cand_scores, const int64_t* __restrict__ cand_idx,
                   int n_shards, int nq, int k, float* __restrict__ out_scores,
                   int64_t* __restrict__ out_idx) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int M = n_shards * k;
    const int n = next_pow2(M);
    int64_t* sidx = reinterpret_cast<int64_t*>(smem_raw);
    uint32_t* skey = reinterpret_cast<uint32_t*>(sidx + n);
    const int q = blockIdx.x;
    for (int r = threadIdx.x; r < n; r += blockDim.x) {
        if (r < M) {
            const int s = r / k, i = r % k;
            const int64_t o = ((int64_t)s * nq + q) * k + i;
            const int64_t id = cand_idx[o];
            skey[r] = id < 0 ? 0u : f32_key(cand_scores[o]);
            sidx[r] = id < 0 ? INT64_MAX : id;
        } else {
            skey[r] = 0u;
            sidx[r] = INT64_MAX;
        }
    }
    for (int size = 2; size <= n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            __syncthreads();
            for (int i = threadIdx.x; i < n / 2; i += blockDim.x) {
                const int lo = 2 * i - (i & (stride - 1));
                const int hi = lo + stride;
                const bool desc = ((lo & size) == 0);
                const bool hi_better = pair_better(skey[hi], sidx[hi], skey[lo], sidx[lo]);
                if (hi_better == desc) {
                    const uint32_t tk = skey[lo]; skey[lo] = skey[hi]; skey[hi] = tk;
                    const int64_t ti = sidx[lo]; sidx[lo] = sidx[hi]; sidx[hi] = ti;
                }
            }
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
        const bool ok = sidx[i] != INT64_MAX;
        out_idx[(int64_t)q * k + i] = ok ? sidx[i] : -1;
        out_scores[(int64_t)q * k + i] = ok ? key_to_f32(skey[i]) : -INFINITY;
    }
}

hmm_status_t check_common(const void* mem, int64_t n, int64_t dim, const void* qry, int64_t nq,
                          int64_t k) {
    HMM_REQUIRE(n >= 0 && n < (int64_t(1) << 31), "n_rows must be in [0, 2^31), got %lld",
                (long long)n);
    HMM_REQUIRE(nq >= 0 && nq <= 65535 * QG, "n_queries out of range: %lld", (long long)nq);
    HMM_REQUIRE(dim >= 1 && dim <= 1024, "dim must be in [1, 1024], got %lld", (long long)dim);
    HMM_REQUIRE(k >= 1, "k must be >= 1, got %lld", (long long)k);
    HMM_REQUIRE(n == 0 || mem, "memory pointer is null");
    HMM_REQUIRE(nq == 0 || qry, "queries pointer is null");
    return HMM_OK;
}

// Score + top-k of a small memory (n <= SMALL_N rows), one CTA per query.
// Columns [c0, c0 + SMALL_KC) of every row are staged in shared memory by
// 16-byte cp.async copies, all of a chunk in flight at once; rows are padded to
// 16 bytes past the chunk, so the 16-byte reads of a quarter-warp (8 rows)
// fall in distinct banks.  Each thread then extends its rows' sums by those
// columns in index order, as the fused kernel does.  The scores' composites go
// to shared memory and one bitonic sort orders them.  Writes what
// fused_ip_topk_kernel + merge_candidates_kernel write, in one launch and
// without radix passes: the one-query-per-call shapes of the reference's API (a
// few hundred page summaries) are set by those two launches' selection passes,
// not by memory traffic.
constexpr int SMALL_N = 1024;
constexpr int SMALL_NT = 512;
constexpr int SMALL_R = SMALL_N / SMALL_NT;   // rows per thread
constexpr int SMALL_NQ = 64;
constexpr int SMALL_KC = 32;                   // columns per staged chunk

template <typename T>
__host__ __device__ constexpr int small_ld() { return SMALL_KC + 16 / (int)sizeof(T); }   // padded row stride (elements)

template <typename In>
size_t small_smem_bytes(int64_t n, int64_t dim) {
    return sizeof(float) * (size_t)((dim + 3) & ~int64_t(3)) +
           sizeof(typename In::T) * (size_t)(n * small_ld<typename In::T>());
}

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(smem_dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

template <typename In, typename IdxT>
__global__ void __launch_bounds__(SMALL_NT)
small_ip_topk_kernel(const typename In::T* __restrict__ mem, int n, int dim,
                     const typename In::T* __restrict__ qry, int k, int64_t row_offset, float thr,
                     uint32_t* __restrict__ bitmap32, float* __restrict__ full_scores,
                     IdxT* __restrict__ out_idx, float* __restrict__ out_scores, bool vec_ok) {
    using T = typename In::T;
    constexpr int LDT = small_ld<T>();
    __shared__ uint64_t keys[SMALL_N];
    extern __shared__ __align__(16) float sdyn[];
    float* sqv = sdyn;                                              // the query, dim values
    T* tile = reinterpret_cast<T*>(sdyn + ((dim + 3) & ~3));        // [n][LDT]
    const int q = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int j = tid; j < dim; j += SMALL_NT) sqv[j] = In::widen1(qry + (int64_t)q * dim + j);

    float acc[SMALL_R];
#pragma unroll
    for (int r = 0; r < SMALL_R; ++r) acc[r] = 0.0f;
    for (int c0 = 0; c0 < dim; c0 += SMALL_KC) {
        const int w = min(SMALL_KC, dim - c0);
        __syncthreads();   // the previous chunk is consumed (and the query written)
        if (vec_ok) {      // dim % VEC == 0 and 16-byte aligned rows, so w % VEC == 0
            const int per_row = w / In::VEC;
            for (int idx = tid; idx < n * per_row; idx += SMALL_NT) {
                const int r = idx / per_row, v = (idx - r * per_row) * In::VEC;
                cp_async16(tile + r * LDT + v, mem + (int64_t)r * dim + c0 + v);
            }
            cp_async_wait_all();
        } else {
            for (int idx = tid; idx < n * w; idx += SMALL_NT) {
                const int r = idx / w, j = idx - r * w;
                tile[r * LDT + j] = mem[(int64_t)r * dim + c0 + j];
            }
        }
        __syncthreads();
#pragma unroll
        for (int r = 0; r < SMALL_R; ++r) {
            const int i = tid + r * SMALL_NT;
            if (i >= n) continue;
            const T* t = tile + i * LDT;
            if (vec_ok) {
                for (int v = 0; v < w; v += In::VEC) {
                    const uint4 u = *reinterpret_cast<const uint4*>(t + v);
                    if constexpr (In::VEC == 4) {
                        acc[r] = In::mac(acc[r], __uint_as_float(u.x), sqv[c0 + v]);
                        acc[r] = In::mac(acc[r], __uint_as_float(u.y), sqv[c0 + v + 1]);
                        acc[r] = In::mac(acc[r], __uint_as_float(u.z), sqv[c0 + v + 2]);
                        acc[r] = In::mac(acc[r], __uint_as_float(u.w), sqv[c0 + v + 3]);
                    } else {
                        const uint32_t h[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            acc[r] = In::mac(acc[r], bf16_bits_to_f32((uint16_t)(h[e] & 0xffffu)),
                                             sqv[c0 + v + 2 * e]);
                            acc[r] = In::mac(acc[r], bf16_bits_to_f32((uint16_t)(h[e] >> 16)),
                                             sqv[c0 + v + 2 * e + 1]);
                        }
                    }
                }
            } else {
                for (int j = 0; j < w; ++j) acc[r] = In::mac(acc[r], In::widen1(t + j), sqv[c0 + j]);
            }
        }
    }

    const int n2 = next_pow2(n);
    const int64_t words32 = 2 * (((int64_t)n + 63) / 64);
    const int cover = max(n2, (int)(32 * words32));   // rows whose key slot or bitmap bit is written
#pragma unroll
    for (int r = 0; r < SMALL_R; ++r) {
        const int base = r * SMALL_NT;
        if (base >= cover) break;   // uniform: the ballot below sees whole warps
        const int i = base + tid;
        const float sc = acc[r];
        if (i < n && full_scores) full_scores[(int64_t)q * n + i] = sc;
        if (bitmap32) {
            const unsigned bits = __ballot_sync(0xffffffffu, i < n && sc >= thr);
            const int64_t w32 = (base >> 5) + warp;
            if (lane == 0 && w32 < words32) bitmap32[(int64_t)q * words32 + w32] = bits;
        }
        if (i < n2) keys[i] = i < n ? make_cand(f32_key(sc), (uint32_t)i) : 0ull;
    }
    block_bitonic_sort_desc(keys, n2);   // synchronises before and after
    for (int i = tid; i < k; i += SMALL_NT) {
        const uint64_t c = i < n2 ? keys[i] : 0ull;
        const bool ok = c != 0ull;
        out_idx[(int64_t)q * k + i] = ok ? (IdxT)((int64_t)cand_row(c) + row_offset) : (IdxT)-1;
        if (out_scores) out_scores[(int64_t)q * k + i] = ok ? cand_score(c) : -INFINITY;
    }
}

// Sets the small kernel's dynamic shared-memory limit (on the current device)
// to the largest any call can need: SMALL_N rows of the widest rows
// check_common accepts, so calls of different shapes never lower it.
template <typename In, typename IdxT>
hmm_status_t prepare_small_kernel() {
    const cudaError_t e = cudaFuncSetAttribute(
        small_ip_topk_kernel<In, IdxT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
        (int)small_smem_bytes<In>(SMALL_N, 1024));
    if (e != cudaSuccess)
        return set_error(HMM_ERR_CUDA, "cudaFuncSetAttribute(small_ip_topk_kernel): %s",
                         cudaGetErrorString(e));
    return HMM_OK;
}

// Few queries (at most NARROW_NQ) over many rows: one CTA per tile of
// NARROW_NT rows, thread = row.  Columns come into shared memory NARROW_KC at a
// time by 16-byte cp.async copies, double buffered so that the next chunk's
// copies are in flight while the current one is summed (rows padded by 16
// bytes: a quarter-warp's 16-byte reads hit distinct banks).  Each thread
// extends its row's sum for every query in column order, exactly as the fused
// kernel does; then the threshold-bitmap words come from warp ballots and one
// bitonic sort per query gives the tile's best k as candidates for the same
// merge the fused kernel feeds.  The fused kernel's 16-query register tiles
// would compute 16 query slots for one query.
constexpr int NARROW_NQ = 4;
constexpr int NARROW_NT = 256;
constexpr int NARROW_KC = 32;   // columns per staged chunk

template <typename T>
__host__ __device__ constexpr int narrow_ld() { return NARROW_KC + 16 / (int)sizeof(T); }

template <typename In>
size_t narrow_smem_bytes(int64_t dim) {
    return sizeof(float) * (size_t)NARROW_NQ * (size_t)((dim + 3) & ~int64_t(3)) +
           sizeof(uint64_t) * NARROW_NQ * NARROW_NT +
           2 * sizeof(typename In::T) * NARROW_NT * narrow_ld<typename In::T>();
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

template <typename In>
__global__ void __launch_bounds__(NARROW_NT)
narrow_ip_topk_kernel(const typename In::T* __restrict__ mem, int64_t n, int dim,
                      const typename In::T* __restrict__ qry, int nq, int k, float thr,
                      uint32_t* __restrict__ bitmap32, uint64_t* __restrict__ cand, bool vec_ok) {
    using T = typename In::T;
    constexpr int LDT = narrow_ld<T>();
    extern __shared__ __align__(16) unsigned char nsm[];
    const int dimp = (dim + 3) & ~3;
    float* sq = reinterpret_cast<float*>(nsm);                                   // [NQ][dimp]
    uint64_t* keys = reinterpret_cast<uint64_t*>(sq + NARROW_NQ * dimp);         // [NQ][NT]
    T* buf = reinterpret_cast<T*>(keys + NARROW_NQ * NARROW_NT);                // 2 x [NT][LDT]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int part = blockIdx.x;
    const int64_t row0 = (int64_t)part * NARROW_NT;
    const int64_t row = row0 + tid;
    const int rows = (int)min((int64_t)NARROW_NT, n - row0);
    for (int i = tid; i < NARROW_NQ * dimp; i += NARROW_NT) {
        const int q = i / dimp, j = i % dimp;
        sq[i] = (q < nq && j < dim) ? In::widen1(qry + (int64_t)q * dim + j) : 0.0f;
    }
    const int nch = (dim + NARROW_KC - 1) / NARROW_KC;
    // stage chunk c of the tile's rows into buffer b (rows past the end are
    // not copied; their sums are never used)
    auto stage = [&](int c, int b) {
        const int c0 = c * NARROW_KC, w = min(NARROW_KC, dim - c0);
        T* dst = buf + b * NARROW_NT * LDT;
        if (vec_ok) {   // dim % VEC == 0 and 16-byte aligned rows, so w % VEC == 0
            const int per_row = w / In::VEC;
            for (int idx = tid; idx < rows * per_row; idx += NARROW_NT) {
                const int r = idx / per_row, v = (idx - r * per_row) * In::VEC;
                cp_async16(dst + r * LDT + v, mem + (row0 + r) * dim + c0 + v);
            }
        } else {
            for (int idx = tid; idx < rows * w; idx += NARROW_NT) {
                const int r = idx / w, j = idx - r * w;
                dst[r * LDT + j] = mem[(row0 + r) * dim + c0 + j];
            }
        }
        cp_async_commit();
    };
    float acc[NARROW_NQ];
#pragma unroll
    for (int q = 0; q < NARROW_NQ; ++q) acc[q] = 0.0f;
    stage(0, 0);
    for (int c = 0; c < nch; ++c) {
        if (c + 1 < nch) {
            stage(c + 1, (c + 1) & 1);
            cp_async_wait_group<1>();   // chunk c has landed (c + 1 may be in flight)
        } else {
            cp_async_wait_group<0>();
        }
        __syncthreads();
        const int c0 = c * NARROW_KC, w = min(NARROW_KC, dim - c0);
        const T* t = buf + (c & 1) * NARROW_NT * LDT + tid * LDT;
        for (int j = 0; j < w; ++j) {
            const float a = In::widen1(t + j);
#pragma unroll
            for (int q = 0; q < NARROW_NQ; ++q)
                if (q < nq) acc[q] = In::mac(acc[q], a, sq[q * dimp + c0 + j]);
        }
        __syncthreads();   // buffer (c & 1) is restaged by the next iteration but one
    }
    const bool valid = row < n;
    const int64_t words32 = 2 * ((n + 63) / 64);
#pragma unroll
    for (int q = 0; q < NARROW_NQ; ++q) {
        if (q >= nq) break;
        if (bitmap32) {
            const unsigned bits = __ballot_sync(0xffffffffu, valid && acc[q] >= thr);
            const int64_t w32 = (row0 >> 5) + warp;
            if (lane == 0 && w32 < words32) bitmap32[(int64_t)q * words32 + w32] = bits;
        }
        keys[q * NARROW_NT + tid] = valid ? make_cand(f32_key(acc[q]), (uint32_t)row) : 0ull;
    }
    const int n_parts = gridDim.x;
    for (int q = 0; q < nq; ++q) {
        block_bitonic_sort_desc(keys + q * NARROW_NT, NARROW_NT);   // synchronises before and after
        uint64_t* dst = cand + ((int64_t)q * n_parts + part) * k;
        for (int i = tid; i < k; i += NARROW_NT) dst[i] = keys[q * NARROW_NT + i];
    }
}

// The narrow kernel applies to few queries over more rows than the small kernel
// takes, with k within one tile.
bool narrow_applies(int64_t n, int64_t nq, int64_t k) {
    return nq >= 1 && nq <= NARROW_NQ && n > SMALL_N && k <= NARROW_NT;
}

template <typename In, typename IdxT>
hmm_status_t run_fused(const typename In::T* mem, int64_t n, int64_t dim, const typename In::T* qry,
                       int64_t nq, int64_t k, int64_t row_offset, IdxT* out_idx,
                       float* out_scores, float thr, uint64_t* out_bitmap, float* full_scores,
                       void* ws, size_t ws_bytes, cudaStream_t st, size_t need) {
    HMM_REQUIRE(k <= KMAX_FUSED, "fused score+top-k supports k <= %d, got %lld", KMAX_FUSED,
                (long long)k);
    HMM_REQUIRE(out_idx, "out_idx is null");
    if (nq == 0) return HMM_OK;
    if (ws_bytes < need || !ws)
        return set_error(HMM_ERR_OOM, "workspace too small: %zu < %zu bytes", ws_bytes, need);
    const bool vec_ok = (dim % In::VEC) == 0 &&
                        (reinterpret_cast<uintptr_t>(mem) % 16) == 0;
    if (n >= 1 && n <= SMALL_N && nq <= SMALL_NQ) {
        const hmm_status_t ps = prepare_small_kernel<In, IdxT>();
        if (ps != HMM_OK) return ps;
        small_ip_topk_kernel<In, IdxT><<<(unsigned)nq, SMALL_NT, small_smem_bytes<In>(n, dim), st>>>(
            mem, (int)n, (int)dim, qry, (int)k, row_offset, thr,
            reinterpret_cast<uint32_t*>(out_bitmap), full_scores, out_idx, out_scores, vec_ok);
        return check_launch("small_ip_topk_kernel");
    }
    Plan p = plan_fused(n, nq);
    uint64_t* cand = static_cast<uint64_t*>(ws);
    if (!full_scores && narrow_applies(n, nq, k)) {
        p.n_parts = (int)((n + NARROW_NT - 1) / NARROW_NT);
        const size_t smem = narrow_smem_bytes<In>(dim);
        auto kern = narrow_ip_topk_kernel<In>;
        HMM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)smem));
        kern<<<(unsigned)p.n_parts, NARROW_NT, smem, st>>>(
            mem, n, (int)dim, qry, (int)nq, (int)k, thr, reinterpret_cast<uint32_t*>(out_bitmap),
            cand, vec_ok);
        hmm_status_t s = check_launch("narrow_ip_topk_kernel");
        if (s != HMM_OK) return s;
    } else if (n > 0) {
        const size_t smem = fused_smem_bytes((int)dim);
        auto kern = fused_ip_topk_kernel<In>;
        HMM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)smem));
        dim3 grid(p.n_parts, p.n_qgroups);
        kern<<<grid, NT, smem, st>>>(mem, n, (int)dim, qry, (int)nq, (int)k, p.rows_per_part, thr,
                                     reinterpret_cast<uint32_t*>(out_bitmap), full_scores, cand,
                                     vec_ok);
        hmm_status_t s = check_launch("fused_ip_topk_kernel");
        if (s != HMM_OK) return s;
    } else {
        HMM_CUDA_TRY(cudaMemsetAsync(cand, 0, sizeof(uint64_t) * nq * p.n_parts * k, st));
    }
    const size_t msmem = sizeof(uint64_t) * next_pow2((int)k);
    hmm_status_t ms = prepare_merge_kernel<IdxT>();
    if (ms != HMM_OK) return ms;
    int64_t M = (int64_t)p.n_parts * k;
    const uint64_t* src = cand;
    if (M > MERGE_ONE_CTA) {   // a first level of CTAs, so that no CTA merges them all
        const int groups = (p.n_parts + MERGE_GROUP - 1) / MERGE_GROUP;
        uint64_t* lvl = cand + (int64_t)nq * M;
        merge_groups_kernel<<<dim3(groups, (unsigned)nq), 256, 0, st>>>(cand, M,
                                                                        (int64_t)MERGE_GROUP * k,
                                                                        (int)k, lvl);
        ms = check_launch("merge_groups_kernel");
        if (ms != HMM_OK) return ms;
        src = lvl;
        M = (int64_t)groups * k;
    }
    merge_candidates_kernel<IdxT><<<(unsigned)nq, 256, msmem, st>>>(
        src, M, (int)k, row_offset, out_idx, out_scores, nullptr);
    return check_launch("merge_candidates_kernel");
}

size_t fused_ws_bytes(int64_t n, int64_t nq, int64_t k) {
    Plan p = plan_fused(n, nq);
    if (narrow_applies(n, nq, k))   // the narrow kernel's tiles are the parts
        p.n_parts = (int)std::max<int64_t>(p.n_parts, (n + NARROW_NT - 1) / NARROW_NT);
    size_t b = sizeof(uint64_t) * (size_t)nq * (size_t)p.n_parts * (size_t)k;
    if ((int64_t)p.n_parts * k > MERGE_ONE_CTA)   // the first merge level's output
        b += sizeof(uint64_t) * (size_t)nq * (size_t)((p.n_parts + MERGE_GROUP - 1) / MERGE_GROUP) *
             (size_t)k;
    return b + 256;
}

}  // namespace
// ---- entry points shared with the tensor-core path (flat_tc.cu)

hmm_status_t flat_bf16_exact(const uint16_t* mem, int64_t n, int64_t dim, const uint16_t* qry,
                             int64_t nq, int64_t k, int64_t row_offset, int64_t* out_idx,
                             float* out_scores, void* ws, size_t ws_bytes, cudaStream_t st) {
    return run_fused<BF16In, int64_t>(mem, n, dim, qry, nq, k, row_offset, out_idx, out_scores,
                                      0.0f, nullptr, nullptr, ws, ws_bytes, st,
                                      fused_ws_bytes(n, nq, k));
}

size_t flat_bf16_exact_ws_bytes(int64_t n, int64_t nq, int64_t k) { return fused_ws_bytes(n, nq, k); }

hmm_status_t launch_pool_merge(const uint64_t* pool, int64_t cap, const int* counts, int nq,
                               int k, int64_t row_offset, int64_t* out_idx, float* out_scores,
                               cudaStream_t st) {
    hmm_status_t s = prepare_merge_kernel<int64_t>();
    if (s != HMM_OK) return s;
    const size_t msmem = sizeof(uint64_t) * next_pow2(k);
    merge_candidates_kernel<int64_t><<<(unsigned)nq, 256, msmem, st>>>(
        pool, cap, k, row_offset, out_idx, out_scores, counts);
    return check_launch("merge_candidates_kernel(pool)");
}

// Same merge with int32 indices (the indexer entry points).
hmm_status_t launch_cand_merge_i32(const uint64_t* cand, int64_t cap, const int* counts, int nq,
                                   int k, int32_t* out_idx, float* out_scores, cudaStream_t st) {
    hmm_status_t s = prepare_merge_kernel<int32_t>();
    if (s != HMM_OK) return s;
    const size_t msmem = sizeof(uint64_t) * next_pow2(k);
    merge_candidates_kernel<int32_t><<<(unsigned)nq, 256, msmem, st>>>(
        cand, cap, k, 0, out_idx, out_scores, counts);
    return check_launch("merge_candidates_kernel(i32)");
}

bool tc_path_applies(int64_t n, int64_t dim, int64_t nq, int64_t k, const void* mem,
                     const void* qry);
size_t tc_ws_bytes(int64_t n, int64_t nq, int64_t k);
hmm_status_t flat_bf16_tc(const uint16_t* mem, int64_t n, const uint16_t* qry, int64_t nq,
                          int64_t k, int64_t row_offset, int64_t* out_idx, float* out_scores,
                          void* ws, size_t ws_bytes, cudaStream_t st, int32_t* dev_status);

// Scratch of hmm_ip_topk_f32_noalloc: a fixed device array, so that the
// entry point never allocates.  Host code may not use `g_noalloc_scratch` as
// a device address; it looks the address up per device with
// cudaGetSymbolAddress (see noalloc_scratch_ptr).
static __device__ __align__(256) unsigned char g_noalloc_scratch[HMM_NOALLOC_SCRATCH_BYTES];

namespace {

// The calling thread's current CUDA context (driver API, reached through the
// runtime's entry-point query so that the library needs no -lcuda).
void* current_context() {
    using GetCurrent = int (*)(void**);
    static GetCurrent fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<GetCurrent>(p);
    });
    void* ctx = nullptr;
    if (fn && fn(&ctx) != 0) ctx = nullptr;
    return ctx;
}

// Device address of g_noalloc_scratch on the current device, looked up on
// the first call per device (with that device current) and cached together
// with the context it was looked up in.  A device reset or a re-created
// primary context reloads the module, possibly at another address, so a
// call made in a context other than the cached one looks the address up
// again.
hmm_status_t noalloc_scratch_ptr(void** out) {
    static std::mutex mu;
    static void* cache[128] = {nullptr};
    static void* cache_ctx[128] = {nullptr};
    int dev = 0;
    HMM_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 128) return set_error(HMM_ERR_UNSUPPORTED, "device id %d", dev);
    void* ctx = current_context();
    std::lock_guard<std::mutex> lock(mu);
    if (!cache[dev] || ctx == nullptr || ctx != cache_ctx[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p)
            return set_error(HMM_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s",
                             cudaGetErrorString(e));
        cache[dev] = p;
        cache_ctx[dev] = current_context();   // the lookup made the primary context current
    }
    *out = cache[dev];
    return HMM_OK;
}

}  // namespace
}  // namespace hmm

using namespace hmm;

extern "C" {

hmm_status_t hmm_ip_score_f32(const float* mem, int64_t n_rows, int64_t dim,
                              const float* queries, int64_t n_queries, float* scores,
                              void* stream) {
    hmm_status_t s = check_common(mem, n_rows, dim, queries, n_queries, 1);
    if (s != HMM_OK) return s;
    HMM_REQUIRE(n_rows == 0 || n_queries == 0 || scores, "scores pointer is null");
    if (n_rows == 0 || n_queries == 0) return HMM_OK;
    // The fused kernel with no candidate output writes every score.
    const Plan p = plan_fused(n_rows, n_queries);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t smem = fused_smem_bytes((int)dim);
    auto kern = fused_ip_topk_kernel<F32In>;
    HMM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const bool vec_ok = (dim % 4) == 0 && (reinterpret_cast<uintptr_t>(mem) % 16) == 0;
    kern<<<dim3(p.n_parts, p.n_qgroups), NT, smem, st>>>(mem, n_rows, (int)dim, queries,
                                                         (int)n_queries, 1, p.rows_per_part, 0.0f,
                                                         nullptr, scores, nullptr, vec_ok);
    return check_launch("fused_ip_topk_kernel(scores)");
}

size_t hmm_topk_f32_workspace_size(int64_t n, int64_t n_queries, int64_t k) {
    if (n < 0 || n_queries < 0 || k < 1) return 0;
    const int64_t parts = std::max<int64_t>(1, (n + TOPK_P - 1) / TOPK_P);
    return sizeof(uint64_t) * (size_t)(parts * n_queries * k) + 256;
}

hmm_status_t hmm_topk_f32(const float* scores, int64_t n, int64_t n_queries, int64_t k,
                          int32_t* out_idx, float* out_scores, void* workspace,
                          size_t workspace_bytes, void* stream) {
    HMM_REQUIRE(n >= 0 && n < (int64_t(1) << 31), "n must be in [0, 2^31)");
    HMM_REQUIRE(n_queries >= 0 && n_queries <= 65535, "n_queries out of range");
    HMM_REQUIRE(k >= 1 && k <= TOPK_KMAX, "k must be in [1, %d], got %lld", TOPK_KMAX,
                (long long)k);
    HMM_REQUIRE(n == 0 || n_queries == 0 || scores, "scores pointer is null");
    HMM_REQUIRE(n_queries == 0 || out_idx, "out_idx is null");
    if (n_queries == 0) return HMM_OK;
    const size_t need = hmm_topk_f32_workspace_size(n, n_queries, k);
    if (!workspace || workspace_bytes < need)
        return set_error(HMM_ERR_OOM, "workspace too small: %zu < %zu bytes", workspace_bytes, need);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint64_t* cand = static_cast<uint64_t*>(workspace);
    const int64_t parts = std::max<int64_t>(1, (n + TOPK_P - 1) / TOPK_P);
    HMM_REQUIRE(parts <= 2147483647, "too many partitions");
    if (n > 0) {
        scores_topk_partition_kernel<<<dim3((unsigned)parts, (unsigned)n_queries), 256, 0, st>>>(
            scores, n, (int)k, cand);
        hmm_status_t s = check_launch("scores_topk_partition_kernel");
        if (s != HMM_OK) return s;
    } else {
        HMM_CUDA_TRY(cudaMemsetAsync(cand, 0, sizeof(uint64_t) * n_queries * k, st));
    }
    const size_t msmem = sizeof(uint64_t) * next_pow2((int)k);
    auto mk = merge_candidates_kernel<int32_t>;
    hmm_status_t ms = prepare_merge_kernel<int32_t>();
    if (ms != HMM_OK) return ms;
    mk<<<(unsigned)n_queries, 256, msmem, st>>>(cand, parts * k, (int)k, 0, out_idx, out_scores,
                                                nullptr);
    return check_launch("merge_candidates_kernel");
}

hmm_status_t hmm_threshold_bitmap_f32(const float* scores, int64_t n, int64_t n_queries,
                                      float threshold, uint64_t* bitmap, void* stream) {
    HMM_REQUIRE(n >= 0 && n_queries >= 0, "negative size");
    HMM_REQUIRE(n == 0 || n_queries == 0 || (scores && bitmap), "null pointer");
    const int64_t words = (n + 63) / 64;
    if (words == 0 || n_queries == 0) return HMM_OK;
    const int64_t threads = words * n_queries * 32;
    const int64_t blocks = (threads + 255) / 256;
    HMM_REQUIRE(blocks <= 2147483647, "problem too large");
    threshold_bitmap_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        scores, n, (int)n_queries, threshold, bitmap);
    return check_launch("threshold_bitmap_kernel");
}

size_t hmm_ip_topk_f32_workspace_size(int64_t n_rows, int64_t dim, int64_t n_queries, int64_t k) {
    (void)dim;
    if (n_rows < 0 || n_queries < 0 || k < 1) return 0;
    return fused_ws_bytes(n_rows, n_queries, k);
}

hmm_status_t hmm_ip_topk_f32(const float* mem, int64_t n_rows, int64_t dim,
                             const float* queries, int64_t n_queries, int64_t k,
                             int32_t* out_idx, float* out_scores, float threshold,
                             uint64_t* out_bitmap, void* workspace, size_t workspace_bytes,
                             void* stream) {
    hmm_status_t s = check_common(mem, n_rows, dim, queries, n_queries, k);
    if (s != HMM_OK) return s;
    return run_fused<F32In, int32_t>(mem, n_rows, dim, queries, n_queries, k, 0, out_idx,
                                     out_scores, threshold, out_bitmap, nullptr, workspace,
                                     workspace_bytes, static_cast<cudaStream_t>(stream),
                                     fused_ws_bytes(n_rows, n_queries, k));
}

size_t hmm_ip_topk_bf16_workspace_size(int64_t n_rows, int64_t dim, int64_t n_queries,
                                       int64_t k) {
    if (n_rows < 0 || n_queries < 0 || k < 1) return 0;
    const size_t v0 = fused_ws_bytes(n_rows, n_queries, k);
    // the tensor-core path applies for aligned pointers; size for it whenever the shape fits
    if (dim == 128 && k <= 128 && n_rows > 8192 && n_queries >= 1)
        return std::max(v0, tc_ws_bytes(n_rows, n_queries, k));
    return v0;
}

hmm_status_t hmm_ip_topk_bf16(const uint16_t* mem, int64_t n_rows, int64_t dim,
                              const uint16_t* queries, int64_t n_queries, int64_t k,
                              int64_t row_offset, int64_t* out_idx, float* out_scores,
                              void* workspace, size_t workspace_bytes, void* stream) {
    hmm_status_t s = check_common(mem, n_rows, dim, queries, n_queries, k);
    if (s != HMM_OK) return s;
    HMM_REQUIRE(row_offset >= 0, "row_offset must be >= 0");
    HMM_REQUIRE(n_queries == 0 || out_scores, "out_scores is null");
    HMM_REQUIRE(n_queries == 0 || out_idx, "out_idx is null");
    if (n_queries > 0 && tc_path_applies(n_rows, dim, n_queries, k, mem, queries)) {
        if (!workspace) return set_error(HMM_ERR_OOM, "workspace is null");
        return flat_bf16_tc(mem, n_rows, queries, n_queries, k, row_offset, out_idx, out_scores,
                            workspace, workspace_bytes, static_cast<cudaStream_t>(stream),
                            nullptr);
    }
    return run_fused<BF16In, int64_t>(mem, n_rows, dim, queries, n_queries, k, row_offset,
                                      out_idx, out_scores, 0.0f, nullptr, nullptr, workspace,
                                      workspace_bytes, static_cast<cudaStream_t>(stream),
                                      fused_ws_bytes(n_rows, n_queries, k));
}

hmm_status_t hmm_ip_topk_bf16_async(const uint16_t* mem, int64_t n_rows, int64_t dim,
                                    const uint16_t* queries, int64_t n_queries, int64_t k,
                                    int64_t row_offset, int64_t* out_idx, float* out_scores,
                                    int32_t* device_status, void* workspace,
                                    size_t workspace_bytes, void* stream) {
    HMM_REQUIRE(device_status, "device_status is null");
    hmm_status_t s = check_common(mem, n_rows, dim, queries, n_queries, k);
    if (s != HMM_OK) return s;
    HMM_REQUIRE(row_offset >= 0, "row_offset must be >= 0");
    HMM_REQUIRE(n_queries == 0 || out_scores, "out_scores is null");
    HMM_REQUIRE(n_queries == 0 || out_idx, "out_idx is null");
    if (n_queries > 0 && tc_path_applies(n_rows, dim, n_queries, k, mem, queries)) {
        if (!workspace) return set_error(HMM_ERR_OOM, "workspace is null");
        return flat_bf16_tc(mem, n_rows, queries, n_queries, k, row_offset, out_idx, out_scores,
                            workspace, workspace_bytes, static_cast<cudaStream_t>(stream),
                            device_status);
    }
    return run_fused<BF16In, int64_t>(mem, n_rows, dim, queries, n_queries, k, row_offset,
                                      out_idx, out_scores, 0.0f, nullptr, nullptr, workspace,
                                      workspace_bytes, static_cast<cudaStream_t>(stream),
                                      fused_ws_bytes(n_rows, n_queries, k));
}

hmm_status_t hmm_ip_topk_f32_noalloc(const float* mem, int64_t n_rows, int64_t dim,
                                     const float* queries, int64_t n_queries, int64_t k,
                                     int32_t* out_idx, float* out_scores, float threshold,
                                     uint64_t* out_bitmap, void* stream) {
    hmm_status_t s = check_common(mem, n_rows, dim, queries, n_queries, k);
    if (s != HMM_OK) return s;
    const size_t need = fused_ws_bytes(n_rows, n_queries, k);
    if (need > HMM_NOALLOC_SCRATCH_BYTES)
        return set_error(HMM_ERR_UNSUPPORTED,
                         "hmm_ip_topk_f32_noalloc: this problem needs %zu bytes of scratch, above "
                         "the fixed %u-byte limit; use hmm_ip_topk_f32 with a workspace",
                         need, (unsigned)HMM_NOALLOC_SCRATCH_BYTES);
    void* scratch = nullptr;
    s = noalloc_scratch_ptr(&scratch);
    if (s != HMM_OK) return s;
    return run_fused<F32In, int32_t>(mem, n_rows, dim, queries, n_queries, k, 0, out_idx,
                                     out_scores, threshold, out_bitmap, nullptr, scratch,
                                     HMM_NOALLOC_SCRATCH_BYTES, static_cast<cudaStream_t>(stream),
                                     need);
}

size_t hmm_shard_merge_topk_workspace_size(int64_t n_shards, int64_t n_queries, int64_t k) {
    (void)n_shards; (void)n_queries; (void)k;
    return 0;
}

hmm_status_t hmm_shard_merge_topk(const float* cand_scores, const int64_t* cand_idx,
                                  int64_t n_shards, int64_t n_queries, int64_t k,
                                  float* out_scores, int64_t* out_idx, void* workspace,
                                  size_t workspace_bytes, void* stream) {
    (void)workspace; (void)workspace_bytes;
    HMM_REQUIRE(n_shards >= 1 && k >= 1 && n_queries >= 0, "bad sizes");
    HMM_REQUIRE(n_shards * k <= MERGE_MAX, "n_shards * k must be <= %d", MERGE_MAX);
    HMM_REQUIRE(n_queries <= 2147483647, "n_queries out of range");
    if (n_queries == 0) return HMM_OK;
    HMM_REQUIRE(cand_scores && cand_idx && out_scores && out_idx, "null pointer");
    const int n = next_pow2((int)(n_shards * k));
    const size_t smem = (sizeof(int64_t) + sizeof(uint32_t)) * (size_t)n;
    HMM_CUDA_TRY(cudaFuncSetAttribute(shard_merge_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    shard_merge_kernel<<<(unsigned)n_queries, 256, smem, static_cast<cudaStream_t>(stream)>>>(
        cand_scores, cand_idx, (int)n_shards, (int)n_queries, (int)k, out_scores, out_idx);
    return check_launch("shard_merge_kernel");
}

}  // extern "C"
