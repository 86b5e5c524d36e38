// paged_kv.cu — paged-KV block summaries, block -> page expansion, block-sparse
// decode attention over a paged bf16 KV cache, and the fused decode step
// (block selection + attention) of the paged-KV retrieval path.
//
// Reference: PagedKVIndexBuilder (steps/example_kernel/paged_kv_index_builder.cpp:18-85),
// BlockSparseAttention (steps/example_kernel/block_sparse_attention.cpp:21-126),
// InnerProductCompute + TopKRetrieval over the block summaries
// (inner_product_compute.cpp:11-31, topk_retrieval.cpp:13-31).
//
// Layout: physical page `phys` of a cache holds `page_tokens` consecutive tokens
// of one sequence as [page_tokens][D] bf16; page_table[s * pages_per_seq + p]
// names the physical page of logical page p of sequence s.  Summaries are fp32
// [n_seq][n_blocks][D].
//
// Every kernel here is HBM-bound CUDA-core work: one query per sequence in
// decode gives matrix-vector shapes (M = 1) that tensor cores cannot use.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <type_traits>

#include "heteromm_cuda.h"
#include "hmm_common.cuh"

namespace hmm {
namespace {

constexpr int PK_MAX_D = 512;           // 4 column groups of 4 per lane
constexpr int PK_GROUPS = PK_MAX_D / 128;
constexpr int BSA_THREADS = 256;
constexpr int BSA_WARPS = BSA_THREADS / 32;
constexpr int BSA_MAX_SEL = 4096;       // selected blocks per sequence
constexpr int BSA_MAX_SPLIT_TOKENS = 8192;
// Smallest share of the token list one block takes when the sequences are too
// few to fill the GPU: one pass of its warps (4 tokens each) in the token-
// granular kernel, one page per warp in the page-granular one.  A single
// decode sequence then spreads over ~n_list / 32 blocks instead of a handful.
constexpr int BSA_MIN_SPLIT_TOKENS = BSA_WARPS * 4;
constexpr int BSA_MIN_SPLIT_PAGES = BSA_WARPS;
constexpr int BSA_PAGES_PER_SPLIT = 8 * BSA_WARPS;   // pages a split takes when sequences are many
constexpr int SEL_MAX_BLOCKS = 8192;    // summaries per sequence for the fused selection
constexpr int SEL_THREADS_MAX = 1024;   // block selection: threads per sequence

struct PagedCache {
    const uint16_t* pages;   // [n_pages][page_tokens][D]
    const int32_t* table;    // [n_seq][pages_per_seq]
    int64_t n_pages;
    int pages_per_seq;
    int seq_len;
    int page_tokens;
    int D;
    bool contiguous;         // [n_seq][seq_len][D] without a page table
};

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// First element of logical token t of sequence s in `base` (a K or V page
// array laid out like c.pages), or nullptr after flagging status bit 0 when
// the page-table entry is outside [0, n_pages).
template <typename T = uint16_t>
__device__ __forceinline__ const T* token_row(const PagedCache& c, const T* base, int s, int t,
                                              int* status) {
    if (c.contiguous) return base + ((int64_t)s * c.seq_len + t) * c.D;
    const int p = t / c.page_tokens;
    const int32_t phys = __ldg(c.table + (int64_t)s * c.pages_per_seq + p);
    if (phys < 0 || (int64_t)phys >= c.n_pages) {
        atomicOr(status, 1);
        return nullptr;
    }
    return base + ((int64_t)phys * c.page_tokens + (t - p * c.page_tokens)) * c.D;
}

// ------------------------------------------------------------------ a-5
// Reference form: contiguous fp32 keys [n_seq][L][D].  One block per
// (page, sequence).  pooled[d] = (sum of keys[t][d], t ascending) / count,
// then out[o] = sum_d W[o][d] * pooled[d], d ascending, no FMA
// (paged_kv_index_builder.cpp:53-79).
__global__ void kv_summary_f32_kernel(const float* __restrict__ keys, int L, int D,
                                      const float* __restrict__ W, int out_dim, int page,
                                      int pages, float* __restrict__ out) {
    extern __shared__ float pooled[];
    const int p = blockIdx.x, s = blockIdx.y;
    const int t0 = p * page;
    const int t1 = min(t0 + page, L);
    const float* kb = keys + (int64_t)s * L * D;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float acc = 0.0f;
        for (int t = t0; t < t1; ++t) acc = __fadd_rn(acc, kb[(int64_t)t * D + d]);
        pooled[d] = acc / (float)(t1 - t0);
    }
    __syncthreads();
    float* o = out + ((int64_t)s * pages + p) * out_dim;
    if (W) {
        for (int i = threadIdx.x; i < out_dim; i += blockDim.x) {
            const float* w = W + (int64_t)i * D;
            float acc = 0.0f;
            for (int d = 0; d < D; ++d) acc = __fadd_rn(acc, __fmul_rn(__ldg(w + d), pooled[d]));
            o[i] = acc;
        }
    } else {
        for (int d = threadIdx.x; d < D; d += blockDim.x) o[d] = pooled[d];
    }
}

// Paged bf16 form: one warp per (sequence, block) summary; lane owns column
// groups 4*(lane + 32g), g < NG.  Tokens are summed in ascending order, per
// column, as the reference does; the division by the token count is IEEE.
// U tokens (up to one 16-token page at D <= 128) are loaded before they are
// summed, to keep a page's worth of loads in flight per warp.
template <int NG>
__global__ void __launch_bounds__(256) paged_summary_kernel(PagedCache c, int block_tokens,
                                                            int n_blocks, int64_t n_units,
                                                            float* __restrict__ out,
                                                            int* status) {
    constexpr int U = 16 / NG;
    const int64_t unit = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (unit >= n_units) return;
    const int s = (int)(unit / n_blocks), b = (int)(unit % n_blocks);
    const int t0 = b * block_tokens;
    const int t1 = min(t0 + block_tokens, c.seq_len);
    const int ng = c.D >> 2;
    float acc[NG][4];
#pragma unroll
    for (int g = 0; g < NG; ++g)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[g][i] = 0.0f;
    bool bad = false;
    for (int t = t0, n = 0; t < t1; t += n) {
        // one page-table lookup per page, then its tokens in order
        const uint16_t* row = token_row(c, c.pages, s, t, status);
        if (!row) { bad = true; break; }
        n = min(c.page_tokens - (t % c.page_tokens), t1 - t);
        for (int j0 = 0; j0 < n; j0 += U) {
            uint2 v[U][NG];
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
                for (int g = 0; g < NG; ++g) {
                    const int gi = lane + 32 * g;
                    v[u][g] = (j0 + u < n && gi < ng)
                                  ? __ldg(reinterpret_cast<const uint2*>(row + (int64_t)(j0 + u) * c.D) + gi)
                                  : make_uint2(0u, 0u);
                }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                if (j0 + u >= n) break;
#pragma unroll
                for (int g = 0; g < NG; ++g) {
                    acc[g][0] = __fadd_rn(acc[g][0], bf16_lo(v[u][g].x));
                    acc[g][1] = __fadd_rn(acc[g][1], bf16_hi(v[u][g].x));
                    acc[g][2] = __fadd_rn(acc[g][2], bf16_lo(v[u][g].y));
                    acc[g][3] = __fadd_rn(acc[g][3], bf16_hi(v[u][g].y));
                }
            }
        }
    }
    const float cnt = (float)(t1 - t0);
    float* o = out + unit * c.D;
#pragma unroll
    for (int g = 0; g < NG; ++g) {
        const int gi = lane + 32 * g;
        if (gi < ng) {
            float4 r;
            r.x = bad ? 0.0f : acc[g][0] / cnt;
            r.y = bad ? 0.0f : acc[g][1] / cnt;
            r.z = bad ? 0.0f : acc[g][2] / cnt;
            r.w = bad ? 0.0f : acc[g][3] / cnt;
            reinterpret_cast<float4*>(o)[gi] = r;
        }
    }
}

// Min/max page summaries (the reference's MinMaxIndexMemory, types/memory.h:
// 127-230: per block a min vector then a max vector): per (sequence, block) and
// column, the smallest and largest key of the block's tokens (fminf / fmaxf:
// NaN ignored unless all are).  Same walk as paged_summary_kernel; out is
// [unit][2][D].
template <int NG>
__global__ void __launch_bounds__(256) paged_minmax_kernel(PagedCache c, int block_tokens,
                                                           int n_blocks, int64_t n_units,
                                                           float* __restrict__ out,
                                                           int* status) {
    constexpr int U = 16 / NG;
    const int64_t unit = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (unit >= n_units) return;
    const int s = (int)(unit / n_blocks), b = (int)(unit % n_blocks);
    const int t0 = b * block_tokens;
    const int t1 = min(t0 + block_tokens, c.seq_len);
    const int ng = c.D >> 2;
    float mn[NG][4], mx[NG][4];
#pragma unroll
    for (int g = 0; g < NG; ++g)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            mn[g][i] = __int_as_float(0x7fc00000);   // NaN: replaced by the first key
            mx[g][i] = __int_as_float(0x7fc00000);
        }
    bool bad = false;
    for (int t = t0, n = 0; t < t1; t += n) {
        const uint16_t* row = token_row(c, c.pages, s, t, status);
        if (!row) { bad = true; break; }
        n = min(c.page_tokens - (t % c.page_tokens), t1 - t);
        for (int j0 = 0; j0 < n; j0 += U) {
            uint2 v[U][NG];
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
                for (int g = 0; g < NG; ++g) {
                    const int gi = lane + 32 * g;
                    v[u][g] = (j0 + u < n && gi < ng)
                                  ? __ldg(reinterpret_cast<const uint2*>(row + (int64_t)(j0 + u) * c.D) + gi)
                                  : make_uint2(0u, 0u);
                }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                if (j0 + u >= n) break;
#pragma unroll
                for (int g = 0; g < NG; ++g) {
                    const float x[4] = {bf16_lo(v[u][g].x), bf16_hi(v[u][g].x),
                                        bf16_lo(v[u][g].y), bf16_hi(v[u][g].y)};
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        mn[g][i] = fminf(mn[g][i], x[i]);
                        mx[g][i] = fmaxf(mx[g][i], x[i]);
                    }
                }
            }
        }
    }
    float* omin = out + unit * 2 * c.D;
    float* omax = omin + c.D;
#pragma unroll
    for (int g = 0; g < NG; ++g) {
        const int gi = lane + 32 * g;
        if (gi < ng) {
            reinterpret_cast<float4*>(omin)[gi] =
                bad ? make_float4(0.f, 0.f, 0.f, 0.f) : make_float4(mn[g][0], mn[g][1], mn[g][2], mn[g][3]);
            reinterpret_cast<float4*>(omax)[gi] =
                bad ? make_float4(0.f, 0.f, 0.f, 0.f) : make_float4(mx[g][0], mx[g][1], mx[g][2], mx[g][3]);
        }
    }
}

// ------------------------------------------------------------------ a-7
// Logical pages [b*ppb, (b+1)*ppb) of each selected block b, in selection
// order, clipped to [0, pages_per_seq), through the page table; one block per
// sequence, chunks of 256 selections with a block scan for the offsets.
__global__ void __launch_bounds__(256) block_pages_kernel(const int32_t* __restrict__ table,
                                                          int pages_per_seq,
                                                          const int32_t* __restrict__ blocks,
                                                          int n_sel, int ppb,
                                                          int32_t* __restrict__ out_pages,
                                                          int32_t* __restrict__ out_counts) {
    __shared__ unsigned wt[8];
    const int s = blockIdx.x;
    const int32_t* tb = table + (int64_t)s * pages_per_seq;
    int32_t* op = out_pages + (int64_t)s * n_sel * ppb;
    unsigned base = 0;
    for (int c0 = 0; c0 < n_sel; c0 += 256) {
        const int i = c0 + threadIdx.x;
        int64_t p0 = 0, lo = 0, hi = 0;
        if (i < n_sel) {
            p0 = (int64_t)blocks[(int64_t)s * n_sel + i] * ppb;
            lo = p0 < 0 ? 0 : p0;
            hi = p0 + ppb < pages_per_seq ? p0 + ppb : pages_per_seq;
            if (hi < lo) hi = lo;
        }
        const unsigned cnt = (unsigned)(hi - lo);
        const unsigned incl = block_scan_incl_256(cnt, wt);
        const unsigned total = wt[7];   // the scan leaves the block total here
        unsigned pos = base + incl - cnt;
        for (int64_t p = lo; p < hi; ++p) op[pos++] = tb[p];
        base += total;
        __syncthreads();
    }
    for (int64_t j = base + threadIdx.x; j < (int64_t)n_sel * ppb; j += blockDim.x) op[j] = -1;
    if (out_counts && threadIdx.x == 0) out_counts[s] = (int32_t)base;
}

// ------------------------------------------------------------------ a-6
struct BsaArgs {
    PagedCache k;            // K cache (pages, table, geometry)
    const uint16_t* v;       // V pages, same layout and table as K
    const uint16_t* q;       // [n_seq][D] bf16
    const float* kf;         // fp32 element form (contiguous caches): K, V, q
    const float* vf;
    const float* qf32;
    const int32_t* blocks;   // [n_seq][blocks_stride], first n_sel used
    int blocks_stride;
    int n_sel;
    int block_tokens;
    float scale;             // 1.0f / sqrtf((float)D), computed on the host
    int splits;
    int split_tokens;        // token-list positions per split
    float* part;             // [n_seq][splits][2 + D]: max, sum, unnormalised out
    int* status;
};

__device__ __forceinline__ float block_reduce_max(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float r = red[0];
    for (int w = 1; w < BSA_WARPS; ++w) r = fmaxf(r, red[w]);
    __syncthreads();
    return r;
}

__device__ __forceinline__ float block_reduce_sum(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float r = 0.0f;
    for (int w = 0; w < BSA_WARPS; ++w) r += red[w];
    __syncthreads();
    return r;
}

// Token at position j of the selected token list: the list concatenates
// [b*BT, min(b*BT + BT, L)) over the selected blocks in order
// (block_sparse_attention.cpp:53-63); pre[] holds the running list lengths.
__device__ __forceinline__ int list_token(const int* pre, const int32_t* bl, int n_sel, int BT,
                                          int j) {
    int lo = 0, hi = n_sel - 1;   // last i with pre[i] <= j
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (pre[mid] <= j) lo = mid; else hi = mid - 1;
    }
    return bl[lo] * BT + (j - pre[lo]);
}

// One block per (split, sequence): scores of its share of the token list,
// softmax statistics of that share, and the unnormalised weighted sum of V.
template <typename T>
__device__ __forceinline__ void load4(const T* row, int gi, float* o);
template <>
__device__ __forceinline__ void load4<uint16_t>(const uint16_t* row, int gi, float* o) {
    const uint2 w = __ldg(reinterpret_cast<const uint2*>(row) + gi);
    o[0] = bf16_lo(w.x); o[1] = bf16_hi(w.x); o[2] = bf16_lo(w.y); o[3] = bf16_hi(w.y);
}
template <>
__device__ __forceinline__ void load4<float>(const float* row, int gi, float* o) {
    const float4 w = __ldg(reinterpret_cast<const float4*>(row) + gi);
    o[0] = w.x; o[1] = w.y; o[2] = w.z; o[3] = w.w;
}

template <typename T>
__global__ void __launch_bounds__(BSA_THREADS) bsa_split_kernel(const BsaArgs a) {
    extern __shared__ float bsm[];
    const int split = blockIdx.x, s = blockIdx.y;
    const int D = a.k.D, ng = D >> 2;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int* pre = reinterpret_cast<int*>(bsm);                  // n_sel + 1
    float* red = bsm + (a.n_sel + 1);                        // BSA_WARPS
    float* sc = red + BSA_WARPS;                             // split_tokens
    float* wacc = sc + a.split_tokens;                       // BSA_WARPS x D
    __shared__ unsigned wt[8];
    const int32_t* bl = a.blocks + (int64_t)s * a.blocks_stride;

    // running list lengths (block lengths clipped to the sequence)
    unsigned base = 0;
    for (int c0 = 0; c0 < a.n_sel; c0 += BSA_THREADS) {
        const int i = c0 + threadIdx.x;
        unsigned len = 0;
        if (i < a.n_sel) {
            const int b = bl[i];
            if (b < 0) {
                atomicOr(a.status, 2);
            } else {
                const int64_t st = (int64_t)b * a.block_tokens;
                const int64_t en = min(st + a.block_tokens, (int64_t)a.k.seq_len);
                len = en > st ? (unsigned)(en - st) : 0u;
            }
        }
        const unsigned incl = block_scan_incl_256(len, wt);
        const unsigned total = wt[7];
        if (i < a.n_sel) pre[i] = (int)(base + incl - len);
        base += total;
        __syncthreads();
    }
    if (threadIdx.x == 0) pre[a.n_sel] = (int)base;
    __syncthreads();
    const int n_list = (int)base;
    const int j0 = split * a.split_tokens;
    const int j1 = min(n_list, j0 + a.split_tokens);
    float* part = a.part + ((int64_t)s * a.splits + split) * (2 + D);
    if (j0 >= j1) {
        for (int d = threadIdx.x; d < D + 2; d += BSA_THREADS)
            part[d] = d == 0 ? -INFINITY : 0.0f;
        return;
    }

    const T* kbase = std::is_same<T, float>::value ? reinterpret_cast<const T*>(a.kf)
                                                  : reinterpret_cast<const T*>(a.k.pages);
    const T* vbase = std::is_same<T, float>::value ? reinterpret_cast<const T*>(a.vf)
                                                  : reinterpret_cast<const T*>(a.v);
    const T* qrow = (std::is_same<T, float>::value ? reinterpret_cast<const T*>(a.qf32)
                                                   : reinterpret_cast<const T*>(a.q)) +
                    (int64_t)s * D;
    // q in registers: lane owns column groups lane + 32g
    float qf[PK_GROUPS][4];
#pragma unroll
    for (int g = 0; g < PK_GROUPS; ++g) {
        const int gi = lane + 32 * g;
        if (gi < ng) load4<T>(qrow, gi, qf[g]);
        else qf[g][0] = qf[g][1] = qf[g][2] = qf[g][3] = 0.0f;
    }

    // pass 1: s_j = (q . k_j) * scale; four tokens per warp in flight
    for (int jb = j0 + warp * 4; jb < j1; jb += BSA_WARPS * 4) {
        float kv[4][PK_GROUPS][4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int j = jb + u;
            const T* row = nullptr;
            if (j < j1) row = token_row<T>(a.k, kbase, s, list_token(pre, bl, a.n_sel, a.block_tokens, j), a.status);
#pragma unroll
            for (int g = 0; g < PK_GROUPS; ++g) {
                const int gi = lane + 32 * g;
                if (row && gi < ng) load4<T>(row, gi, kv[u][g]);
                else kv[u][g][0] = kv[u][g][1] = kv[u][g][2] = kv[u][g][3] = 0.0f;
            }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            float dot = 0.0f;
#pragma unroll
            for (int g = 0; g < PK_GROUPS; ++g) {
                dot = fmaf(qf[g][0], kv[u][g][0], dot);
                dot = fmaf(qf[g][1], kv[u][g][1], dot);
                dot = fmaf(qf[g][2], kv[u][g][2], dot);
                dot = fmaf(qf[g][3], kv[u][g][3], dot);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
            if (lane == 0 && jb + u < j1) sc[jb + u - j0] = dot * a.scale;
        }
    }
    __syncthreads();

    // softmax statistics of this share (max subtracted, as :93-108)
    float m = -INFINITY;
    for (int j = threadIdx.x; j < j1 - j0; j += BSA_THREADS) m = fmaxf(m, sc[j]);
    m = block_reduce_max(m, red);
    float l = 0.0f;
    for (int j = threadIdx.x; j < j1 - j0; j += BSA_THREADS) {
        const float e = expf(sc[j] - m);
        sc[j] = e;
        l += e;
    }
    l = block_reduce_sum(l, red);

    // pass 2: sum_j e_j * v_j, per warp, then across warps in a fixed order
    float acc[PK_GROUPS][4];
#pragma unroll
    for (int g = 0; g < PK_GROUPS; ++g)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[g][i] = 0.0f;
    for (int jb = j0 + warp * 4; jb < j1; jb += BSA_WARPS * 4) {
        float vv[4][PK_GROUPS][4];
        float e[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int j = jb + u;
            const T* row = nullptr;
            e[u] = 0.0f;
            if (j < j1) {
                row = token_row<T>(a.k, vbase, s, list_token(pre, bl, a.n_sel, a.block_tokens, j), a.status);
                e[u] = sc[j - j0];
            }
#pragma unroll
            for (int g = 0; g < PK_GROUPS; ++g) {
                const int gi = lane + 32 * g;
                if (row && gi < ng) load4<T>(row, gi, vv[u][g]);
                else vv[u][g][0] = vv[u][g][1] = vv[u][g][2] = vv[u][g][3] = 0.0f;
            }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int g = 0; g < PK_GROUPS; ++g)
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[g][i] = fmaf(e[u], vv[u][g][i], acc[g][i]);
    }
#pragma unroll
    for (int g = 0; g < PK_GROUPS; ++g) {
        const int gi = lane + 32 * g;
        if (gi < ng)
#pragma unroll
            for (int i = 0; i < 4; ++i) wacc[warp * D + 4 * gi + i] = acc[g][i];
    }
    __syncthreads();
    for (int d = threadIdx.x; d < D; d += BSA_THREADS) {
        float t = 0.0f;
        for (int w = 0; w < BSA_WARPS; ++w) t += wacc[w * D + d];
        part[2 + d] = t;
    }
    if (threadIdx.x == 0) { part[0] = m; part[1] = l; }
}

// Page-granular form for blocks that start on page boundaries
// (block_tokens % page_tokens == 0) and D in {64, 128, 256}: the selected
// token list is then a list of whole pages (the last one of a block may be
// cut by seq_len).  A warp takes one page at a time, loading its K and V rows
// with 16-byte loads (lane l of load i holds 8 columns of token i*TPI + l/G),
// and keeps an online softmax (running max, rescaled sum and output), so K and
// V stream through in a single pass.  The warps of a block then merge their
// (max, sum, output) triples.
template <int D, int PT>
__global__ void __launch_bounds__(BSA_THREADS) bsa_page_kernel(const BsaArgs a) {
    constexpr int G = D / 8;        // lanes per token
    constexpr int TPI = 32 / G;     // tokens per load instruction
    constexpr int NLD = PT / TPI;   // load instructions per page
    static_assert(PT % TPI == 0, "page must fill whole load instructions");
    extern __shared__ float bsm[];
    const int split = blockIdx.x, s = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int ppb = a.block_tokens / PT;
    int* pre = reinterpret_cast<int*>(bsm);               // n_sel + 1 page counts
    float* wm = bsm + (a.n_sel + 1);                      // BSA_WARPS
    float* wl = wm + BSA_WARPS;                           // BSA_WARPS
    float* wacc = wl + BSA_WARPS;                         // BSA_WARPS x D
    __shared__ unsigned wt[8];
    const int32_t* bl = a.blocks + (int64_t)s * a.blocks_stride;

    unsigned base = 0;
    for (int c0 = 0; c0 < a.n_sel; c0 += BSA_THREADS) {
        const int i = c0 + threadIdx.x;
        unsigned np = 0;
        if (i < a.n_sel) {
            const int b = bl[i];
            if (b < 0) {
                atomicOr(a.status, 2);
            } else {
                const int64_t st = (int64_t)b * a.block_tokens;
                const int64_t en = min(st + a.block_tokens, (int64_t)a.k.seq_len);
                np = en > st ? (unsigned)((en - st + PT - 1) / PT) : 0u;
            }
        }
        const unsigned incl = block_scan_incl_256(np, wt);
        const unsigned total = wt[7];
        if (i < a.n_sel) pre[i] = (int)(base + incl - np);
        base += total;
        __syncthreads();
    }
    const int n_list = (int)base;    // pages in the list
    const int P0 = split * a.split_tokens;   // split_tokens counts pages here
    const int P1 = min(n_list, P0 + a.split_tokens);

    const int col = (lane % G) * 8;
    float qf[8];
    {
        const uint4 w = __ldg(reinterpret_cast<const uint4*>(a.q + (int64_t)s * D + col));
        qf[0] = bf16_lo(w.x); qf[1] = bf16_hi(w.x); qf[2] = bf16_lo(w.y); qf[3] = bf16_hi(w.y);
        qf[4] = bf16_lo(w.z); qf[5] = bf16_hi(w.z); qf[6] = bf16_lo(w.w); qf[7] = bf16_hi(w.w);
    }
    float m_w = -INFINITY, l_w = 0.0f, acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.0f;

    for (int P = P0 + warp; P < P1; P += BSA_WARPS) {
        // list page P -> (selected block i, page j of that block)
        int lo = 0, hi = a.n_sel - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (pre[mid] <= P) lo = mid; else hi = mid - 1;
        }
        const int j = P - pre[lo];
        const int64_t t0 = (int64_t)bl[lo] * a.block_tokens + (int64_t)j * PT;
        const int valid = (int)min((int64_t)PT, (int64_t)a.k.seq_len - t0);
        const int lp = bl[lo] * ppb + j;
        const int32_t phys = __ldg(a.k.table + (int64_t)s * a.k.pages_per_seq + lp);
        if (phys < 0 || (int64_t)phys >= a.k.n_pages) {
            if (lane == 0) atomicOr(a.status, 1);
            continue;
        }
        const uint4* kr = reinterpret_cast<const uint4*>(a.k.pages + (int64_t)phys * PT * D);
        const uint4* vr = reinterpret_cast<const uint4*>(a.v + (int64_t)phys * PT * D);
        uint4 kv[NLD], vv[NLD];
#pragma unroll
        for (int i = 0; i < NLD; ++i) kv[i] = __ldg(kr + i * 32 + lane);
#pragma unroll
        for (int i = 0; i < NLD; ++i) vv[i] = __ldg(vr + i * 32 + lane);
        float sc[NLD];
        float mp = -INFINITY;
#pragma unroll
        for (int i = 0; i < NLD; ++i) {
            float d = qf[0] * bf16_lo(kv[i].x);
            d = fmaf(qf[1], bf16_hi(kv[i].x), d);
            d = fmaf(qf[2], bf16_lo(kv[i].y), d);
            d = fmaf(qf[3], bf16_hi(kv[i].y), d);
            d = fmaf(qf[4], bf16_lo(kv[i].z), d);
            d = fmaf(qf[5], bf16_hi(kv[i].z), d);
            d = fmaf(qf[6], bf16_lo(kv[i].w), d);
            d = fmaf(qf[7], bf16_hi(kv[i].w), d);
#pragma unroll
            for (int o = G / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
            const int tok = i * TPI + lane / G;
            sc[i] = tok < valid ? d * a.scale : -INFINITY;
            mp = fmaxf(mp, sc[i]);
        }
#pragma unroll
        for (int o = G; o < 32; o <<= 1) mp = fmaxf(mp, __shfl_xor_sync(0xffffffffu, mp, o));
        const float m_new = fmaxf(m_w, mp);
        const float corr = expf(m_w - m_new);
        l_w *= corr;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] *= corr;
#pragma unroll
        for (int i = 0; i < NLD; ++i) {
            const float p = expf(sc[i] - m_new);     // 0 for masked tokens
            if (lane % G == 0) l_w += p;
            acc[0] = fmaf(p, bf16_lo(vv[i].x), acc[0]);
            acc[1] = fmaf(p, bf16_hi(vv[i].x), acc[1]);
            acc[2] = fmaf(p, bf16_lo(vv[i].y), acc[2]);
            acc[3] = fmaf(p, bf16_hi(vv[i].y), acc[3]);
            acc[4] = fmaf(p, bf16_lo(vv[i].z), acc[4]);
            acc[5] = fmaf(p, bf16_hi(vv[i].z), acc[5]);
            acc[6] = fmaf(p, bf16_lo(vv[i].w), acc[6]);
            acc[7] = fmaf(p, bf16_hi(vv[i].w), acc[7]);
        }
        m_w = m_new;
    }
    // lanes l, l+G, ... hold the same columns for different tokens
#pragma unroll
    for (int o = G; o < 32; o <<= 1)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], o);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l_w += __shfl_xor_sync(0xffffffffu, l_w, o);
    if (lane < G)
#pragma unroll
        for (int e = 0; e < 8; ++e) wacc[warp * D + col + e] = acc[e];
    if (lane == 0) { wm[warp] = m_w; wl[warp] = l_w; }
    __syncthreads();
    float M = -INFINITY;
    for (int w = 0; w < BSA_WARPS; ++w) M = fmaxf(M, wm[w]);
    float* part = a.part + ((int64_t)s * a.splits + split) * (2 + D);
    for (int d = threadIdx.x; d < D; d += BSA_THREADS) {
        float t = 0.0f;
        for (int w = 0; w < BSA_WARPS; ++w)
            if (wm[w] != -INFINITY) t += expf(wm[w] - M) * wacc[w * D + d];
        part[2 + d] = t;
    }
    if (threadIdx.x == 0) {
        float L = 0.0f;
        for (int w = 0; w < BSA_WARPS; ++w)
            if (wm[w] != -INFINITY) L += expf(wm[w] - M) * wl[w];
        part[0] = M;
        part[1] = L;
    }
}

// out[d] = sum_s e^(m_s - M) acc_s[d] / sum_s e^(m_s - M) l_s; zeros for an
// empty token list (block_sparse_attention.cpp:42-47, 67-71).  One block per
// sequence.  The max reduces over the splits in parallel; then, a chunk of
// CMB_CHUNK splits at a time, the weights f_s = e^(m_s - M) (0 for an empty
// split) go to shared memory, thread (g, d) adds f_s acc_s[d] over splits g,
// g + G, ... of the chunk (G = CMB_THREADS / D groups, eight loads in flight per
// batch), and each thread adds f_s l_s over its own splits.  Partial sums are
// combined in group / warp order, so results repeat bit for bit.
constexpr int CMB_THREADS = 512;
constexpr int CMB_WARPS = CMB_THREADS / 32;
constexpr int CMB_CHUNK = 2048;
static_assert(PK_MAX_D <= CMB_THREADS, "one column per thread at least");

template <bool IS_MAX>
__device__ __forceinline__ float cmb_reduce(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float u = __shfl_xor_sync(0xffffffffu, v, o);
        v = IS_MAX ? fmaxf(v, u) : v + u;
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float r = red[0];
    for (int w = 1; w < CMB_WARPS; ++w) r = IS_MAX ? fmaxf(r, red[w]) : r + red[w];
    __syncthreads();
    return r;
}

__global__ void __launch_bounds__(CMB_THREADS) bsa_combine_kernel(const float* __restrict__ part,
                                                                   int splits, int D,
                                                                   float* __restrict__ out) {
    __shared__ float red[CMB_WARPS];
    __shared__ float tsum[CMB_THREADS];
    __shared__ float fs[CMB_CHUNK];
    const int s = blockIdx.x;
    const int64_t stride = 2 + D;
    const float* p = part + (int64_t)s * splits * stride;
    float m = -INFINITY;
    for (int i = threadIdx.x; i < splits; i += CMB_THREADS) m = fmaxf(m, p[i * stride]);
    const float M = cmb_reduce<true>(m, red);
    const int G = CMB_THREADS / D;
    const int g = threadIdx.x / D, d = threadIdx.x % D;
    float l = 0.0f, t = 0.0f;
    for (int c0 = 0; c0 < splits; c0 += CMB_CHUNK) {
        const int cn = min(CMB_CHUNK, splits - c0);
        for (int i = threadIdx.x; i < cn; i += CMB_THREADS) {
            const float* pi = p + (c0 + i) * stride;
            const float f = pi[0] != -INFINITY ? expf(pi[0] - M) : 0.0f;
            fs[i] = f;
            l += f * pi[1];
        }
        __syncthreads();
        if (g < G) {
            const float* col = p + (int64_t)c0 * stride + 2 + d;
            int i = g;
            for (; i + 7 * G < cn; i += 8 * G) {
                float x[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) x[u] = col[(i + u * G) * stride];
#pragma unroll
                for (int u = 0; u < 8; ++u) t += fs[i + u * G] * x[u];
            }
            for (; i < cn; i += G) t += fs[i] * col[i * stride];
        }
        __syncthreads();   // fs is rewritten by the next chunk
    }
    const float L = cmb_reduce<false>(l, red);
    if (g < G) tsum[threadIdx.x] = t;
    __syncthreads();
    if (threadIdx.x < D) {
        float o = 0.0f;
        for (int h = 0; h < G; ++h) o += tsum[h * D + threadIdx.x];
        out[(int64_t)s * D + threadIdx.x] = M == -INFINITY ? 0.0f : o / L;
    }
}

// ------------------------------------------------------ fused selection
// Per sequence: score each block summary against q (fp32, d ascending,
// fl(fl(S*q) + acc), inner_product_compute.cpp:23-29), then keep the best
// `top` (topk_retrieval.cpp:13-31; ties to the lowest block id).
// MINMAX: summ rows are [block][2][D] (min, max) and a block's score is the
// upper bound of q.k over its keys, sum_j max(q_j * min_j, q_j * max_j) in j
// order; otherwise rows are [block][D] and the score is q . summary.
template <bool MINMAX>
__global__ void __launch_bounds__(SEL_THREADS_MAX) block_select_kernel(
    const float* __restrict__ summ, int n_blocks, int D, const uint16_t* __restrict__ q, int top,
    int32_t* __restrict__ sel) {
    extern __shared__ unsigned char ssm[];
    const int s = blockIdx.x;
    const int n2 = next_pow2(n_blocks);
    uint64_t* keys = reinterpret_cast<uint64_t*>(ssm);
    float* qf = reinterpret_cast<float*>(keys + n2);
    for (int d = threadIdx.x; d < D; d += blockDim.x)
        qf[d] = bf16_bits_to_f32(q[(int64_t)s * D + d]);
    __syncthreads();
    const float* S = summ + (int64_t)s * n_blocks * D * (MINMAX ? 2 : 1);
    // one thread per summary row (blockDim >= n2 up to SEL_THREADS_MAX); each
    // thread keeps 8 16-byte loads of its row (4 of each bound row) in flight
    // ahead of the in-order sum (the reference's separate multiply and add)
    constexpr int U = MINMAX ? 4 : 8;
    for (int b = threadIdx.x; b < n2; b += blockDim.x) {
        uint64_t key = 0ull;
        if (b < n_blocks) {
            const float4* lo = reinterpret_cast<const float4*>(S + (int64_t)b * (MINMAX ? 2 : 1) * D);
            const float4* hi = lo + (D >> 2);
            float acc = 0.0f;
            for (int d0 = 0; d0 < (D >> 2); d0 += U) {
                float4 a[U], z[U];
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const bool in = d0 + u < (D >> 2);
                    a[u] = in ? __ldg(lo + d0 + u) : make_float4(0.f, 0.f, 0.f, 0.f);
                    if (MINMAX) z[u] = in ? __ldg(hi + d0 + u) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    if (d0 + u >= (D >> 2)) break;
                    const float av[4] = {a[u].x, a[u].y, a[u].z, a[u].w};
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float qv = qf[4 * (d0 + u) + i];
                        if (MINMAX) {
                            const float zv[4] = {z[u].x, z[u].y, z[u].z, z[u].w};
                            const float l = __fmul_rn(qv, av[i]);
                            const float h = __fmul_rn(qv, zv[i]);
                            acc = __fadd_rn(acc, l > h ? l : h);
                        } else {
                            acc = __fadd_rn(acc, __fmul_rn(av[i], qv));
                        }
                    }
                }
            }
            key = make_cand(f32_key(acc), (uint32_t)b);
        }
        keys[b] = key;
    }
    block_bitonic_sort_desc(keys, n2);
    const int m = min(top, n_blocks);
    for (int i = threadIdx.x; i < top; i += blockDim.x)
        sel[(int64_t)s * top + i] = i < m ? (int32_t)cand_row(keys[i]) : -1;
}

// ---------------------------------------------------------------- host
// Threads of the block selection: one per summary row, 128 .. SEL_THREADS_MAX.
int select_threads(int n2) { return std::max(128, std::min(SEL_THREADS_MAX, n2)); }

struct BsaPlan {
    int splits, split_tokens;
    size_t smem, part_bytes;
};

BsaPlan bsa_plan(int64_t n_seq, int64_t n_sel, int64_t block_tokens, int64_t D) {
    BsaPlan p;
    const int64_t max_tokens = std::max<int64_t>(1, n_sel * block_tokens);
    const int64_t sms = device_sm_count();
    int64_t want = (8 * sms + n_seq - 1) / std::max<int64_t>(1, n_seq);
    int64_t by_tokens = (max_tokens + BSA_MIN_SPLIT_TOKENS - 1) / BSA_MIN_SPLIT_TOKENS;
    int64_t sp = std::max<int64_t>(1, std::min(want, by_tokens));
    sp = std::max<int64_t>(sp, (max_tokens + BSA_MAX_SPLIT_TOKENS - 1) / BSA_MAX_SPLIT_TOKENS);
    p.splits = (int)sp;
    p.split_tokens = (int)((max_tokens + sp - 1) / sp);
    p.smem = sizeof(int) * (n_sel + 1) + sizeof(float) * (BSA_WARPS + p.split_tokens) +
             sizeof(float) * BSA_WARPS * D;
    p.part_bytes = sizeof(float) * (size_t)n_seq * p.splits * (2 + D);
    return p;
}

size_t up256(size_t v) { return (v + 255) & ~size_t(255); }

BsaPlan bsa_page_plan(int64_t n_seq, int64_t n_sel, int64_t block_tokens, int64_t page_tokens,
                      int64_t D);

// Partial-result bytes that cover both the token-granular and the
// page-granular plans (the page path has 16-token pages, so its plan is
// computed for page_tokens 16).
size_t bsa_part_bytes(int64_t n_seq, int64_t n_sel, int64_t block_tokens, int64_t D) {
    const BsaPlan t = bsa_plan(n_seq, n_sel, block_tokens, D);
    const BsaPlan g = bsa_page_plan(n_seq, n_sel, block_tokens, 16, D);
    return std::max(t.part_bytes, g.part_bytes);
}

hmm_status_t check_cache(const void* pages, int64_t n_pages, const int32_t* table, int64_t n_seq,
                         int64_t pages_per_seq, int64_t seq_len, int64_t page_tokens, int64_t D) {
    HMM_REQUIRE(n_seq >= 0 && n_seq <= 65535, "n_seq must be in [0, 65535], got %lld",
                (long long)n_seq);
    HMM_REQUIRE(D >= 4 && D <= PK_MAX_D && D % 4 == 0,
                "D must be a multiple of 4 in [4, %d], got %lld", PK_MAX_D, (long long)D);
    HMM_REQUIRE(page_tokens >= 1, "page_tokens must be >= 1");
    HMM_REQUIRE(pages_per_seq >= 0 && n_pages >= 0, "negative page counts");
    HMM_REQUIRE(seq_len >= 0 && seq_len <= pages_per_seq * page_tokens,
                "seq_len %lld exceeds pages_per_seq * page_tokens", (long long)seq_len);
    HMM_REQUIRE(seq_len < (int64_t(1) << 31), "seq_len must be < 2^31");
    HMM_REQUIRE(n_seq == 0 || seq_len == 0 || (pages && table), "null cache pointer");
    HMM_REQUIRE((reinterpret_cast<uintptr_t>(pages) % 8) == 0,
                "page array must be 8-byte aligned");
    return HMM_OK;
}

// Reads the device status word written by the kernels (waits for the stream).
hmm_status_t read_status(const int* status, cudaStream_t st, const char* what) {
    int h = 0;
    HMM_CUDA_TRY(cudaMemcpyAsync(&h, status, sizeof(int), cudaMemcpyDeviceToHost, st));
    HMM_CUDA_TRY(cudaStreamSynchronize(st));
    if (h & HMM_STATUS_PAGE_BOUNDS)
        return set_error(HMM_ERR_BOUNDS, "%s: a page-table entry is outside [0, n_pages)", what);
    if (h & HMM_STATUS_BLOCK_BOUNDS)
        return set_error(HMM_ERR_BOUNDS, "%s: a selected block id is negative", what);
    if (h & HMM_STATUS_TIMEOUT)
        return set_error(HMM_ERR_TIMEOUT, "%s: a bounded pipeline wait gave up; outputs invalid",
                         what);
    if (h & HMM_STATUS_POOL_OVERFLOW)
        return set_error(HMM_ERR_UNSUPPORTED,
                         "%s: a candidate pool filled up (rows ordered so that the k-th best "
                         "keeps rising); outputs incomplete: recompute with hmm_ip_topk_bf16",
                         what);
    return HMM_OK;
}

// Resident blocks per SM of the page kernel for head size D with `smem`
// bytes of dynamic shared memory on the current device (0 if unknown).
int page_kernel_blocks_per_sm(int64_t D, size_t smem) {
    int n = 0;
    cudaError_t e = cudaErrorInvalidValue;
    if (D == 64)
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, bsa_page_kernel<64, 16>, BSA_THREADS, smem);
    else if (D == 128)
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, bsa_page_kernel<128, 16>, BSA_THREADS, smem);
    else if (D == 256)
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, bsa_page_kernel<256, 16>, BSA_THREADS, smem);
    if (e != cudaSuccess) {
        cudaGetLastError();   // a failed query leaves no sticky error behind
        return 0;
    }
    return n;
}

// Page-granular plan: splits over the pages of the selected list.  A split
// carries fixed costs (its page-list scan, its partial result, its share of
// the combine), and measured on a B200 fewer, longer splits win: at 256
// sequences of 256 pages 4 splits took 101 us, 8 took 102-105, 16 took 117;
// at 64 sequences 4, 8, 16 took 31, 33, 37 us.  So a split gets 64 pages (8
// per warp) or more, and more splits only when the sequences are too few to
// give every resident block slot of the GPU one (a single decode sequence
// spreads over up to 32 blocks of 8 pages).
BsaPlan bsa_page_plan(int64_t n_seq, int64_t n_sel, int64_t block_tokens, int64_t page_tokens,
                      int64_t D) {
    BsaPlan p;
    const int64_t max_pages = std::max<int64_t>(1, n_sel * (block_tokens / page_tokens));
    const int64_t sms = device_sm_count();
    const int64_t by_pages = (max_pages + BSA_MIN_SPLIT_PAGES - 1) / BSA_MIN_SPLIT_PAGES;
    p.smem = sizeof(int) * (n_sel + 1) + sizeof(float) * (2 * BSA_WARPS + BSA_WARPS * D);
    const int64_t per_sm = page_kernel_blocks_per_sm(D, p.smem);
    const int64_t slots = sms * (per_sm > 0 ? per_sm : 2);
    const int64_t fill = slots / std::max<int64_t>(1, n_seq);   // splits giving each slot a block
    const int64_t sp = std::max<int64_t>(
        1, std::min(by_pages, std::max((max_pages + BSA_PAGES_PER_SPLIT - 1) / BSA_PAGES_PER_SPLIT,
                                       fill)));
    p.splits = (int)sp;
    p.split_tokens = (int)((max_pages + sp - 1) / sp);   // pages per split
    p.part_bytes = sizeof(float) * (size_t)n_seq * p.splits * (2 + D);
    return p;
}

template <int D, int PT>
hmm_status_t launch_page_kernel(BsaArgs a, const BsaPlan& p, int64_t n_seq, cudaStream_t st) {
    auto kern = bsa_page_kernel<D, PT>;
    HMM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)p.smem));
    kern<<<dim3((unsigned)p.splits, (unsigned)n_seq), BSA_THREADS, p.smem, st>>>(a);
    return check_launch("bsa_page_kernel");
}

bool page_path_applies(int64_t D, int64_t page_tokens, int64_t block_tokens, const void* k,
                       const void* v, const void* q) {
    return page_tokens == 16 && (D == 64 || D == 128 || D == 256) &&
           block_tokens % page_tokens == 0 && (reinterpret_cast<uintptr_t>(k) % 16) == 0 &&
           (reinterpret_cast<uintptr_t>(v) % 16) == 0 && (reinterpret_cast<uintptr_t>(q) % 16) == 0;
}

hmm_status_t run_bsa(const BsaArgs& a0, int64_t n_seq, int64_t D, float* out, unsigned char* ws,
                     size_t ws_bytes, cudaStream_t st) {
    if (!a0.kf && !a0.k.contiguous &&
        page_path_applies(D, a0.k.page_tokens, a0.block_tokens, a0.k.pages, a0.v, a0.q)) {
        const BsaPlan p = bsa_page_plan(n_seq, a0.n_sel, a0.block_tokens, a0.k.page_tokens, D);
        const size_t need = up256(p.part_bytes) + 256;
        if (!ws || ws_bytes < need)
            return set_error(HMM_ERR_OOM, "workspace too small: %zu < %zu", ws_bytes, need);
        BsaArgs a = a0;
        a.splits = p.splits;
        a.split_tokens = p.split_tokens;
        a.part = reinterpret_cast<float*>(ws);
        const ProfileMark pm = profile_begin(st);
        hmm_status_t s = D == 64    ? launch_page_kernel<64, 16>(a, p, n_seq, st)
                         : D == 128 ? launch_page_kernel<128, 16>(a, p, n_seq, st)
                                    : launch_page_kernel<256, 16>(a, p, n_seq, st);
        profile_end(pm, st);
        if (s != HMM_OK) return s;
        bsa_combine_kernel<<<(unsigned)n_seq, CMB_THREADS, 0, st>>>(a.part, p.splits, (int)D, out);
        return check_launch("bsa_combine_kernel");
    }
    const BsaPlan p = bsa_plan(n_seq, a0.n_sel, a0.block_tokens, D);
    const size_t need = up256(p.part_bytes) + 256;
    if (!ws || ws_bytes < need)
        return set_error(HMM_ERR_OOM, "workspace too small: %zu < %zu", ws_bytes, need);
    BsaArgs a = a0;
    a.splits = p.splits;
    a.split_tokens = p.split_tokens;
    a.part = reinterpret_cast<float*>(ws);
    const bool f32 = a.kf != nullptr;
    auto kern = f32 ? bsa_split_kernel<float> : bsa_split_kernel<uint16_t>;
    HMM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)p.smem));
    const ProfileMark pm = profile_begin(st);
    kern<<<dim3((unsigned)p.splits, (unsigned)n_seq), BSA_THREADS, p.smem, st>>>(a);
    hmm_status_t s = check_launch("bsa_split_kernel");
    profile_end(pm, st);
    if (s != HMM_OK) return s;
    bsa_combine_kernel<<<(unsigned)n_seq, CMB_THREADS, 0, st>>>(a.part, p.splits, (int)D, out);
    return check_launch("bsa_combine_kernel");
}

}  // namespace
}  // namespace hmm

using namespace hmm;

extern "C" hmm_status_t hmm_paged_kv_summary_f32(const float* keys, int64_t n_seq, int64_t L,
                                                 int64_t D, const float* weight, int64_t out_dim,
                                                 int64_t page_size, float* out, void* stream) {
    HMM_REQUIRE(n_seq >= 0 && n_seq <= 65535, "n_seq must be in [0, 65535]");
    HMM_REQUIRE(L >= 0 && L < (int64_t(1) << 31), "L out of range");
    HMM_REQUIRE(D >= 0 && D <= 12288, "D must be in [0, 12288]");
    HMM_REQUIRE(page_size >= 1, "page_size must be >= 1, got %lld", (long long)page_size);
    HMM_REQUIRE(!weight || out_dim >= 1, "out_dim must be >= 1 with a weight");
    // the reference returns an empty memory for empty keys (:30-44)
    if (n_seq == 0 || L == 0 || D == 0 || (weight && out_dim == 0)) return HMM_OK;
    HMM_REQUIRE(keys && out, "null pointer");
    const int64_t pages = (L + page_size - 1) / page_size;
    HMM_REQUIRE(pages <= 2147483647, "too many pages");
    const int od = weight ? (int)out_dim : (int)D;
    kv_summary_f32_kernel<<<dim3((unsigned)pages, (unsigned)n_seq), 256, sizeof(float) * D,
                            static_cast<cudaStream_t>(stream)>>>(keys, (int)L, (int)D, weight, od,
                                                                 (int)page_size, (int)pages, out);
    return check_launch("kv_summary_f32_kernel");
}

extern "C" size_t hmm_paged_workspace_size(int64_t n_seq, int64_t n_sel, int64_t block_tokens,
                                           int64_t D) {
    if (n_seq < 0 || n_sel < 0 || block_tokens < 1 || D < 0) return 0;
    return up256(bsa_part_bytes(n_seq, n_sel, block_tokens, D)) + 256 +
           up256(sizeof(int32_t) * (size_t)n_seq * n_sel) + 256;
}

extern "C" hmm_status_t hmm_paged_kv_summary_bf16(const uint16_t* k_pages, int64_t n_pages,
                                                  const int32_t* page_table, int64_t n_seq,
                                                  int64_t pages_per_seq, int64_t seq_len,
                                                  int64_t page_tokens, int64_t block_tokens,
                                                  int64_t D, float* out, void* workspace,
                                                  size_t workspace_bytes, void* stream) {
    hmm_status_t s = check_cache(k_pages, n_pages, page_table, n_seq, pages_per_seq, seq_len,
                                 page_tokens, D);
    if (s != HMM_OK) return s;
    HMM_REQUIRE(block_tokens >= 1, "block_tokens must be >= 1");
    if (n_seq == 0 || seq_len == 0) return HMM_OK;
    HMM_REQUIRE(out, "out is null");
    HMM_REQUIRE(workspace && workspace_bytes >= 256, "workspace must hold >= 256 bytes");
    HMM_REQUIRE((reinterpret_cast<uintptr_t>(out) % 16) == 0, "out must be 16-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int* status = static_cast<int*>(workspace);
    HMM_CUDA_TRY(cudaMemsetAsync(status, 0, sizeof(int), st));
    PagedCache c{k_pages, page_table, n_pages, (int)pages_per_seq, (int)seq_len,
                 (int)page_tokens, (int)D, false};
    const int n_blocks = (int)((seq_len + block_tokens - 1) / block_tokens);
    const int64_t units = n_seq * n_blocks;
    const unsigned grid = (unsigned)((units + 7) / 8);
    if (D <= 128)
        paged_summary_kernel<1><<<grid, 256, 0, st>>>(c, (int)block_tokens, n_blocks, units, out,
                                                       status);
    else if (D <= 256)
        paged_summary_kernel<2><<<grid, 256, 0, st>>>(c, (int)block_tokens, n_blocks, units, out,
                                                       status);
    else
        paged_summary_kernel<4><<<grid, 256, 0, st>>>(c, (int)block_tokens, n_blocks, units, out,
                                                       status);
    s = check_launch("paged_summary_kernel");
    if (s != HMM_OK) return s;
    return read_status(status, st, "hmm_paged_kv_summary_bf16");
}

extern "C" hmm_status_t hmm_paged_kv_minmax_bf16(const uint16_t* k_pages, int64_t n_pages,
                                                 const int32_t* page_table, int64_t n_seq,
                                                 int64_t pages_per_seq, int64_t seq_len,
                                                 int64_t page_tokens, int64_t block_tokens,
                                                 int64_t D, float* out, void* workspace,
                                                 size_t workspace_bytes, void* stream) {
    hmm_status_t s = check_cache(k_pages, n_pages, page_table, n_seq, pages_per_seq, seq_len,
                                 page_tokens, D);
    if (s != HMM_OK) return s;
    HMM_REQUIRE(block_tokens >= 1, "block_tokens must be >= 1");
    if (n_seq == 0 || seq_len == 0) return HMM_OK;
    HMM_REQUIRE(out, "out is null");
    HMM_REQUIRE(workspace && workspace_bytes >= 256, "workspace must hold >= 256 bytes");
    HMM_REQUIRE((reinterpret_cast<uintptr_t>(out) % 16) == 0, "out must be 16-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int* status = static_cast<int*>(workspace);
    HMM_CUDA_TRY(cudaMemsetAsync(status, 0, sizeof(int), st));
    PagedCache c{k_pages, page_table, n_pages, (int)pages_per_seq, (int)seq_len,
                 (int)page_tokens, (int)D, false};
    const int n_blocks = (int)((seq_len + block_tokens - 1) / block_tokens);
    const int64_t units = n_seq * n_blocks;
    const unsigned grid = (unsigned)((units + 7) / 8);
    if (D <= 128)
        paged_minmax_kernel<1><<<grid, 256, 0, st>>>(c, (int)block_tokens, n_blocks, units, out,
                                                      status);
    else if (D <= 256)
        paged_minmax_kernel<2><<<grid, 256, 0, st>>>(c, (int)block_tokens, n_blocks, units, out,
                                                      status);
    else
        paged_minmax_kernel<4><<<grid, 256, 0, st>>>(c, (int)block_tokens, n_blocks, units, out,
                                                      status);
    s = check_launch("paged_minmax_kernel");
    if (s != HMM_OK) return s;
    return read_status(status, st, "hmm_paged_kv_minmax_bf16");
}

extern "C" hmm_status_t hmm_block_select_minmax(const uint16_t* q, const float* minmax,
                                                int64_t n_seq, int64_t n_blocks, int64_t D,
                                                int64_t top_blocks, int32_t* out_blocks,
                                                void* stream) {
    HMM_REQUIRE(n_seq >= 0 && n_seq <= 65535, "n_seq must be in [0, 65535]");
    HMM_REQUIRE(n_blocks >= 0 && n_blocks <= 16384, "n_blocks must be in [0, 16384]");
    HMM_REQUIRE(D >= 4 && D % 4 == 0 && D <= 1024, "D must be a multiple of 4 in [4, 1024]");
    HMM_REQUIRE(top_blocks >= 1, "top_blocks must be >= 1");
    if (n_seq == 0) return HMM_OK;
    HMM_REQUIRE(q && out_blocks && (minmax || n_blocks == 0), "null pointer");
    HMM_REQUIRE((reinterpret_cast<uintptr_t>(minmax) % 16) == 0, "minmax must be 16-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int n2 = next_pow2((int)std::max<int64_t>(n_blocks, 1));
    const size_t ssm = sizeof(uint64_t) * n2 + sizeof(float) * D;
    HMM_CUDA_TRY(cudaFuncSetAttribute(block_select_kernel<true>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ssm));
    block_select_kernel<true><<<(unsigned)n_seq, select_threads(n2), ssm, st>>>(
        minmax, (int)n_blocks, (int)D, q, (int)top_blocks, out_blocks);
    return check_launch("block_select_kernel");
}

extern "C" hmm_status_t hmm_block_pages(const int32_t* page_table, int64_t n_seq,
                                        int64_t pages_per_seq, const int32_t* blocks,
                                        int64_t n_sel, int64_t pages_per_block,
                                        int32_t* out_pages, int32_t* out_counts, void* stream) {
    HMM_REQUIRE(n_seq >= 0 && n_seq <= 65535, "n_seq must be in [0, 65535]");
    HMM_REQUIRE(n_sel >= 0 && pages_per_block >= 1 && pages_per_seq >= 0, "bad sizes");
    HMM_REQUIRE(n_sel * pages_per_block < (int64_t(1) << 31), "output too large");
    if (n_seq == 0) return HMM_OK;
    HMM_REQUIRE(out_pages || n_sel == 0, "out_pages is null");
    HMM_REQUIRE((page_table || pages_per_seq == 0) && (blocks || n_sel == 0), "null input");
    block_pages_kernel<<<(unsigned)n_seq, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        page_table, (int)pages_per_seq, blocks, (int)n_sel, (int)pages_per_block, out_pages,
        out_counts);
    return check_launch("block_pages_kernel");
}

namespace {
hmm_status_t bsa_common(const uint16_t* q, const uint16_t* k_pages, const uint16_t* v_pages,
                        int64_t n_pages, const int32_t* page_table, int64_t n_seq,
                        int64_t pages_per_seq, int64_t seq_len, int64_t page_tokens,
                        int64_t block_tokens, int64_t D, int64_t n_sel, float* out) {
    hmm_status_t s = check_cache(k_pages, n_pages, page_table, n_seq, pages_per_seq, seq_len,
                                 page_tokens, D);
    if (s != HMM_OK) return s;
    HMM_REQUIRE((reinterpret_cast<uintptr_t>(v_pages) % 8) == 0, "v_pages must be 8-byte aligned");
    HMM_REQUIRE(block_tokens >= 1, "block_tokens must be >= 1");
    HMM_REQUIRE(n_sel >= 0 && n_sel <= BSA_MAX_SEL, "n_sel must be in [0, %d]", BSA_MAX_SEL);
    HMM_REQUIRE(n_seq == 0 || (q && out), "null q / out");
    HMM_REQUIRE(seq_len == 0 || v_pages, "v_pages is null");
    HMM_REQUIRE((reinterpret_cast<uintptr_t>(q) % 8) == 0, "q must be 8-byte aligned");
    return HMM_OK;
}
}  // namespace

extern "C" hmm_status_t hmm_block_sparse_attention_bf16(
    const uint16_t* q, const uint16_t* k_pages, const uint16_t* v_pages, int64_t n_pages,
    const int32_t* page_table, int64_t n_seq, int64_t pages_per_seq, int64_t seq_len,
    int64_t page_tokens, int64_t block_tokens, int64_t D, const int32_t* blocks, int64_t n_sel,
    float* out, void* workspace, size_t workspace_bytes, void* stream) {
    hmm_status_t s = bsa_common(q, k_pages, v_pages, n_pages, page_table, n_seq, pages_per_seq,
                                seq_len, page_tokens, block_tokens, D, n_sel, out);
    if (s != HMM_OK) return s;
    if (n_seq == 0) return HMM_OK;
    HMM_REQUIRE(blocks || n_sel == 0, "blocks is null");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (n_sel == 0 || seq_len == 0) {
        HMM_CUDA_TRY(cudaMemsetAsync(out, 0, sizeof(float) * n_seq * D, st));
        return HMM_OK;
    }
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    const size_t st_off = up256(bsa_part_bytes(n_seq, n_sel, block_tokens, D));
    if (!ws || workspace_bytes < st_off + 256)
        return set_error(HMM_ERR_OOM, "workspace too small: %zu < %zu", workspace_bytes,
                         st_off + 256);
    int* status = reinterpret_cast<int*>(ws + st_off);
    HMM_CUDA_TRY(cudaMemsetAsync(status, 0, sizeof(int), st));
    BsaArgs a{};
    a.k = PagedCache{k_pages, page_table, n_pages, (int)pages_per_seq, (int)seq_len,
                     (int)page_tokens, (int)D, false};
    a.v = v_pages;
    a.q = q;
    a.blocks = blocks;
    a.blocks_stride = (int)n_sel;
    a.n_sel = (int)n_sel;
    a.block_tokens = (int)block_tokens;
    a.scale = 1.0f / sqrtf((float)D);
    a.status = status;
    s = run_bsa(a, n_seq, D, out, ws, st_off + 256, st);
    if (s != HMM_OK) return s;
    return read_status(status, st, "hmm_block_sparse_attention_bf16");
}

extern "C" hmm_status_t hmm_block_sparse_decode_bf16_async(
    const uint16_t* q, const float* summaries, const uint16_t* k_pages, const uint16_t* v_pages,
    int64_t n_pages, const int32_t* page_table, int64_t n_seq, int64_t pages_per_seq,
    int64_t seq_len, int64_t page_tokens, int64_t block_tokens, int64_t D, int64_t top_blocks,
    int32_t* out_blocks, float* out, int32_t* device_status, void* workspace,
    size_t workspace_bytes, void* stream) {
    hmm_status_t s = bsa_common(q, k_pages, v_pages, n_pages, page_table, n_seq, pages_per_seq,
                                seq_len, page_tokens, block_tokens, D, top_blocks, out);
    if (s != HMM_OK) return s;
    HMM_REQUIRE(top_blocks >= 1, "top_blocks must be >= 1");
    if (n_seq == 0) return HMM_OK;
    const int64_t n_blocks = (seq_len + block_tokens - 1) / block_tokens;
    HMM_REQUIRE(n_blocks <= SEL_MAX_BLOCKS, "at most %d blocks per sequence, got %lld",
                SEL_MAX_BLOCKS, (long long)n_blocks);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (n_blocks == 0) {
        if (out_blocks)
            HMM_CUDA_TRY(cudaMemsetAsync(out_blocks, 0xff, sizeof(int32_t) * n_seq * top_blocks, st));
        HMM_CUDA_TRY(cudaMemsetAsync(out, 0, sizeof(float) * n_seq * D, st));
        return HMM_OK;
    }
    HMM_REQUIRE(summaries, "summaries is null");
    HMM_REQUIRE((reinterpret_cast<uintptr_t>(summaries) % 16) == 0,
                "summaries must be 16-byte aligned");
    const size_t st_off = up256(bsa_part_bytes(n_seq, top_blocks, block_tokens, D));
    const size_t sel_off = st_off + 256;
    const size_t need = sel_off + up256(sizeof(int32_t) * (size_t)n_seq * top_blocks) + 256;
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    if (!ws || workspace_bytes < need)
        return set_error(HMM_ERR_OOM, "workspace too small: %zu < %zu", workspace_bytes, need);
    HMM_REQUIRE(device_status, "device_status is null");
    int* status = device_status;
    int32_t* sel = out_blocks ? out_blocks : reinterpret_cast<int32_t*>(ws + sel_off);
    const int n2 = next_pow2((int)n_blocks);
    const size_t ssm = sizeof(uint64_t) * n2 + sizeof(float) * D;
    HMM_CUDA_TRY(cudaFuncSetAttribute(block_select_kernel<false>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ssm));
    block_select_kernel<false><<<(unsigned)n_seq, select_threads(n2), ssm, st>>>(
        summaries, (int)n_blocks, (int)D, q, (int)top_blocks, sel);
    s = check_launch("block_select_kernel");
    if (s != HMM_OK) return s;
    // slots past the number of blocks hold -1: treat them as absent by
    // attending over min(top_blocks, n_blocks) selections
    const int64_t n_sel = std::min<int64_t>(top_blocks, n_blocks);
    BsaArgs a{};
    a.k = PagedCache{k_pages, page_table, n_pages, (int)pages_per_seq, (int)seq_len,
                     (int)page_tokens, (int)D, false};
    a.v = v_pages;
    a.q = q;
    a.blocks = sel;
    a.blocks_stride = (int)top_blocks;
    a.n_sel = (int)n_sel;
    a.block_tokens = (int)block_tokens;
    a.scale = 1.0f / sqrtf((float)D);
    a.status = status;
    return run_bsa(a, n_seq, D, out, ws, st_off + 256, st);
}

extern "C" hmm_status_t hmm_block_sparse_decode_bf16(
    const uint16_t* q, const float* summaries, const uint16_t* k_pages, const uint16_t* v_pages,
    int64_t n_pages, const int32_t* page_table, int64_t n_seq, int64_t pages_per_seq,
    int64_t seq_len, int64_t page_tokens, int64_t block_tokens, int64_t D, int64_t top_blocks,
    int32_t* out_blocks, float* out, void* workspace, size_t workspace_bytes, void* stream) {
    // the status word sits just past the partial results of the workspace
    const size_t st_off = up256(bsa_part_bytes(n_seq, top_blocks, block_tokens, D));
    if (!workspace || workspace_bytes < st_off + 256)
        return set_error(HMM_ERR_OOM, "workspace too small: %zu < %zu", workspace_bytes,
                         st_off + 256);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int* status = reinterpret_cast<int*>(static_cast<unsigned char*>(workspace) + st_off);
    HMM_CUDA_TRY(cudaMemsetAsync(status, 0, sizeof(int), st));
    hmm_status_t s = hmm_block_sparse_decode_bf16_async(
        q, summaries, k_pages, v_pages, n_pages, page_table, n_seq, pages_per_seq, seq_len,
        page_tokens, block_tokens, D, top_blocks, out_blocks, out, status, workspace,
        workspace_bytes, stream);
    if (s != HMM_OK) return s;
    if (n_seq == 0 || seq_len == 0) return HMM_OK;
    return read_status(status, st, "hmm_block_sparse_decode_bf16");
}

extern "C" hmm_status_t hmm_status_read(const int32_t* device_status, void* stream) {
    HMM_REQUIRE(device_status, "device_status is null");
    return read_status(device_status, static_cast<cudaStream_t>(stream), "device status");
}

extern "C" hmm_status_t hmm_block_sparse_attention_f32(const float* q, const float* keys,
                                                       const float* values, int64_t n_seq,
                                                       int64_t L, int64_t D,
                                                       int64_t block_tokens,
                                                       const int32_t* blocks, int64_t n_sel,
                                                       float* out, void* workspace,
                                                       size_t workspace_bytes, void* stream) {
    HMM_REQUIRE(n_seq >= 0 && n_seq <= 65535, "n_seq must be in [0, 65535]");
    HMM_REQUIRE(D >= 4 && D <= PK_MAX_D && D % 4 == 0,
                "D must be a multiple of 4 in [4, %d], got %lld", PK_MAX_D, (long long)D);
    HMM_REQUIRE(L >= 0 && L < (int64_t(1) << 31), "L out of range");
    HMM_REQUIRE(block_tokens >= 1, "block_tokens must be >= 1");
    HMM_REQUIRE(n_sel >= 0 && n_sel <= BSA_MAX_SEL, "n_sel must be in [0, %d]", BSA_MAX_SEL);
    if (n_seq == 0) return HMM_OK;
    HMM_REQUIRE(q && out && (blocks || n_sel == 0), "null pointer");
    HMM_REQUIRE(L == 0 || (keys && values), "null keys / values");
    HMM_REQUIRE((reinterpret_cast<uintptr_t>(q) % 16) == 0 &&
                    (reinterpret_cast<uintptr_t>(keys) % 16) == 0 &&
                    (reinterpret_cast<uintptr_t>(values) % 16) == 0,
                "q, keys and values must be 16-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (n_sel == 0 || L == 0) {
        HMM_CUDA_TRY(cudaMemsetAsync(out, 0, sizeof(float) * n_seq * D, st));
        return HMM_OK;
    }
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    const size_t st_off = up256(bsa_part_bytes(n_seq, n_sel, block_tokens, D));
    if (!ws || workspace_bytes < st_off + 256)
        return set_error(HMM_ERR_OOM, "workspace too small: %zu < %zu", workspace_bytes,
                         st_off + 256);
    int* status = reinterpret_cast<int*>(ws + st_off);
    HMM_CUDA_TRY(cudaMemsetAsync(status, 0, sizeof(int), st));
    BsaArgs a{};
    a.k = PagedCache{nullptr, nullptr, n_seq, 1, (int)L, (int)L, (int)D, true};
    a.kf = keys;
    a.vf = values;
    a.qf32 = q;
    a.blocks = blocks;
    a.blocks_stride = (int)n_sel;
    a.n_sel = (int)n_sel;
    a.block_tokens = (int)block_tokens;
    a.scale = 1.0f / sqrtf((float)D);
    a.status = status;
    hmm_status_t s = run_bsa(a, n_seq, D, out, ws, st_off + 256, st);
    if (s != HMM_OK) return s;
    return read_status(status, st, "hmm_block_sparse_attention_f32");
}
