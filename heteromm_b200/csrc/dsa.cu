// dsa.cu — DSA lightning indexer on tcgen05 FP8 (e4m3) tensor cores.
//
// Reference: indexer_top_ref (kernels/dsa_indexer/indexer_tb.cpp:17-57) with
// the multi-head FP8 form of _fp8_index
// (kernels/deepseek_engram/deepseek_v32_dsa_bench.py:77-101):
//   score[t][j] = sum_h w[t][h] * ReLU(q[t][h] . k[j]),  j visible to t,
// then the top-k keys per query token.  Query token t sits at position
// pos0 + t and sees keys j <= pos0 + t.
//
// One persistent CTA per SM, 12 warps:
//   warp 0      TMA producer: the 256 query rows (4 tokens x 64 heads, or
//               8 x 32, 16 x 16) of a token group into one of two 32 KB
//               buffers, then 128-key x 128-byte tiles into an 8-stage ring
//   warp 1      MMA issuer: per tile 4 x tcgen05.mma.kind::f8f6f4 (M = 128
//               keys, N = 256 query rows, K = 32) into one of two TMEM
//               accumulators of 256 fp32 columns
//   warp 2      TMEM allocator
//   warps 4-19  epilogue, four warpgroups (tile parity x token half):
//               thread = key; per token, sum_h w * max(x, 0) over the
//               token's head columns (weights staged in shared memory per
//               warp and group), causal mask; then (COLLECT) one ballot per
//               warp marks the keys whose upper bound reaches the token's
//               threshold in a bitmap word; (WRITE) coalesced fp32 score rows
// Scores are fp32 tensor-core sums of exact e4m3 products; they differ from
// the exact dot products by the accumulation's rounding.  The selection is
// exact: dsa_exact.cu takes each token's keys whose score could reach the
// k-th (the bitmap), rescores them exactly (integer limbs on the tensor
// cores) and selects the top-k from the exact scores.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "dsa_exact.cuh"
#include "heteromm_cuda.h"
#include "hmm_common.cuh"
#include "sm100_ptx.cuh"

namespace hmm {
using namespace sm100;

namespace {

constexpr int DK = 128;                 // head dim (bytes per fp8 row)
constexpr int KT = 128;                 // keys per tile (MMA M, TMEM lanes)
constexpr int NQ = 256;                 // query rows per group (MMA N)
constexpr int D_STAGES = 8;
constexpr int K_TILE_BYTES = KT * DK;   // 16 KB
constexpr int Q_TILE_BYTES = NQ * DK;   // 32 KB
constexpr int D_EPI_WG = 4;              // epilogue warpgroups: (tile parity, token half)
constexpr int D_THREADS = 128 + 128 * D_EPI_WG;

struct DsaCtrl {
    float wsm[4 * D_EPI_WG][NQ / 2];        // each epilogue warp's token weights for its group
    float esm[4 * D_EPI_WG][8];             // ... its tokens' E_t (COLLECT)
    float tsm[4 * D_EPI_WG][8];             // ... its tokens' thresholds (COLLECT)
    uint64_t a_full[D_STAGES], a_empty[D_STAGES];
    uint64_t q_full[2], q_empty[2];
    uint64_t acc_full[2], acc_empty[2];
    uint32_t tmem_base;
    int abort;
};
constexpr size_t D_SMEM = 1024 + 2 * Q_TILE_BYTES + D_STAGES * K_TILE_BYTES + sizeof(DsaCtrl);

struct DsaArgs {
    const float* w;       // [T][H]
    float* scores;        // [T][L] (WRITE)
    const float* norms;   // [L] ||k_j|| rounded up (COLLECT)
    const float* tok_e;   // [T] E_t (COLLECT)
    const float* tok_tau; // [T] thresholds (COLLECT)
    uint32_t* bitmap;     // [T][W] keys with s~ + E_t ||k_j|| >= tau (COLLECT)
    int W;                // bitmap words per token
    int* status;          // [0] timeout, [1] a row the sampled top-k could not select
    int64_t T, L, pos0;
    int H, tg;            // heads, tokens per group (NQ / H)
    int n_groups, key_tiles;
    uint64_t wait_ns;     // limit of every bounded wait (wait_limit_ns())
};

// Packed fp32 pairs for fma.rn.f32x2 (sm_100a).
__device__ __forceinline__ uint64_t pack_f32x2(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void unpack_f32x2(uint64_t v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

__device__ __forceinline__ int group_tiles(const DsaArgs& a, int g) {
    const int64_t t_last = min(a.T, (int64_t)(g + 1) * a.tg) - 1;
    const int64_t vis = a.pos0 + t_last + 1;            // keys visible to the group's last token
    if (vis <= 0) return 0;
    return (int)min((int64_t)a.key_tiles, (vis + KT - 1) / KT);
}

__device__ __forceinline__ bool wait_all(uint64_t* bar, uint32_t parity, volatile int* abort,
                                         uint64_t limit_ns) {
    const bool ok = mbar_wait_bounded(bar, parity, abort, limit_ns);
    return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ void dsa_abort(DsaCtrl* c, int* status) {
    atomicExch(&c->abort, 1);
    atomicExch(&status[0], 1);
}

template <int H, bool WRITE, bool COLLECT>   // heads: 16, 32 or 64; the epilogue loops unroll fully
__global__ void __launch_bounds__(D_THREADS, 1)
dsa_scores_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmQ,
                  const DsaArgs a) {
    constexpr int TG2 = NQ / H / 2;   // tokens per epilogue warp and tile
    static_assert(TG2 <= 8, "per-warp token slots");
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    unsigned char* Qs = smem;                                  // 2 x 32 KB
    unsigned char* Ks = Qs + 2 * Q_TILE_BYTES;                 // D_STAGES x 16 KB
    DsaCtrl* ctl = reinterpret_cast<DsaCtrl*>(Ks + D_STAGES * K_TILE_BYTES);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x;
    volatile int* abort = &ctl->abort;

    if (threadIdx.x == 0) {
        for (int s = 0; s < D_STAGES; ++s) {
            mbar_init(&ctl->a_full[s], 1);
            mbar_init(&ctl->a_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&ctl->q_full[b], 1);
            mbar_init(&ctl->q_empty[b], 1);
            mbar_init(&ctl->acc_full[b], 1);
            mbar_init(&ctl->acc_empty[b], 8);   // two warpgroups per accumulator
        }
        ctl->abort = 0;
        fence_barrier_init();
    }
    if (warp == 2) {
        tmem_alloc(&ctl->tmem_base, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ctl->tmem_base;

    if (warp == 0) {
        // -------------------------------------------------------- producer
        if (lane == 0) {
            prefetch_tmap(&tmK);
            prefetch_tmap(&tmQ);
        }
        int i = 0, k = 0, issued = 0, qk = 0;   // k counts the groups that load queries
        bool ok = true;
        for (int g = blockIdx.x; ok && g < a.n_groups; g += G) {
            const int nt = group_tiles(a, g);
            if (nt == 0) continue;
            const int qb = k & 1;
            if (!wait_all(&ctl->q_empty[qb], ((k >> 1) & 1) ^ 1, abort, a.wait_ns)) { ok = false; break; }
            if (lane == 0) {
                mbar_expect_tx(&ctl->q_full[qb], Q_TILE_BYTES);
                tma_load_2d(Qs + qb * Q_TILE_BYTES, &tmQ, &ctl->q_full[qb], 0, g * NQ);
            }
            qk = ++k;
            for (int t = 0; t < nt; ++t, ++i) {
                const int s = i % D_STAGES;
                if (!wait_all(&ctl->a_empty[s], ((i / D_STAGES) & 1) ^ 1, abort, a.wait_ns)) { ok = false; break; }
                if (lane == 0) {
                    mbar_expect_tx(&ctl->a_full[s], K_TILE_BYTES);
                    tma_load_2d(Ks + s * K_TILE_BYTES, &tmK, &ctl->a_full[s], 0, t * KT);
                }
                __syncwarp();
                issued = i + 1;
            }
        }
        if (!ok) {
            if (lane == 0) dsa_abort(ctl, a.status);
            // drain: the copies in flight must land before the CTA exits
            for (int j = max(0, issued - D_STAGES); j < issued; ++j)
                mbar_wait_drain(&ctl->a_full[j % D_STAGES], (j / D_STAGES) & 1);
            for (int j = max(0, qk - 2); j < qk; ++j)
                mbar_wait_drain(&ctl->q_full[j & 1], (j >> 1) & 1);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------- MMA
        const uint32_t idesc = idesc_f8(KT, NQ, 0, 0);
        int i = 0, k = 0, last = -1;   // k counts the groups that use queries
        bool ok = true;
        for (int g = blockIdx.x; ok && g < a.n_groups; g += G) {
            const int nt = group_tiles(a, g);
            if (nt == 0) continue;
            const int qb = k & 1;
            if (!wait_all(&ctl->q_full[qb], (k >> 1) & 1, abort, a.wait_ns)) { ok = false; break; }
            ++k;
            for (int t = 0; t < nt; ++t, ++i) {
                const int s = i % D_STAGES, b = i & 1;
                if (!wait_all(&ctl->a_full[s], (i / D_STAGES) & 1, abort, a.wait_ns) ||
                    !wait_all(&ctl->acc_empty[b], ((i >> 1) & 1) ^ 1, abort, a.wait_ns)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t ka = smem_u32(Ks + s * K_TILE_BYTES);
                    const uint32_t qa = smem_u32(Qs + qb * Q_TILE_BYTES);
                    const uint32_t d = tmem + (uint32_t)(b * NQ);
#pragma unroll
                    for (int ks = 0; ks < DK / 32; ++ks)
                        mma_f8(d, desc_k_sw128(ka + ks * 32), desc_k_sw128(qa + ks * 32), idesc,
                               ks != 0);
                    mma_commit(&ctl->acc_full[b]);
                    mma_commit(&ctl->a_empty[s]);
                    if (t == nt - 1) mma_commit(&ctl->q_empty[qb]);
                }
                __syncwarp();
                last = i;
            }
        }
        if (!ok) {
            if (lane == 0) dsa_abort(ctl, a.status);
            if (last >= 0)   // the MMAs issued must finish before TMEM is freed
                mbar_wait_drain(&ctl->acc_full[last & 1], (last >> 1) & 1);
        }
    } else if (warp >= 4) {
        // -------------------------------------------------------- epilogue
        const int ew = warp - 4;               // 0..15
        const int wg = ew >> 2;                // 0..3
        const int par = wg & 1;                // tiles with i % 2 == par
        const int half = wg >> 1;              // tokens [half * tg / 2, (half + 1) * tg / 2)
        const int sub = warp & 3;              // TMEM lanes 32*sub .. +31
        const int r = sub * 32 + lane;         // key within the tile
        float* wsm = ctl->wsm[ew];   // per warp: no cross-warp barrier on any path
        float* esm = ctl->esm[ew];
        float* tsm = ctl->tsm[ew];
        int i = 0, g_loaded = -1;
        bool ok = true;
        for (int g = blockIdx.x; ok && g < a.n_groups; g += G) {
            const int nt = group_tiles(a, g);
            for (int t = 0; t < nt; ++t, ++i) {
                if ((i & 1) != par) continue;
                if (g_loaded != g) {
                    // this warp's tokens' weights for group g
                    __syncwarp();
                    const int n = TG2 * H;
                    const int64_t base = ((int64_t)g * (2 * TG2) + half * TG2) * H;
                    for (int e = lane; e < n; e += 32)
                        wsm[e] = base + e < a.T * H ? a.w[base + e] : 0.0f;
                    if (COLLECT && lane < TG2) {
                        const int64_t tok = (int64_t)g * (2 * TG2) + half * TG2 + lane;
                        esm[lane] = tok < a.T ? a.tok_e[tok] : 0.0f;
                        tsm[lane] = tok < a.T ? a.tok_tau[tok] : INFINITY;
                    }
                    __syncwarp();
                    g_loaded = g;
                }
                const int b = i & 1;
                if (!wait_all(&ctl->acc_full[b], (i >> 1) & 1, abort, a.wait_ns)) { ok = false; break; }
                tc_fence_after();
                const int64_t j = (int64_t)t * KT + r;
                const uint32_t tb = tmem + (uint32_t)(b * NQ) + ((uint32_t)(sub * 32) << 16);
                const float nj = COLLECT && j < a.L ? __ldg(a.norms + j) : 0.0f;
#pragma unroll
                for (int tl = 0; tl < TG2; ++tl) {
                    const int tcol = (half * TG2 + tl) * H;
                    const int64_t tok = (int64_t)g * (2 * TG2) + half * TG2 + tl;
                    const float* wr = wsm + tl * H;
                    // even / odd heads in the two halves of a packed fp32 pair
                    // (fma.rn.f32x2: one instruction per two heads); one TMEM load
                    // of up to 32 heads per wait
                    uint64_t s2 = pack_f32x2(0.0f, 0.0f);
#pragma unroll
                    for (int c0 = 0; c0 < H; c0 += 32) {
                        constexpr int CW = H < 32 ? H : 32;
                        uint32_t v[CW];
                        if constexpr (CW == 32) tmem_ld_x32(tb + (uint32_t)(tcol + c0), v);
                        else tmem_ld_x16(tb + (uint32_t)(tcol + c0), v);
                        tmem_wait_ld();
#pragma unroll
                        for (int h4 = 0; h4 < CW; h4 += 4) {
                            const float4 w4 = *reinterpret_cast<const float4*>(wr + c0 + h4);
                            s2 = fma_f32x2(pack_f32x2(w4.x, w4.y),
                                           pack_f32x2(fmaxf(__uint_as_float(v[h4 + 0]), 0.0f),
                                                      fmaxf(__uint_as_float(v[h4 + 1]), 0.0f)),
                                           s2);
                            s2 = fma_f32x2(pack_f32x2(w4.z, w4.w),
                                           pack_f32x2(fmaxf(__uint_as_float(v[h4 + 2]), 0.0f),
                                                      fmaxf(__uint_as_float(v[h4 + 3]), 0.0f)),
                                           s2);
                        }
                    }
                    float s_lo, s_hi;
                    unpack_f32x2(s2, s_lo, s_hi);
                    const float s = s_lo + s_hi;
                    const bool vis = tok < a.T && j < a.L && j <= a.pos0 + tok;
                    if (WRITE && tok < a.T && j < a.L) a.scores[tok * a.L + j] = vis ? s : -INFINITY;
                    if (COLLECT) {
                        // the key's upper bound s~ + E_t ||k_j|| (rounded up) against
                        // the token's threshold; one bitmap word per warp and token
                        const unsigned bh = __ballot_sync(
                            0xffffffffu, vis && __fadd_ru(s, __fmul_ru(esm[tl], nj)) >= tsm[tl]);
                        const int64_t w0 = ((int64_t)t * KT + sub * 32) >> 5;   // this warp's 32 keys
                        if (lane == 0 && tok < a.T && w0 < a.W) a.bitmap[tok * a.W + w0] = bh;
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&ctl->acc_empty[b]);
            }
        }
        if (!ok && lane == 0) dsa_abort(ctl, a.status);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 2) tmem_dealloc(tmem, 512);
}

// Positions of each token's score row that no tile of its group covers.
__global__ void dsa_tail_kernel(float* __restrict__ scores, int64_t T, int64_t L, int64_t pos0,
                                int tg, int key_tiles) {
    const int64_t t = blockIdx.y;
    const int g = (int)(t / tg);
    const int64_t t_last = min(T, (int64_t)(g + 1) * tg) - 1;
    const int64_t vis = pos0 + t_last + 1;
    const int64_t covered = vis <= 0 ? 0 : min(L, min((int64_t)key_tiles, (vis + KT - 1) / KT) * KT);
    for (int64_t j = covered + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < L;
         j += (int64_t)gridDim.x * blockDim.x)
        scores[t * L + j] = -INFINITY;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn_dsa() {
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

// Row-major [rows][128] bytes as a 2-D uint8 tensor map, {128, box_rows}
// boxes, 128-byte swizzle (one swizzle row per fp8 row).
hmm_status_t make_tmap_u8(CUtensorMap* m, const void* base, int64_t rows, int box_rows) {
    auto fn = encode_fn_dsa();
    if (!fn) return set_error(HMM_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[2] = {(cuuint64_t)DK, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)DK};
    cuuint32_t box[2] = {(cuuint32_t)DK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims,
                          strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(HMM_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return HMM_OK;
}

// Selections of keys nobody can see (score -inf: fewer visible keys than k)
// become -1, as the reference returns only min(k, visible) indices.
__global__ void dsa_pad_kernel(int32_t* __restrict__ idx, float* __restrict__ sc, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n && sc[i] == -INFINITY) idx[i] = -1;
}

__global__ void dsa_fill_kernel(float* __restrict__ sc, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) sc[i] = -INFINITY;
}

size_t up256(size_t v) { return (v + 255) & ~size_t(255); }

}  // namespace
}  // namespace hmm

using namespace hmm;

namespace {

// One scoring pass over keys[0, L) (the call's keys or the sample): TMA maps,
// then the kernel for the head count and the pass's outputs.
template <bool WRITE, bool COLLECT>
hmm_status_t launch_scores(const uint8_t* q, const uint8_t* keys, int64_t T, int64_t H, int64_t L,
                           DsaArgs a, bool profiled, cudaStream_t st) {
    CUtensorMap tmK, tmQ;
    hmm_status_t s = make_tmap_u8(&tmK, keys, L, KT);
    if (s != HMM_OK) return s;
    s = make_tmap_u8(&tmQ, q, T * H, NQ);
    if (s != HMM_OK) return s;
    a.T = T;
    a.L = L;
    a.H = (int)H;
    a.tg = NQ / (int)H;
    a.n_groups = (int)((T + a.tg - 1) / a.tg);
    a.key_tiles = (int)((L + KT - 1) / KT);
    a.wait_ns = wait_limit_ns();
    auto kern = H == 64 ? dsa_scores_kernel<64, WRITE, COLLECT>
              : H == 32 ? dsa_scores_kernel<32, WRITE, COLLECT>
                        : dsa_scores_kernel<16, WRITE, COLLECT>;
    HMM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)D_SMEM));
    const int grid = std::max(1, std::min(device_sm_count(), a.n_groups));
    // the profile marks time the pass over every key, not the sample's
    ProfileMark pm{};
    if (profiled) pm = profile_begin(st);
    kern<<<grid, D_THREADS, D_SMEM, st>>>(tmK, tmQ, a);
    s = check_launch("dsa_scores_kernel");
    if (profiled) profile_end(pm, st);
    return s;
}

}  // namespace

extern "C" size_t hmm_dsa_indexer_fp8_workspace_size(int64_t T, int64_t H, int64_t L,
                                                     int64_t topk) {
    if (T < 0 || H < 1 || L < 0 || topk < 1) return 0;
    return up256(dsa_exact_ws_bytes(T, L)) + up256(sizeof(float) * (size_t)T * (size_t)topk);
}

extern "C" hmm_status_t hmm_dsa_indexer_fp8(const uint8_t* q, const uint8_t* keys,
                                            const float* w, int64_t T, int64_t H, int64_t L,
                                            int64_t D, int64_t pos0, int64_t topk,
                                            int32_t* out_idx, float* out_scores,
                                            float* all_scores, void* workspace,
                                            size_t workspace_bytes, void* stream) {
    HMM_REQUIRE(D == DK, "head dim must be %d, got %lld", DK, (long long)D);
    HMM_REQUIRE(H == 16 || H == 32 || H == 64, "heads must be 16, 32 or 64, got %lld",
                (long long)H);
    HMM_REQUIRE(T >= 0 && T * H < (int64_t(1) << 31), "T out of range");
    HMM_REQUIRE(L >= 0 && L < (int64_t(1) << 31), "L out of range");
    HMM_REQUIRE(topk >= 1 && topk <= 4096, "topk must be in [1, 4096]");
    HMM_REQUIRE(pos0 >= -1, "pos0 must be >= -1");
    if (T == 0) return HMM_OK;
    HMM_REQUIRE(q && w && out_idx && (L == 0 || keys), "null pointer");
    HMM_REQUIRE((reinterpret_cast<uintptr_t>(q) % 16) == 0 &&
                    (reinterpret_cast<uintptr_t>(keys) % 16) == 0 &&
                    (reinterpret_cast<uintptr_t>(w) % 16) == 0,
                "q, keys and w must be 16-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    const size_t ex_bytes = up256(dsa_exact_ws_bytes(T, L));
    const size_t sel_bytes = up256(sizeof(float) * (size_t)T * (size_t)topk);
    const size_t need = ex_bytes + sel_bytes;
    if (!ws || workspace_bytes < need)
        return set_error(HMM_ERR_OOM, "workspace too small: %zu < %zu", workspace_bytes, need);
    void* ex_ws = ws;
    float* sel_sc = out_scores ? out_scores : reinterpret_cast<float*>(ws + ex_bytes);
    const int64_t n_sel = T * topk;

    if (L == 0) {   // no key is visible to any token
        HMM_CUDA_TRY(cudaMemsetAsync(out_idx, 0xff, sizeof(int32_t) * (size_t)n_sel, st));
        dsa_fill_kernel<<<(unsigned)((n_sel + 255) / 256), 256, 0, st>>>(sel_sc, n_sel);
        return check_launch("dsa_fill_kernel");
    }
    DsaExactBufs b;
    hmm_status_t s = dsa_exact_prepare(keys, T, L, topk, ex_ws, st, &b);
    if (s != HMM_OK) return s;
    DsaArgs a{};
    a.w = w;
    a.status = b.status;   // [0]: a bounded wait gave up
    a.norms = b.norms;
    a.tok_e = b.tok_e;
    a.tok_tau = b.tok_tau;
    a.bitmap = b.bitmap;
    a.W = b.W;
    if (b.S > 0) {
        // 1. the sampled keys' scores (every sampled key visible to every token)
        DsaArgs sa = a;
        sa.scores = b.sscores;
        sa.pos0 = b.S;
        s = launch_scores<true, false>(q, b.skeys, T, H, b.S, sa, false, st);
        if (s != HMM_OK) return s;
    }
    // 2. E_t and the thresholds
    s = dsa_exact_thresholds(q, w, T, H, L, pos0, topk, b, st);
    if (s != HMM_OK) return s;
    // 3. the scoring pass over every key: the bitmap of each token's keys that
    //    can reach its k-th (and the scores themselves when asked for); when no
    //    token sees more than the candidate capacity, every visible key is a
    //    candidate and only the asked-for scores need the pass
    a.pos0 = pos0;
    if (all_scores) {
        a.scores = all_scores;
        s = b.S > 0 ? launch_scores<true, true>(q, keys, T, H, L, a, true, st)
                    : launch_scores<true, false>(q, keys, T, H, L, a, true, st);
        if (s != HMM_OK) return s;
        const int tg = NQ / (int)H;
        const int key_tiles = (int)((L + KT - 1) / KT);
        dsa_tail_kernel<<<dim3(16, (unsigned)T), 256, 0, st>>>(all_scores, T, L, pos0, tg,
                                                               key_tiles);
        s = check_launch("dsa_tail_kernel");
        if (s != HMM_OK) return s;
    } else if (b.S > 0) {
        s = launch_scores<false, true>(q, keys, T, H, L, a, true, st);
        if (s != HMM_OK) return s;
    }
    // 4. exact selection (reads the status words, so this waits for the
    //    stream), then -1 for the slots of keys nobody sees
    s = dsa_exact_select(q, keys, w, T, H, L, pos0, topk, b, out_idx, sel_sc, ex_ws, st);
    if (s != HMM_OK) return s;
    dsa_pad_kernel<<<(unsigned)((n_sel + 255) / 256), 256, 0, st>>>(out_idx, sel_sc, n_sel);
    return check_launch("dsa_pad_kernel");
}
