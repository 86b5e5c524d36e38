// dsa_exact.cu — exact selection for the FP8 DSA lightning indexer.
//
// Reference: indexer_top_ref (kernels/dsa_indexer/indexer_tb.cpp:27-56): per
// key j, total = sum over heads h (in order) of w[h] * (float)ReLU(q_h . k_j)
// with the dot exact, then the TOP_K best keys, best first.  With e4m3 inputs
// the exact dot is an integer multiple of 2^-18, so that arithmetic is:
//   x_h = fl32(ReLU(D_h) * 2^-18),  total = fl32(total + fl32(w_h * x_h)).
//
// The tensor-core pass (dsa.cu) gives approximate scores s~ with
//   |s~ - s| <= C_TOL * sum_h |w_h| sum_d |q_hd| |k_jd|
//            <= C_TOL * ||u_t||_2 * ||k_j||_2 = E_t ||k_j||,  u_t[d] = sum_h |w_h| |q_hd|
// where C_TOL covers the tensor core's fp32 accumulation (assumed to lose at
// most 2^-10 of sum_d |q_hd||k_jd|, 128x the worst case of sequential fp32;
// measured below 2e-5 of that) and the fp32 roundings of both head sums.
// With hi_j = s~_j + E_t ||k_j|| (rounded up) >= s_j and any threshold tau:
// the keys with hi < tau have exact scores s < tau, so if the m-th best exact
// score (m = min(k, visible)) among the keys with hi >= tau is >= tau, the
// exact top-k (ties included) lies among them.  Per call:
//   1. dsa_key_prep_kernel: ||k_j|| per key (rounded up) and a NaN check;
//      dsa_sample_gather_kernel: S keys at j_i = floor(i L / S);
//      the scoring pass (dsa.cu) scores the sample: [T][S] approximate scores
//   2. dsa_threshold_kernel: E_t and tau, a floor of the r1-th largest
//      lo = s~ - E_t ||k_j|| of the token's visible sample keys, r1 chosen so
//      that at least m keys of the row have s >= lo >= tau except with
//      negligible probability
//   3. the scoring pass over every key (dsa.cu) marks the keys with hi >= tau
//      in a bitmap; no score is stored
//   4. dsa_cand_kernel: the marked keys become the token's candidates
//   5. dsa_rescore_kernel: the candidates' exact scores on the tensor cores
//      (tcgen05.mma kind::i8, exact int32 accumulation): every e4m3 value
//      times 2^9 is an integer v, |v| <= 229,376, split into three signed
//      6-bit limbs v = l0 + 64 l1 + 4096 l2; the nine limb products are summed
//      in five TMEM accumulators by the scale 64^(i+i') they carry and joined
//      exactly; the head sum is then the reference's.
//   6. dsa_select_kernel: the exact top-k of the candidates, best first,
//      ties to the lowest key, after checking that the m-th of them is >= tau.
// A token whose candidates do not fit or whose check fails (possible only
// for near-identical keys, whose scores crowd the k-th) is flagged; the host
// recomputes its whole row exactly on CUDA cores (dsa_exact_rows_kernel) and
// selects from that.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "heteromm_cuda.h"
#include "dsa_exact.cuh"
#include "hmm_common.cuh"
#include "sm100_ptx.cuh"

namespace hmm {
using namespace sm100;

namespace {

constexpr int DK = 128;                    // head dim: bytes per fp8 row and per limb row
constexpr int NLIMB = 3;
constexpr int CAP_C = 8192;                // candidates per token
constexpr int BAND_THREADS = 512;          // threshold and candidate kernels
constexpr int BAND_SAMPLE = 4096;          // sampled keys per call
constexpr int FB_ROWS = 32;                // flagged tokens per exact-row fallback pass
constexpr int SEL_THREADS = 512;
constexpr int KMAX = 4096;
// C_TOL: 2^-10 for the tensor-core accumulation plus 2^-16, which covers the
// fp32 roundings of x_h and of both head sums (about 100 * 2^-24).
constexpr double C_TOL = 1.0 / 1024.0 + 1.0 / 65536.0;

// Status words (int) at the start of the selection workspace, then up to T
// flagged token ids.
enum { ST_TIMEOUT = 0, ST_NAN = 1, ST_NFLAG = 2, ST_FLAGS = 4 };

// e4m3 (OCP FP8: bias 7, no infinities, S.1111.111 = NaN) times 2^9 as an
// integer; the NaN encodings give 0 and are reported by the callers.
__device__ __forceinline__ int e4m3_scaled(uint32_t b) {
    const int e = (int)((b >> 3) & 15u), m = (int)(b & 7u);
    if (e == 15 && m == 7) return 0;
    const int mag = e == 0 ? m : (8 + m) << (e - 1);
    return (b & 0x80u) ? -mag : mag;
}
__device__ __forceinline__ bool e4m3_is_nan(uint32_t b) { return (b & 0x7fu) == 0x7fu; }

// Limb i of v (signed 6-bit pieces of |v|, carrying v's sign), as a byte.
__device__ __forceinline__ uint32_t limb_byte(int v, int i) {
    const int a = v < 0 ? -v : v;
    int l = (a >> (6 * i)) & (i == 2 ? 0xff : 63);
    if (v < 0) l = -l;
    return (uint32_t)(l & 0xff);
}

// Limb bytes of one e4m3 byte packed as (l0 | l1 << 8 | l2 << 16).
__device__ __forceinline__ uint32_t limb_entry(uint32_t b) {
    const int v = e4m3_scaled(b);
    return limb_byte(v, 0) | (limb_byte(v, 1) << 8) | (limb_byte(v, 2) << 16);
}

// Limbs of 16 e4m3 bytes through the table: out[i] = 16 bytes of limb i.
__device__ __forceinline__ void limbs16_lut(const uint4 raw, const uint32_t* lut, uint4 out[3]) {
    const uint32_t wv[4] = {raw.x, raw.y, raw.z, raw.w};
    uint32_t o[3][4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const uint32_t x = wv[q];
        const uint32_t e0 = lut[x & 255u], e1 = lut[(x >> 8) & 255u];
        const uint32_t e2 = lut[(x >> 16) & 255u], e3 = lut[x >> 24];
#pragma unroll
        for (int i = 0; i < NLIMB; ++i) {
            const uint32_t sel = 0x0040u + (uint32_t)i * 0x0011u;   // bytes i of (e_a, e_b)
            o[i][q] = __byte_perm(__byte_perm(e0, e1, sel), __byte_perm(e2, e3, sel), 0x5410u);
        }
    }
#pragma unroll
    for (int i = 0; i < NLIMB; ++i) out[i] = make_uint4(o[i][0], o[i][1], o[i][2], o[i][3]);
}

// ---------------------------------------------------------------------------
// K0: ||k_j||_2 of every key rounded up; flags NaN encodings.  One warp per
// key (4 bytes per lane), warps striding over keys.
__global__ void dsa_key_prep_kernel(const uint8_t* __restrict__ keys, int64_t L,
                                    float* __restrict__ norms, int* __restrict__ status) {
    const int lane = threadIdx.x & 31;
    const int64_t w0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
    bool nan = false;
    for (int64_t j = w0; j < L; j += nw) {
        const uint32_t w = reinterpret_cast<const uint32_t*>(keys + j * DK)[lane];
        long long sq = 0;   // sum of v^2 (v = value * 2^9): exact in 64 bits
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const uint32_t byte = (w >> (8 * b)) & 0xffu;
            nan |= e4m3_is_nan(byte);
            const long long v = e4m3_scaled(byte);
            sq += v * v;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
        if (lane == 0) norms[j] = __double2float_ru(__dsqrt_ru((double)sq) * (1.0 / 512.0));
    }
    if (__any_sync(0xffffffffu, nan) && lane == 0) atomicOr(&status[ST_NAN], 1);
}

// K0c: the sampled keys, j_i = floor(i L / S), as a contiguous [S][128] array
// for the scoring pass.  One thread per 16 bytes.
__global__ void dsa_sample_gather_kernel(const uint8_t* __restrict__ keys, int64_t L, int S,
                                         uint8_t* __restrict__ skeys) {
    const int64_t n16 = (int64_t)S * (DK / 16);
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n16;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = e >> 3, c = e & 7;
        const int64_t j = i * L / S;
        reinterpret_cast<uint4*>(skeys)[e] = __ldg(reinterpret_cast<const uint4*>(keys + j * DK) + c);
    }
}

// K0b: the keys' limb rows [L][3][128] (int8), written just before the
// rescoring so that they are still in L2 when its gather reads them.  One
// thread per 16 key bytes.
__global__ void dsa_key_limbs_kernel(const uint8_t* __restrict__ keys, int64_t L,
                                     uint8_t* __restrict__ limbs) {
    __shared__ uint32_t lut[256];
    for (int b = threadIdx.x; b < 256; b += blockDim.x) lut[b] = limb_entry((uint32_t)b);
    __syncthreads();
    const int64_t n16 = L * (DK / 16);
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n16;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = e >> 3;
        const int c = (int)(e & 7);
        uint4 l[3];
        limbs16_lut(__ldg(reinterpret_cast<const uint4*>(keys) + e), lut, l);
#pragma unroll
        for (int i = 0; i < NLIMB; ++i)
            *reinterpret_cast<uint4*>(limbs + j * (NLIMB * DK) + i * DK + c * 16) = l[i];
    }
}

// ---------------------------------------------------------------------------
// K2: the candidate band of each token (one block per token).

// Histogram add of `bucket` (when `act`) by a whole warp, one shared atomic
// per distinct bucket (scores of one token crowd into few buckets).  All 32
// lanes must call it.
__device__ __forceinline__ void warp_hist_add(unsigned* hist, bool act, unsigned bucket) {
    const int lane = threadIdx.x & 31;
    const unsigned b = act ? bucket : 256u + (unsigned)lane;   // inactive lanes match nobody
    const unsigned peers = __match_any_sync(0xffffffffu, b);
    if (act && lane == __ffs(peers) - 1) atomicAdd(&hist[b], (unsigned)__popc(peers));
}

// Slot of this lane in a list grown by counter (when `take`), one shared
// atomic per warp; -1 if the lane takes none.  All 32 lanes must call it.
__device__ __forceinline__ int warp_append(bool take, int* counter) {
    const int lane = threadIdx.x & 31;
    const unsigned bal = __ballot_sync(0xffffffffu, take);
    if (bal == 0u) return -1;
    int base = 0;
    if (lane == __ffs(bal) - 1) base = atomicAdd(counter, __popc(bal));
    base = __shfl_sync(0xffffffffu, base, __ffs(bal) - 1);
    return take ? base + __popc(bal & ((1u << lane) - 1u)) : -1;
}

template <int NT>
__device__ __forceinline__ unsigned band_scan_incl(unsigned v, unsigned* warp_tot) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
    }
    if (lane == 31) warp_tot[w] = v;
    __syncthreads();
    if (w == 0) {
        unsigned t = lane < NT / 32 ? warp_tot[lane] : 0u;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned u = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= o) t += u;
        }
        if (lane < NT / 32) warp_tot[lane] = t;
    }
    __syncthreads();
    const unsigned r = v + (w > 0 ? warp_tot[w - 1] : 0u);
    __syncthreads();
    return r;
}

// Threshold T such that exactly min(k, M) of the distinct nonzero composites
// key_at(0 .. M-1) are >= T (0 if k >= M); NT threads; sm >= 256 + NT/32 + 3
// words.
template <int NT, class KeyAt>
__device__ __forceinline__ uint64_t band_select_fn(KeyAt key_at, int64_t M, int64_t k,
                                                   unsigned* sm) {
    unsigned* hist = sm;
    unsigned* wt = sm + 256;
    unsigned* res = sm + 256 + NT / 32;
    if (k >= M) return 0ull;
    uint64_t prefix = 0, mask = 0;
    unsigned need = (unsigned)k;
    for (int shift = 56; shift >= 0; shift -= 8) {
        if (threadIdx.x < 256) hist[threadIdx.x] = 0;
        __syncthreads();
        for (int64_t i0 = threadIdx.x & ~31; i0 < M; i0 += NT) {
            const int64_t i = i0 + (threadIdx.x & 31);
            const uint64_t key = i < M ? key_at(i) : 0ull;
            warp_hist_add(hist, i < M && (key & mask) == prefix, (unsigned)(key >> shift) & 255u);
        }
        __syncthreads();
        const unsigned c = threadIdx.x < 256 ? hist[255 - threadIdx.x] : 0u;
        const unsigned incl = band_scan_incl<NT>(c, wt);
        const unsigned excl = incl - c;
        if (threadIdx.x < 256 && excl < need && need <= incl) {
            res[0] = 255 - threadIdx.x; res[1] = excl; res[2] = c;
        }
        __syncthreads();
        const unsigned bucket = res[0], before = res[1], cnt = res[2];
        need -= before;
        prefix |= (uint64_t)bucket << shift;
        mask |= (uint64_t)0xff << shift;
        __syncthreads();
        if (cnt == need) break;
    }
    return prefix;
}

template <int NT>
__device__ __forceinline__ uint64_t band_select(const uint64_t* keys, int64_t M, int64_t k,
                                                unsigned* sm) {
    return band_select_fn<NT>([keys](int64_t i) { return keys[i]; }, M, k, sm);
}

// Largest P = (24-bit prefix << 8) such that at least `need` (>= 1, <= M) of
// the 32-bit keys key_at(0 .. M-1) are >= P: a floor of the need-th largest
// key, three 8-bit histogram passes.  NT threads; sm >= 256 + NT/32 + 3.
template <int NT, class KeyAt>
__device__ __forceinline__ uint32_t key_floor(KeyAt key_at, int64_t M, int64_t need_in,
                                              unsigned* sm) {
    unsigned* hist = sm;
    unsigned* wt = sm + 256;
    unsigned* res = sm + 256 + NT / 32;
    uint32_t prefix = 0, mask = 0;
    unsigned need = (unsigned)need_in;
    for (int shift = 24; shift >= 8; shift -= 8) {
        if (threadIdx.x < 256) hist[threadIdx.x] = 0;
        __syncthreads();
        for (int64_t i0 = threadIdx.x & ~31; i0 < M; i0 += NT) {
            const int64_t i = i0 + (threadIdx.x & 31);
            const uint32_t key = i < M ? key_at(i) : 0u;
            warp_hist_add(hist, i < M && (key & mask) == prefix, (key >> shift) & 255u);
        }
        __syncthreads();
        const unsigned c = threadIdx.x < 256 ? hist[255 - threadIdx.x] : 0u;
        const unsigned incl = band_scan_incl<NT>(c, wt);
        const unsigned excl = incl - c;
        if (threadIdx.x < 256 && excl < need && need <= incl) {
            res[0] = 255 - threadIdx.x; res[1] = excl;
        }
        __syncthreads();
        need -= res[1];
        prefix |= res[0] << shift;
        mask |= 0xffu << shift;
        __syncthreads();
    }
    return prefix;
}

struct TokArgs {
    const uint8_t* q;        // [T][H][128] e4m3
    const float* w;          // [T][H]
    const float* norms;      // [L]
    const float* sscores;    // [T][S] approximate scores of the sampled keys
    const uint32_t* bitmap;  // [T][W]
    float* tok_e;            // [T]
    float* tok_tau;          // [T] the threshold as a float (-inf: every visible key)
    int32_t* cand;           // [T][CAP_C] candidate keys
    int* cand_cnt;           // [T]
    int* status;
    int64_t T, L, pos0;
    int H, k, S, W;
};

__device__ __forceinline__ void band_flag(const TokArgs& a, int64_t t) {
    const int pos = atomicAdd(&a.status[ST_NFLAG], 1);
    if (pos < a.T) a.status[ST_FLAGS + pos] = (int)t;
}

// K2: one block per token: E_t = C_TOL * ||u_t||_2 rounded up, and tau.
// Tokens that see at most CAP_C keys take all of them (tau = key 0).  The
// others: the sample holds S_t visible keys; a key of the row reaches the
// k-th with probability p = m / vis, so the sample holds Binomial(S_t, p)
// such keys; tau = a floor of the (mean + 5 sd + 8)-th largest lo among them.
__global__ void __launch_bounds__(BAND_THREADS) dsa_threshold_kernel(const TokArgs a) {
    __shared__ uint32_t samp[BAND_SAMPLE];
    __shared__ unsigned sm[256 + BAND_THREADS / 32 + 4];
    __shared__ float ured[4][DK];
    __shared__ float nred[BAND_THREADS / 32];
    __shared__ int nan_seen, st_cnt;
    __shared__ float e_t;
    const int64_t t = blockIdx.x;
    const int64_t vis = max((int64_t)0, min(a.L, a.pos0 + t + 1));
    const int m = (int)min((int64_t)a.k, vis);
    if (threadIdx.x == 0) { nan_seen = 0; st_cnt = 0; }
    __syncthreads();
    {
        const uint8_t* qt = a.q + t * (int64_t)a.H * DK;
        const float* wt = a.w + t * a.H;
        const int d = threadIdx.x & (DK - 1), hq = threadIdx.x >> 7;   // 4 head quarters
        float u = 0.0f;
        bool nan = false;
#pragma unroll 4
        for (int h = hq; h < a.H; h += BAND_THREADS / DK) {
            const uint32_t b = qt[h * DK + d];
            nan |= e4m3_is_nan(b);
            const int v = e4m3_scaled(b);
            u = __fmaf_ru(fabsf(wt[h]), (float)(v < 0 ? -v : v) * (1.0f / 512.0f), u);
        }
        ured[hq][d] = u;
        if (nan) atomicOr(&nan_seen, 1);
        __syncthreads();
        float sq = 0.0f;
        if (threadIdx.x < DK) {
            const float ud = __fadd_ru(__fadd_ru(ured[0][d], ured[1][d]),
                                       __fadd_ru(ured[2][d], ured[3][d]));
            sq = __fmul_ru(ud, ud);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sq = __fadd_ru(sq, __shfl_xor_sync(0xffffffffu, sq, o));
        if ((threadIdx.x & 31) == 0) nred[threadIdx.x >> 5] = sq;
        __syncthreads();
        if (threadIdx.x == 0) {
            float s2 = 0.0f;
            for (int i = 0; i < BAND_THREADS / 32; ++i) s2 = __fadd_ru(s2, nred[i]);
            e_t = __fmul_ru(__fsqrt_ru(s2), (float)C_TOL * (1.0f + 1.0f / 4096.0f));
            if (nan_seen) atomicOr(&a.status[ST_NAN], 1);
            a.tok_e[t] = e_t;
        }
        __syncthreads();
    }
    if (vis <= CAP_C || a.S == 0) {   // every visible key is a candidate
        if (threadIdx.x == 0) a.tok_tau[t] = -INFINITY;
        return;
    }
    const float E = e_t;
    // the visible sample keys: i with floor(i L / S) < vis, a prefix of the sample
    const float* srow = a.sscores + t * a.S;
    for (int i = threadIdx.x; i < a.S; i += BAND_THREADS) {
        const int64_t j = (int64_t)i * a.L / a.S;
        if (j < vis) {
            atomicAdd(&st_cnt, 1);
            samp[i] = f32_key(__fsub_rd(srow[i], __fmul_ru(E, a.norms[j])));
        }
    }
    __syncthreads();
    const int St = st_cnt;
    const double p_k = (double)m / (double)vis;
    const double mean_k = St * p_k;
    const int64_t r1 = (int64_t)ceil(mean_k + 5.0 * sqrt(mean_k * (1.0 - p_k)) + 8.0);
    if (r1 > St) {   // too few sample keys to place tau: take all (the row is then flagged)
        if (threadIdx.x == 0) a.tok_tau[t] = -INFINITY;
        return;
    }
    const uint32_t* sp = samp;
    const uint32_t tk = key_floor<BAND_THREADS>([sp](int64_t i) { return sp[i]; }, St, r1, sm);
    // the key floor as a float (keys at or below that of -inf mean no threshold)
    if (threadIdx.x == 0) a.tok_tau[t] = tk <= 0x007fffffu ? -INFINITY : key_to_f32(tk);
}

// K4: one block per token: the keys marked in the bitmap become its
// candidates (all visible keys when the token sees at most CAP_C); if they do
// not fit, the token is flagged for the exact-row path.
__global__ void __launch_bounds__(BAND_THREADS) dsa_cand_kernel(const TokArgs a) {
    __shared__ int out_n;
    const int64_t t = blockIdx.x;
    const int64_t vis = max((int64_t)0, min(a.L, a.pos0 + t + 1));
    int32_t* cand = a.cand + t * CAP_C;
    if (vis <= CAP_C) {
        for (int64_t j = threadIdx.x; j < vis; j += BAND_THREADS) cand[j] = (int32_t)j;
        if (threadIdx.x == 0) a.cand_cnt[t] = (int)vis;
        return;
    }
    if (threadIdx.x == 0) out_n = 0;
    __syncthreads();
    const uint32_t* row = a.bitmap + t * a.W;
    const int nw = (int)((vis + 31) >> 5);
    const int lane = threadIdx.x & 31;
    for (int w0 = threadIdx.x & ~31; w0 < nw; w0 += BAND_THREADS) {
        const int wi = w0 + lane;
        uint32_t bits = wi < nw ? row[wi] : 0u;
        if (wi == nw - 1 && (vis & 31)) bits &= (1u << (vis & 31)) - 1u;   // keys past vis
        const int c = __popc(bits);
        // one shared atomic per warp for the warp's candidates, in lane order
        int incl = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int u = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += u;
        }
        const int tot = __shfl_sync(0xffffffffu, incl, 31);
        int base = 0;
        if (lane == 31 && tot) base = atomicAdd(&out_n, tot);
        base = __shfl_sync(0xffffffffu, base, 31);
        int pos = base + incl - c;
        while (bits) {
            const int b = __ffs(bits) - 1;
            bits &= bits - 1;
            if (pos < CAP_C) cand[pos] = wi * 32 + b;
            ++pos;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        if (out_n > CAP_C) {
            band_flag(a, t);
            a.cand_cnt[t] = 0;
        } else {
            a.cand_cnt[t] = out_n;
        }
    }
}

// ---------------------------------------------------------------------------
// K3: exact scores of the candidates on the tensor cores.

constexpr int R_M = 128;                         // candidates per tile (MMA M)
constexpr int R_STAGES = 3;
constexpr int R_A_LIMB = R_M * DK;               // 16 KB: one limb of a tile
constexpr int R_A_STAGE = NLIMB * R_A_LIMB;      // 48 KB
constexpr int R_PROD_WARPS = 4;
constexpr int R_THREADS = 32 * 14;               // producers 0-3, MMA 4, TMEM 5, epilogue 6-13
constexpr int R_GROUPS = 5;                      // limb scales 64^0 .. 64^4
constexpr int R_SLOTS = 8;                       // TMEM group slots of H columns (a ring)

template <int H>
struct RescoreSmem {
    static constexpr int Q_LIMB = H * DK;            // one query limb (H rows of 128 B)
    static constexpr int Q_BUF = NLIMB * Q_LIMB;
    static constexpr size_t A_OFF = 0;
    static constexpr size_t Q_OFF = A_OFF + (size_t)R_STAGES * R_A_STAGE;
    static constexpr size_t W_OFF = Q_OFF + 2 * (size_t)Q_BUF;
    static constexpr size_t LUT_OFF = W_OFF + 2 * H * sizeof(float);   // 256 limb entries
    static constexpr size_t CTRL_OFF = LUT_OFF + 256 * sizeof(uint32_t);
    static constexpr size_t BYTES = CTRL_OFF + 1536 + 1024;   // + barriers, + alignment slack
};

struct RescoreCtrl {
    uint64_t a_full[R_STAGES], a_empty[R_STAGES];
    uint64_t q_full[2], q_empty[2];
    uint64_t slot_full[R_SLOTS];     // group accumulator written (MMA commit per group)
    uint64_t slot_empty[R_SLOTS];    // group accumulator read by both epilogue warpgroups
    uint64_t hand_full[2], hand_empty[2];   // partial head sums, first -> second warpgroup
    float hand[2][R_M];
    uint64_t drain;                  // MMA warp: every MMA issued has completed (abort path)
    uint32_t tmem_base;
    int abort;
};

struct RescoreArgs {
    const uint8_t* q;          // [T][H][128] e4m3
    const float* w;            // [T][H]
    const uint8_t* klimbs;     // [L][3][128] key limbs
    const int32_t* cand;       // [T][CAP_C]
    const int* cand_cnt;       // [T]
    float* exact;              // [T][CAP_C] exact scores of the candidates
    int* status;
    int64_t T;
    uint64_t wait_ns;
};

__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
    // s32 accumulator (2 << 4), signed 8-bit A and B (1 << 7, 1 << 10), K-major
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// fl32(v * 2^-18) for v = A + 4096 B + 2^24 D4, A = D0 + 64 D1, B = D2 + 64
// D3 (the exact dot of the limbs, |v| < 2^46), correctly rounded with
// full-rate int32 and fp32 instructions only:
//   t = A + 4096 (B mod 2048)   (|t| < 2^28)
//   v = Q 2^23 + R,  R = t mod 2^23 in [0, 2^23),  Q = floor(t / 2^23)
//       + floor(B / 2048) + 2 D4  (|Q| < 2^22)
// Q 2^5 and R 2^-18 are exact floats (the 1.5 * 2^23 and 2^23 magic-number
// conversions, scaled by exact fused multiply-adds), so their one rounded sum
// is the rounded v * 2^-18.
__device__ __forceinline__ float exact_dot_f32(int A, int B, int d4) {
    const int t = A + ((B & 2047) << 12);
    const int R = t & ((1 << 23) - 1);
    const int Q = (t >> 23) + (B >> 11) + 2 * d4;
    const float X = __fmaf_rn(__int_as_float(0x4B400000 + Q), 32.0f, -402653184.0f);   // Q 2^5
    const float Y = __fmaf_rn(__int_as_float(0x4B000000 | R), 0x1p-18f, -32.0f);       // R 2^-18
    return __fadd_rn(X, Y);
}

__device__ __forceinline__ bool r_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                       uint64_t limit) {
    const bool ok = mbar_wait_bounded(bar, parity, abort, limit);
    return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ void r_abort(RescoreCtrl* c, int* status) {
    atomicExch(&c->abort, 1);
    atomicExch(&status[ST_TIMEOUT], 1);
}

// 16-byte asynchronous copy global -> shared (L2 only), and its groups.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Byte offset of 16-byte chunk c of row r in a K-major tile of 128-byte rows
// with the 128-byte swizzle (the layout the UMMA descriptor expects).
__device__ __forceinline__ uint32_t sw128(int r, int c) {
    return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4));
}

// One persistent CTA per SM over the tokens.  Roles (16 warps):
//   warps 0-3   producers: per token, its query limbs (B operand, H rows x 3
//               limbs of 128 B) and weights; per tile, the 128 candidates' key
//               limbs gathered by cp.async (A operand, 3 x 16 KB, 128-byte
//               swizzle), one tile's copies in flight while the previous
//               tile's complete
//   warp 4      MMA issuer: per tile, 9 limb pairs x 4 K-steps of
//               tcgen05.mma kind::i8 (M = 128 candidates, N = H heads, K = 32),
//               summed by the scale 64^g they carry into 5 group accumulators
//               of H columns, each taken from a ring of 8 TMEM slots and
//               committed on its own (the issue of one MMA costs about as much
//               as an N = 32 MMA computes, so MMAs are kept at N = H)
//   warp 5      TMEM allocator
//   warps 6-13  epilogue, two warpgroups over the heads of the same tile:
//               thread = candidate; each joins the 5 groups of its heads exactly;
//               the first sums heads 0 .. H/2-1 in order and hands the partial
//               sum (shared memory) to the second, which adds its heads in order
template <int H>
__global__ void __launch_bounds__(R_THREADS, 1) dsa_rescore_kernel(const RescoreArgs a) {
    using S = RescoreSmem<H>;
    extern __shared__ __align__(1024) unsigned char rsm_raw[];
    unsigned char* smem = rsm_raw + ((1024u - (smem_u32(rsm_raw) & 1023u)) & 1023u);
    unsigned char* As = smem + S::A_OFF;
    unsigned char* Qs = smem + S::Q_OFF;
    float* Ws = reinterpret_cast<float*>(smem + S::W_OFF);
    RescoreCtrl* ctl = reinterpret_cast<RescoreCtrl*>(smem + S::CTRL_OFF);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    volatile int* abort = &ctl->abort;
    constexpr uint32_t TMEM_COLS = R_SLOTS * H < 32 ? 32 : R_SLOTS * H;

    if (threadIdx.x == 0) {
        for (int s = 0; s < R_STAGES; ++s) {
            mbar_init(&ctl->a_full[s], 32 * R_PROD_WARPS);
            mbar_init(&ctl->a_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&ctl->q_full[b], 32 * R_PROD_WARPS);
            mbar_init(&ctl->q_empty[b], 1 + 8);   // the MMAs' commit + the 8 epilogue warps
            mbar_init(&ctl->hand_full[b], 4);
            mbar_init(&ctl->hand_empty[b], 4);
        }
        for (int s = 0; s < R_SLOTS; ++s) {
            mbar_init(&ctl->slot_full[s], 1);
            mbar_init(&ctl->slot_empty[s], 8);
        }
        mbar_init(&ctl->drain, 1);
        ctl->abort = 0;
        fence_barrier_init();
    }
    if (warp == 5) {
        tmem_alloc(&ctl->tmem_base, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ctl->tmem_base;
    const int G = gridDim.x;

    if (warp < R_PROD_WARPS) {
        // ---------------------------------------------------------- producers
        // Each thread copies one candidate row per tile: its three limb rows
        // (384 B) by cp.async; one tile's copies stay in flight while the
        // previous tile's complete, and the next tile's candidate index is
        // read a tile early.
        const int p = threadIdx.x;   // 0..127
        uint32_t* lut = reinterpret_cast<uint32_t*>(smem + S::LUT_OFF);
        for (int b = p; b < 256; b += 32 * R_PROD_WARPS) lut[b] = limb_entry((uint32_t)b);
        asm volatile("bar.sync 1, %0;" ::"n"(32 * R_PROD_WARPS));   // producers only
        int tile_seq = 0, tok_seq = 0;
        int pending = -1;            // stage whose copies are still in flight
        bool ok = true;
        auto complete = [&](int keep) {
            if (pending < 0) return;
            if (keep) cp_async_wait<1>(); else cp_async_wait<0>();
            fence_proxy_async_smem();
            mbar_arrive(&ctl->a_full[pending]);
            pending = -1;
        };
        for (int64_t t = blockIdx.x; ok && t < a.T; t += G) {
            const int n = a.cand_cnt[t];
            if (n <= 0) continue;
            const int qb = tok_seq & 1;
            const int32_t* cl = a.cand + t * CAP_C;
            int j_next = p < n ? cl[p] : 0;   // candidate of this thread's row in tile 0
            if (!r_wait(&ctl->q_empty[qb], ((tok_seq >> 1) & 1) ^ 1, abort, a.wait_ns)) {
                ok = false;
                break;
            }
            // the token's query limbs (B operand, H rows of 128 B per limb) and weights
            unsigned char* Qb = Qs + qb * S::Q_BUF;
            const uint8_t* qt = a.q + t * (int64_t)H * DK;
            for (int e = p; e < H * 8; e += 32 * R_PROD_WARPS) {   // (row, 16-byte chunk)
                const int r = e >> 3, c = e & 7;
                uint4 l[3];
                limbs16_lut(__ldg(reinterpret_cast<const uint4*>(qt + r * DK + c * 16)), lut, l);
#pragma unroll
                for (int i = 0; i < NLIMB; ++i)
                    *reinterpret_cast<uint4*>(Qb + i * S::Q_LIMB + sw128(r, c)) = l[i];
            }
            for (int h = p; h < H; h += 32 * R_PROD_WARPS) Ws[qb * H + h] = a.w[t * H + h];
            fence_proxy_async_smem();
            mbar_arrive(&ctl->q_full[qb]);
            ++tok_seq;
            // the candidates' key limbs, 128 per tile (A operand)
            const int tiles = (n + R_M - 1) / R_M;
            for (int ti = 0; ti < tiles; ++ti, ++tile_seq) {
                const int s = tile_seq % R_STAGES;
                const int j = j_next;
                const int row = ti * R_M + p;
                if (!r_wait(&ctl->a_empty[s], ((tile_seq / R_STAGES) & 1) ^ 1, abort, a.wait_ns)) {
                    ok = false;
                    break;
                }
                if (row < n) {
                    unsigned char* Ab = As + s * R_A_STAGE;
                    const unsigned char* src = a.klimbs + (int64_t)j * (NLIMB * DK);
#pragma unroll
                    for (int i = 0; i < NLIMB; ++i)
#pragma unroll
                        for (int c = 0; c < 8; ++c)
                            cp_async16(Ab + i * R_A_LIMB + sw128(p, c), src + i * DK + c * 16);
                }
                cp_async_commit();
                if (row + R_M < n) j_next = cl[row + R_M];   // next tile's candidate, early
                complete(1);                                   // the previous tile
                pending = s;
            }
            complete(0);
        }
        complete(0);
        if (!ok && lane == 0) r_abort(ctl, a.status);
    } else if (warp == 4) {
        // --------------------------------------------------------- MMA issuer
        int tile_seq = 0, tok_seq = 0;
        bool ok = true, issued = false;
        for (int64_t t = blockIdx.x; ok && t < a.T; t += G) {
            const int n = a.cand_cnt[t];
            if (n <= 0) continue;
            const int qb = tok_seq & 1;
            if (!r_wait(&ctl->q_full[qb], (tok_seq >> 1) & 1, abort, a.wait_ns)) {
                ok = false;
                break;
            }
            ++tok_seq;
            const uint32_t qbase = smem_u32(Qs + qb * S::Q_BUF);
            const int tiles = (n + R_M - 1) / R_M;
            for (int ti = 0; ti < tiles && ok; ++ti, ++tile_seq) {
                const int s = tile_seq % R_STAGES;
                if (!r_wait(&ctl->a_full[s], (tile_seq / R_STAGES) & 1, abort, a.wait_ns)) {
                    ok = false;
                    break;
                }
                const uint32_t abase = smem_u32(As + s * R_A_STAGE);
                constexpr uint32_t idesc = idesc_i8(R_M, H);
                // descriptors from two bases: the start-address field (bits 0-13,
                // address / 16) takes the byte offsets as plain adds (every
                // offset stays below 256 KB)
                const uint64_t ad0 = desc_k_sw128(abase);
                const uint64_t bd0 = desc_k_sw128(qbase);
                // Issue order: key limb i, then K-step, then the three groups
                // g = i .. i + 2 it feeds (query limb g - i), so that
                // consecutive MMAs accumulate into different groups and never
                // wait on each other.  Group g's slot is claimed before its first
                // MMA (g0-g2 at i = 0, g3 at i = 1, g4 at i = 2) and committed
                // after its last (g0 after i = 0, g1 after i = 1, the rest after
                // i = 2).
                auto claim = [&](int g) {
                    const int n_slot = R_GROUPS * tile_seq + g;
                    return r_wait(&ctl->slot_empty[n_slot % R_SLOTS], ((n_slot / R_SLOTS) & 1) ^ 1,
                                  abort, a.wait_ns);
                };
                auto slot_of = [&](int g) { return (R_GROUPS * tile_seq + g) % R_SLOTS; };
#pragma unroll
                for (int i = 0; i < NLIMB; ++i) {
                    if (i == 0) ok = claim(0) && claim(1) && claim(2);
                    else ok = claim(i + 2);
                    if (!ok) break;
                    tc_fence_after();
                    if (lane == 0) {
#pragma unroll
                        for (int kc = 0; kc < DK / 32; ++kc)
#pragma unroll
                            for (int g = i; g < i + NLIMB; ++g)
                                mma_i8(tmem + (uint32_t)(slot_of(g) * H),
                                       ad0 + (uint64_t)((i * R_A_LIMB + kc * 32) >> 4),
                                       bd0 + (uint64_t)(((g - i) * S::Q_LIMB + kc * 32) >> 4),
                                       idesc, (i == (g > 2 ? g - 2 : 0) && kc == 0) ? 0u : 1u);
                        issued = true;
                        if (i < NLIMB - 1) {
                            mma_commit(&ctl->slot_full[slot_of(i)]);
                        } else {
#pragma unroll
                            for (int g = NLIMB - 1; g < R_GROUPS; ++g)
                                mma_commit(&ctl->slot_full[slot_of(g)]);
                        }
                    }
                    __syncwarp();
                }
                if (!ok) break;
                if (lane == 0) {
                    mma_commit(&ctl->a_empty[s]);
                    if (ti == tiles - 1) mma_commit(&ctl->q_empty[qb]);
                }
                __syncwarp();
            }
        }
        if (!ok) {
            if (lane == 0) r_abort(ctl, a.status);
            // the MMAs issued (a tile may stop between groups) must finish
            // before TMEM is freed: one more commit, and wait for it
            if (__shfl_sync(0xffffffffu, issued ? 1 : 0, 0)) {
                if (lane == 0) mma_commit(&ctl->drain);
                __syncwarp();
                mbar_wait_drain(&ctl->drain, 0);
            }
        }
    } else if (warp >= 6) {
        // ----------------------------------------------------------- epilogue
        constexpr int HA = H >= 32 ? H / 2 : H;   // heads of the first warpgroup
        constexpr int HC = HA;                    // heads of either warpgroup, at most
        const int wg = (warp - 6) >> 2;           // 0: heads [0, HA), 1: heads [HA, H)
        const int h_lo = wg == 0 ? 0 : HA, h_hi = wg == 0 ? HA : H;
        const int sub = warp & 3;
        const int r = sub * 32 + lane;   // candidate row of the tile (TMEM lane)
        const uint32_t lane_base = tmem + ((uint32_t)(sub * 32) << 16);
        int tile_seq = 0, tok_seq = 0;
        bool ok = true;
        for (int64_t t = blockIdx.x; ok && t < a.T; t += G) {
            const int n = a.cand_cnt[t];
            if (n <= 0) continue;
            const int qb = tok_seq & 1;
            // this warpgroup's head weights, in registers for the whole token,
            // once the producers have written them
            if (!r_wait(&ctl->q_full[qb], (tok_seq >> 1) & 1, abort, a.wait_ns)) {
                ok = false;
                break;
            }
            ++tok_seq;
            float wr[HC];
#pragma unroll
            for (int h = 0; h < HC; ++h) wr[h] = h < h_hi - h_lo ? Ws[qb * H + h_lo + h] : 0.0f;
            const int tiles = (n + R_M - 1) / R_M;
            for (int ti = 0; ti < tiles; ++ti, ++tile_seq) {
                uint32_t col[R_GROUPS];
#pragma unroll
                for (int g = 0; g < R_GROUPS; ++g) {
                    const int n_slot = R_GROUPS * tile_seq + g;
                    if (!r_wait(&ctl->slot_full[n_slot % R_SLOTS], (n_slot / R_SLOTS) & 1, abort,
                                a.wait_ns)) {
                        ok = false;
                        break;
                    }
                    col[g] = lane_base + (uint32_t)((n_slot % R_SLOTS) * H);
                }
                if (!ok) break;
                tc_fence_after();
                // p_h = fl(w_h * x_h) for this warpgroup's heads, x_h from the 5 groups
                // p_h = fl(w_h * x_h) for this warpgroup's heads, 8 heads per TMEM read;
                // the first warpgroup adds them to its in-order sum at once
                float p[HC];
                float total = 0.0f;
#pragma unroll
                for (int c0 = 0; c0 < HC; c0 += 8) {
                    if (c0 >= h_hi - h_lo) break;   // (H = 16: the second warpgroup has no heads)
                    const int h0 = h_lo + c0;
                    uint32_t d[R_GROUPS][8];
#pragma unroll
                    for (int g = 0; g < R_GROUPS; ++g) tmem_ld_x8(col[g] + (uint32_t)h0, d[g]);
                    tmem_wait_ld();
#pragma unroll
                    for (int h = 0; h < 8; ++h) {
                        const int A = (int)d[0][h] + 64 * (int)d[1][h];   // |A| < 2^27
                        const int B = (int)d[2][h] + 64 * (int)d[3][h];   // |B| < 2^27
                        const float x = fmaxf(exact_dot_f32(A, B, (int)d[4][h]), 0.0f);
                        p[c0 + h] = __fmul_rn(wr[c0 + h], x);
                        if (wg == 0) total = __fadd_rn(total, p[c0 + h]);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0)
#pragma unroll
                    for (int g = 0; g < R_GROUPS; ++g)
                        mbar_arrive(&ctl->slot_empty[(R_GROUPS * tile_seq + g) % R_SLOTS]);
                // the head sum, in head order across the two warpgroups
                const int hb = tile_seq & 1;
                if (wg == 1) {
                    if (!r_wait(&ctl->hand_full[hb], (tile_seq >> 1) & 1, abort, a.wait_ns)) {
                        ok = false;
                        break;
                    }
                    total = ctl->hand[hb][r];
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&ctl->hand_empty[hb]);
                }
                if (wg == 1)
#pragma unroll
                    for (int h = 0; h < HC; ++h)
                        if (h < h_hi - h_lo) total = __fadd_rn(total, p[h]);
                if (wg == 0) {
                    if (!r_wait(&ctl->hand_empty[hb], ((tile_seq >> 1) & 1) ^ 1, abort,
                                a.wait_ns)) {
                        ok = false;
                        break;
                    }
                    ctl->hand[hb][r] = total;
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&ctl->hand_full[hb]);
                } else {
                    const int row = ti * R_M + r;
                    if (row < n) a.exact[t * CAP_C + row] = total;
                }
            }
            if (!ok) break;
            __syncwarp();
            if (lane == 0) mbar_arrive(&ctl->q_empty[qb]);   // weights of this token read
        }
        if (!ok && lane == 0) r_abort(ctl, a.status);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 5) tmem_dealloc(tmem, TMEM_COLS);
}

// ---------------------------------------------------------------------------
// K6: exact top-k of each token's candidates, best first, ties to the lowest
// key; fewer visible keys than k pad with -1 / -inf.  Unless the candidates
// are all the visible keys, the m-th best of them (m = min(k, visible)) must
// reach the token's threshold (every other key scores below it); otherwise
// the token is flagged for the exact-row path, which overwrites its outputs.
__global__ void __launch_bounds__(SEL_THREADS) dsa_select_kernel(
    const int32_t* __restrict__ cand, const float* __restrict__ exact,
    const int* __restrict__ cand_cnt, const float* __restrict__ tok_tau, int64_t n_tok, int64_t L,
    int64_t pos0, int k, int* __restrict__ status, int32_t* __restrict__ out_idx,
    float* __restrict__ out_sc) {
    extern __shared__ uint64_t ssm[];
    uint64_t* keys = ssm;               // CAP_C
    uint64_t* best = ssm + CAP_C;       // KMAX
    __shared__ unsigned sm[256 + SEL_THREADS / 32 + 4];
    __shared__ int nb;
    const int64_t t = blockIdx.x;
    const int n = cand_cnt[t];
    const int64_t vis = max((int64_t)0, min(L, pos0 + t + 1));
    if (n <= 0 && vis > 0) return;   // flagged: the exact-row fallback writes this token
    const int m = (int)min((int64_t)k, (int64_t)n);
    for (int i = threadIdx.x; i < n; i += SEL_THREADS)
        keys[i] = make_cand(f32_key(exact[t * CAP_C + i]), (uint32_t)cand[t * CAP_C + i]);
    const int kp = next_pow2(max(m, 1));
    for (int i = threadIdx.x; i < kp; i += SEL_THREADS) best[i] = 0ull;
    if (threadIdx.x == 0) nb = 0;
    __syncthreads();
    const uint64_t T = band_select<SEL_THREADS>(keys, n, m, sm);
    for (int i0 = threadIdx.x & ~31; i0 < n; i0 += SEL_THREADS) {
        const int i = i0 + (threadIdx.x & 31);
        const uint64_t c = i < n ? keys[i] : 0ull;
        const int pos = warp_append(i < n && c >= T, &nb);
        if (pos >= 0) best[pos] = c;
    }
    __syncthreads();
    block_bitonic_sort_desc(best, kp);
    if (threadIdx.x == 0 && n < vis) {
        const int m_req = (int)min((int64_t)k, vis);
        if (n < m_req || !(cand_score(best[m_req - 1]) >= tok_tau[t])) {
            const int pos = atomicAdd(&status[ST_NFLAG], 1);
            if (pos < n_tok) status[ST_FLAGS + pos] = (int)t;
        }
    }
    for (int i = threadIdx.x; i < k; i += SEL_THREADS) {
        const uint64_t c = i < m ? best[i] : 0ull;
        out_idx[t * k + i] = c ? (int32_t)cand_row(c) : -1;
        out_sc[t * k + i] = c ? cand_score(c) : -INFINITY;
    }
}

constexpr size_t SEL_SMEM = sizeof(uint64_t) * (CAP_C + KMAX);

// ---------------------------------------------------------------------------
// Fallback: every visible key's exact score of each flagged token of a pass
// (blockIdx.y picks the token from the pass's part of the flagged list), on
// CUDA cores, in the reference's arithmetic (exact integer dots, fp32 head
// sum in order), into row blockIdx.y of `rows` ([FB_ROWS][L]).
__global__ void dsa_exact_rows_kernel(const uint8_t* __restrict__ q, const float* __restrict__ w,
                                      const uint8_t* __restrict__ keys, int64_t L, int64_t pos0,
                                      int H, const int* __restrict__ flagged,
                                      float* __restrict__ rows) {
    __shared__ int qv[64 * DK];
    __shared__ float ws[64];
    const int64_t t = flagged[blockIdx.y];
    const uint8_t* qt = q + t * (int64_t)H * DK;
    for (int i = threadIdx.x; i < H * DK; i += blockDim.x) qv[i] = e4m3_scaled(qt[i]);
    for (int h = threadIdx.x; h < H; h += blockDim.x) ws[h] = w[t * H + h];
    __syncthreads();
    float* row = rows + (int64_t)blockIdx.y * L;
    const int64_t vis = max((int64_t)0, min(L, pos0 + t + 1));
    for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < vis;
         j += (int64_t)gridDim.x * blockDim.x) {
        int kv[DK];
#pragma unroll 8
        for (int d = 0; d < DK; ++d) kv[d] = e4m3_scaled(keys[j * DK + d]);
        float total = 0.0f;
        for (int h = 0; h < H; ++h) {
            long long acc = 0;
#pragma unroll 8
            for (int d = 0; d < DK; ++d) acc += (long long)qv[h * DK + d] * kv[d];
            const float x = acc > 0 ? __ll2float_rn(acc) * (1.0f / 262144.0f) : 0.0f;
            total = __fadd_rn(total, __fmul_rn(ws[h], x));
        }
        row[j] = total;
    }
}

// Fallback: the exact top-k of each flagged token's exact row (one block per
// flagged token of the pass, its row in `rows`): a block radix select over
// the visible scores, then the k best sorted, ties to the lowest key.
__global__ void __launch_bounds__(SEL_THREADS) dsa_row_select_kernel(
    const float* __restrict__ rows, int64_t L, int64_t pos0, int k,
    const int* __restrict__ flagged, int32_t* __restrict__ out_idx, float* __restrict__ out_sc) {
    extern __shared__ uint64_t fsm[];   // KMAX
    __shared__ unsigned sm[256 + SEL_THREADS / 32 + 4];
    __shared__ int nb;
    const int64_t t = flagged[blockIdx.x];
    const float* row = rows + (int64_t)blockIdx.x * L;
    const int64_t vis = max((int64_t)0, min(L, pos0 + t + 1));
    const int m = (int)min((int64_t)k, vis);
    auto key_at = [row](int64_t j) { return make_cand(f32_key(row[j]), (uint32_t)j); };
    const int kp = next_pow2(max(m, 1));
    for (int i = threadIdx.x; i < kp; i += SEL_THREADS) fsm[i] = 0ull;
    if (threadIdx.x == 0) nb = 0;
    __syncthreads();
    const uint64_t T = band_select_fn<SEL_THREADS>(key_at, vis, m, sm);
    for (int64_t j0 = threadIdx.x & ~31; j0 < vis; j0 += SEL_THREADS) {
        const int64_t j = j0 + (threadIdx.x & 31);
        const uint64_t c = j < vis ? key_at(j) : 0ull;
        const int pos = warp_append(j < vis && c >= T, &nb);
        if (pos >= 0) fsm[pos] = c;
    }
    __syncthreads();
    block_bitonic_sort_desc(fsm, kp);
    for (int i = threadIdx.x; i < k; i += SEL_THREADS) {
        const uint64_t c = i < m ? fsm[i] : 0ull;
        out_idx[t * k + i] = c ? (int32_t)cand_row(c) : -1;
        out_sc[t * k + i] = c ? cand_score(c) : -INFINITY;
    }
}

size_t up256(size_t v) { return (v + 255) & ~size_t(255); }

}  // namespace

// Workspace of the exact selection: status words and flagged tokens, key
// norms, limbs and the sample, per-token thresholds and bitmaps, candidate
// lists and their exact scores, and the fallback's exact rows.
struct DsaExactLayout {
    size_t status, norms, limbs, skeys, sscores, tok_e, tok_tau, bitmap, cand,
        cand_cnt, exact, rows, total;
    int S, W;
};

static DsaExactLayout dsa_exact_layout(int64_t T, int64_t L) {
    DsaExactLayout d;
    // the sample only matters for tokens that see more keys than CAP_C
    d.S = L > CAP_C ? BAND_SAMPLE : 0;
    d.W = (int)((L + 31) / 32);
    size_t o = 0;
    d.status = o; o += up256(sizeof(int) * (size_t)(ST_FLAGS + T));
    d.norms = o; o += up256(sizeof(float) * (size_t)L);
    d.limbs = o; o += up256((size_t)L * NLIMB * DK);
    d.skeys = o; o += up256((size_t)d.S * DK);
    d.sscores = o; o += up256(sizeof(float) * (size_t)T * d.S);
    d.tok_e = o; o += up256(sizeof(float) * (size_t)T);
    d.tok_tau = o; o += up256(sizeof(float) * (size_t)T);
    d.bitmap = o; o += up256(sizeof(uint32_t) * (size_t)T * d.W);
    d.cand = o; o += up256(sizeof(int32_t) * (size_t)T * CAP_C);
    d.cand_cnt = o; o += up256(sizeof(int) * (size_t)T);
    d.exact = o; o += up256(sizeof(float) * (size_t)T * CAP_C);
    d.rows = o; o += up256(sizeof(float) * (size_t)FB_ROWS * L);
    d.total = o;
    return d;
}

size_t dsa_exact_ws_bytes(int64_t T, int64_t L) { return dsa_exact_layout(T, L).total; }

static TokArgs tok_args(const uint8_t* q, const float* w, int64_t T, int64_t H, int64_t L,
                        int64_t pos0, int64_t topk, const DsaExactBufs& b, unsigned char* wb,
                        const DsaExactLayout& d) {
    TokArgs a;
    a.q = q; a.w = w; a.norms = b.norms; a.sscores = b.sscores; a.bitmap = b.bitmap;
    a.tok_e = b.tok_e; a.tok_tau = b.tok_tau;
    a.cand = reinterpret_cast<int32_t*>(wb + d.cand);
    a.cand_cnt = reinterpret_cast<int*>(wb + d.cand_cnt);
    a.status = b.status;
    a.T = T; a.L = L; a.pos0 = pos0; a.H = (int)H; a.k = (int)topk; a.S = b.S; a.W = b.W;
    return a;
}

hmm_status_t dsa_exact_prepare(const uint8_t* keys, int64_t T, int64_t L, int64_t topk,
                               void* ws, cudaStream_t st, DsaExactBufs* b) {
    (void)topk;
    const DsaExactLayout d = dsa_exact_layout(T, L);
    unsigned char* w = static_cast<unsigned char*>(ws);
    b->status = reinterpret_cast<int*>(w + d.status);
    b->norms = reinterpret_cast<float*>(w + d.norms);
    b->skeys = w + d.skeys;
    b->sscores = reinterpret_cast<float*>(w + d.sscores);
    b->tok_e = reinterpret_cast<float*>(w + d.tok_e);
    b->tok_tau = reinterpret_cast<float*>(w + d.tok_tau);
    b->bitmap = reinterpret_cast<uint32_t*>(w + d.bitmap);
    b->S = d.S;
    b->W = d.W;
    HMM_CUDA_TRY(cudaMemsetAsync(b->status, 0, sizeof(int) * ST_FLAGS, st));
    if (L > 0) {
        const int64_t blocks = std::min<int64_t>((L + 7) / 8, 8 * (int64_t)device_sm_count());
        dsa_key_prep_kernel<<<(unsigned)blocks, 256, 0, st>>>(keys, L, b->norms, b->status);
        hmm_status_t s = check_launch("dsa_key_prep_kernel");
        if (s != HMM_OK) return s;
    }
    if (d.S > 0) {
        const int64_t n16 = (int64_t)d.S * (DK / 16);
        dsa_sample_gather_kernel<<<(unsigned)((n16 + 255) / 256), 256, 0, st>>>(keys, L, d.S,
                                                                                 b->skeys);
        return check_launch("dsa_sample_gather_kernel");
    }
    return HMM_OK;
}

hmm_status_t dsa_exact_thresholds(const uint8_t* q, const float* w, int64_t T, int64_t H,
                                  int64_t L, int64_t pos0, int64_t topk, const DsaExactBufs& b,
                                  cudaStream_t st) {
    const DsaExactLayout d = dsa_exact_layout(T, L);
    unsigned char* wb = reinterpret_cast<unsigned char*>(b.status) - d.status;
    const TokArgs a = tok_args(q, w, T, H, L, pos0, topk, b, wb, d);
    dsa_threshold_kernel<<<(unsigned)T, BAND_THREADS, 0, st>>>(a);
    return check_launch("dsa_threshold_kernel");
}

hmm_status_t dsa_exact_select(const uint8_t* q, const uint8_t* keys, const float* w, int64_t T,
                              int64_t H, int64_t L, int64_t pos0, int64_t topk,
                              const DsaExactBufs& b, int32_t* out_idx, float* out_sc, void* ws,
                              cudaStream_t st) {
    const DsaExactLayout d = dsa_exact_layout(T, L);
    unsigned char* wb = static_cast<unsigned char*>(ws);
    int* status = b.status;
    int32_t* cand = reinterpret_cast<int32_t*>(wb + d.cand);
    int* cand_cnt = reinterpret_cast<int*>(wb + d.cand_cnt);
    float* exact = reinterpret_cast<float*>(wb + d.exact);
    float* rows = reinterpret_cast<float*>(wb + d.rows);
    hmm_status_t s;

    const TokArgs ta = tok_args(q, w, T, H, L, pos0, topk, b, wb, d);
    dsa_cand_kernel<<<(unsigned)T, BAND_THREADS, 0, st>>>(ta);
    s = check_launch("dsa_cand_kernel");
    if (s != HMM_OK) return s;

    // the key limbs, right before the gather that reads them
    {
        const int64_t n16 = L * (DK / 16);
        const int64_t blocks = std::min<int64_t>((n16 + 255) / 256, 8 * (int64_t)device_sm_count());
        dsa_key_limbs_kernel<<<(unsigned)blocks, 256, 0, st>>>(keys, L, wb + d.limbs);
        s = check_launch("dsa_key_limbs_kernel");
        if (s != HMM_OK) return s;
    }
    RescoreArgs ra;
    ra.q = q; ra.w = w; ra.klimbs = wb + d.limbs; ra.cand = cand; ra.cand_cnt = cand_cnt;
    ra.exact = exact; ra.status = status; ra.T = T; ra.wait_ns = wait_limit_ns();
    const int grid = std::max(1, (int)std::min<int64_t>(device_sm_count(), T));
    if (H == 64) {
        HMM_CUDA_TRY(cudaFuncSetAttribute(dsa_rescore_kernel<64>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)RescoreSmem<64>::BYTES));
        dsa_rescore_kernel<64><<<grid, R_THREADS, RescoreSmem<64>::BYTES, st>>>(ra);
    } else if (H == 32) {
        HMM_CUDA_TRY(cudaFuncSetAttribute(dsa_rescore_kernel<32>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)RescoreSmem<32>::BYTES));
        dsa_rescore_kernel<32><<<grid, R_THREADS, RescoreSmem<32>::BYTES, st>>>(ra);
    } else {
        HMM_CUDA_TRY(cudaFuncSetAttribute(dsa_rescore_kernel<16>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)RescoreSmem<16>::BYTES));
        dsa_rescore_kernel<16><<<grid, R_THREADS, RescoreSmem<16>::BYTES, st>>>(ra);
    }
    s = check_launch("dsa_rescore_kernel");
    if (s != HMM_OK) return s;

    HMM_CUDA_TRY(cudaFuncSetAttribute(dsa_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)SEL_SMEM));
    dsa_select_kernel<<<(unsigned)T, SEL_THREADS, SEL_SMEM, st>>>(
        cand, exact, cand_cnt, b.tok_tau, T, L, pos0, (int)topk, status, out_idx, out_sc);
    s = check_launch("dsa_select_kernel");
    if (s != HMM_OK) return s;

    int h[ST_FLAGS] = {0, 0, 0, 0};
    HMM_CUDA_TRY(cudaMemcpyAsync(h, status, sizeof(h), cudaMemcpyDeviceToHost, st));
    HMM_CUDA_TRY(cudaStreamSynchronize(st));
    if (h[ST_TIMEOUT])
        return set_error(HMM_ERR_TIMEOUT,
                         "dsa indexer: a bounded pipeline wait gave up; outputs invalid");
    if (h[ST_NAN])
        return set_error(HMM_ERR_INVALID,
                         "q or keys hold an e4m3 NaN encoding (0x7f / 0xff), which has no "
                         "exact score");
    const int nflag = (int)std::min<int64_t>(h[ST_NFLAG], T);
    // tokens whose candidates did not fit: exact rows, then their top-k, FB_ROWS
    // tokens per pass through the rows buffer
    const int bx = (int)std::max<int64_t>(1, std::min<int64_t>((L + 127) / 128,
                                                               2 * device_sm_count()));
    for (int f0 = 0; f0 < nflag; f0 += FB_ROWS) {
        const int nf = std::min(FB_ROWS, nflag - f0);
        const int* flagged = status + ST_FLAGS + f0;
        dsa_exact_rows_kernel<<<dim3(bx, nf), 128, 0, st>>>(q, w, keys, L, pos0, (int)H, flagged,
                                                           rows);
        s = check_launch("dsa_exact_rows_kernel");
        if (s != HMM_OK) return s;
        const size_t fsm = sizeof(uint64_t) * KMAX;
        dsa_row_select_kernel<<<nf, SEL_THREADS, fsm, st>>>(rows, L, pos0, (int)topk, flagged,
                                                           out_idx, out_sc);
        s = check_launch("dsa_row_select_kernel");
        if (s != HMM_OK) return s;
    }
    return HMM_OK;
}

}  // namespace hmm
