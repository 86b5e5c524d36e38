// hmm_common.cuh — shared device helpers for the HeteroMM sm_100a kernels:
// status reporting, orderable score keys, warp/block radix select and a
// shared-memory bitonic sort.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "heteromm_cuda.h"

namespace hmm {

// ---------------------------------------------------------------- status

// Records `msg` as the calling thread's last error and returns `st`.
hmm_status_t set_error(hmm_status_t st, const char* fmt, ...);
// Maps the current CUDA error state after a launch to a status.
hmm_status_t check_launch(const char* what);
// CUDA-event bracket around one launch of a dominant kernel, recorded only
// while hmm_profile_enable(1) is in effect (both events null otherwise).
struct ProfileMark {
    cudaEvent_t start, stop;
};
ProfileMark profile_begin(cudaStream_t st);
void profile_end(const ProfileMark& m, cudaStream_t st);
// Number of SMs of the current device (cached per device).
int device_sm_count();
// Limit of every bounded pipeline wait of the tensor-core kernels, in ns:
// 2 s unless hmm_debug_set_wait_limit_ns changed it.
uint64_t wait_limit_ns();

#define HMM_REQUIRE(cond, ...)                                   \
    do {                                                         \
        if (!(cond)) return ::hmm::set_error(HMM_ERR_INVALID, __VA_ARGS__); \
    } while (0)

#define HMM_CUDA_TRY(call)                                                   \
    do {                                                                     \
        cudaError_t e_ = (call);                                             \
        if (e_ != cudaSuccess)                                               \
            return ::hmm::set_error(HMM_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
    } while (0)

// ------------------------------------------------------------------ keys
// A score maps to a 32-bit key whose unsigned order is the reference's
// `a > b` order: NaN -> 0 (below every number), -0.0 -> key of +0.0.  A
// candidate is the 64-bit composite (key << 32) | ~row, so larger composite =
// better score, and among equal scores the lower row wins.  Rows are < 2^31,
// so every real composite is >= 2^31 and the value 0 can mark an empty slot.

__host__ __device__ __forceinline__ uint32_t f32_key(float f) {
#ifdef __CUDA_ARCH__
    uint32_t u = __float_as_uint(f);
#else
    uint32_t u;
    __builtin_memcpy(&u, &f, 4);
#endif
    if (f != f) return 0u;
    if (f == 0.0f) u = 0u;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__host__ __device__ __forceinline__ float key_to_f32(uint32_t k) {
    uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
#ifdef __CUDA_ARCH__
    return __uint_as_float(u);
#else
    float f;
    __builtin_memcpy(&f, &u, 4);
    return f;
#endif
}

__host__ __device__ __forceinline__ uint64_t make_cand(uint32_t key, uint32_t row) {
    return ((uint64_t)key << 32) | (uint64_t)(~row);
}
__host__ __device__ __forceinline__ uint32_t cand_row(uint64_t c) { return ~(uint32_t)c; }
__host__ __device__ __forceinline__ float cand_score(uint64_t c) {
    return key_to_f32((uint32_t)(c >> 32));
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t h) {
    return __uint_as_float((uint32_t)h << 16);
}

// --------------------------------------------------------- radix select
// Threshold T such that exactly min(k, M) of the unique, nonzero composites
// keys[0..M) are >= T.  Eight 8-bit passes from the top byte, stopping as soon
// as the bucket that holds the k-th key is taken whole.  One warp; `hist` is
// 256 words of shared memory owned by the warp.
__device__ __forceinline__ uint64_t warp_select_threshold(const uint64_t* keys, int M, int k,
                                                          unsigned* hist) {
    const int lane = threadIdx.x & 31;
    if (k >= M) return 0ull;
    uint64_t prefix = 0, mask = 0;
    unsigned need = (unsigned)k;
    for (int shift = 56; shift >= 0; shift -= 8) {
        for (int b = lane; b < 256; b += 32) hist[b] = 0;
        __syncwarp();
        for (int i = lane; i < M; i += 32) {
            const uint64_t key = keys[i];
            if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255], 1u);
        }
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
        if (cnt == need) break;
    }
    return prefix;
}

// Stable in-place compaction of keys >= T; returns the new count.  One warp.
__device__ __forceinline__ int warp_compact_ge(uint64_t* keys, int M, uint64_t T) {
    const int lane = threadIdx.x & 31;
    int out = 0;
    for (int base = 0; base < M; base += 32) {
        const int i = base + lane;
        const uint64_t key = i < M ? keys[i] : 0ull;
        const bool keep = i < M && key >= T;
        const unsigned b = __ballot_sync(0xffffffffu, keep);
        __syncwarp();
        if (keep) keys[out + __popc(b & ((1u << lane) - 1u))] = key;
        out += __popc(b);
        __syncwarp();
    }
    return out;
}

// Block-wide inclusive scan of one value per thread (blockDim.x == 256).
__device__ __forceinline__ unsigned block_scan_incl_256(unsigned v, unsigned* warp_tot) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
    }
    if (lane == 31) warp_tot[w] = v;
    __syncthreads();
    if (w == 0) {
        unsigned t = lane < 8 ? warp_tot[lane] : 0u;
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
            const unsigned u = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= o) t += u;
        }
        if (lane < 8) warp_tot[lane] = t;
    }
    __syncthreads();
    const unsigned r = v + (w > 0 ? warp_tot[w - 1] : 0u);
    __syncthreads();
    return r;
}

// Same threshold as warp_select_threshold over keys in global memory, one
// block of 256 threads; `sm` is >= 300 words of shared memory.  Zero keys
// (empty slots) are allowed; they are all equal and below every real key.
__device__ __forceinline__ uint64_t block_select_threshold(const uint64_t* keys, int64_t M,
                                                           int64_t k, unsigned* sm) {
    unsigned* hist = sm;          // 256
    unsigned* wt = sm + 256;      // 8
    unsigned* res = sm + 272;     // 3
    if (k >= M) return 0ull;
    uint64_t prefix = 0, mask = 0;
    unsigned need = (unsigned)k;
    for (int shift = 56; shift >= 0; shift -= 8) {
        hist[threadIdx.x] = 0;
        __syncthreads();
        for (int64_t i = threadIdx.x; i < M; i += 256) {
            const uint64_t key = keys[i];
            if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255], 1u);
        }
        __syncthreads();
        const unsigned c = hist[255 - threadIdx.x];
        const unsigned incl = block_scan_incl_256(c, wt);
        const unsigned excl = incl - c;
        if (excl < need && need <= incl) {
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

// Descending bitonic sort of n (power of two) keys in shared memory.
__device__ __forceinline__ void block_bitonic_sort_desc(uint64_t* a, int n) {
    for (int size = 2; size <= n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            __syncthreads();
            for (int i = threadIdx.x; i < n / 2; i += blockDim.x) {
                const int lo = 2 * i - (i & (stride - 1));
                const int hi = lo + stride;
                const bool desc = ((lo & size) == 0);
                const uint64_t x = a[lo], y = a[hi];
                if ((x < y) == desc) { a[lo] = y; a[hi] = x; }
            }
        }
    }
    __syncthreads();
}

__host__ __device__ __forceinline__ int next_pow2(int v) {
    int p = 1;
    while (p < v) p <<= 1;
    return p;
}

}  // namespace hmm
