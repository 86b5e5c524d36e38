// indexers.cu — int16 sparse-attention indexers: LServe block top-k,
// SeerAttention token-budget top-k and SeerAttention threshold bitmap.
//
// Reference: the CPU references inside the HLS testbenches
// kernels/lserve/indexer_lserve_tb.cpp:20-92,
// kernels/seerattention/indexer_seer_token_budget_tb.cpp:19-73 and
// kernels/seerattention/indexer_seer_threshold_tb.cpp:18-77 (one index head,
// int16 keys and queries, exact integer dot products).
//
// Causal layout of the testbenches: query q sits at position L + q / 8 and
// sees positions 0 .. L + q / 8.  Position p < L is past key p; position
// L + g is the key produced by the last query of group g,
// new_keys[min(8g + 7, q)] (the query's own key for its own group).
//
// One thread per visible position computes the exact int64 dot product
// (int16 x int16 products summed in int64; the order is irrelevant for
// integers).  The threshold bitmap is written straight from warp ballots;
// the top-k indexers write 64-bit (score key, position) candidates and reuse
// the exact candidate merge of the flat path.
#include <cuda_runtime.h>

#include <algorithm>

#include "heteromm_cuda.h"
#include "hmm_common.cuh"

namespace hmm {
hmm_status_t launch_cand_merge_i32(const uint64_t* cand, int64_t cap, const int* counts, int nq,
                                   int k, int32_t* out_idx, float* out_scores, cudaStream_t st);

namespace {

constexpr int IX_THREADS = 256;
constexpr int IX_MAX_D = 256;

enum IxMode { IX_THRESHOLD = 0, IX_BUDGET = 1, IX_LSERVE = 2 };

struct IxArgs {
    const int16_t* past;      // [L][D]
    const int16_t* queries;   // [nq][D]
    const int16_t* new_keys;  // [nq][D]
    int64_t L;
    int nq;
    int D;
    int64_t threshold;
    int block;                // LServe block (16)
    int64_t cap;              // candidates per query (positions or blocks)
    uint64_t* cand;           // [nq][cap]
    int* counts;              // [nq]
    uint64_t* bitmap;         // [nq][wpq]
    int64_t wpq;
};

__device__ __forceinline__ const int16_t* key_at(const IxArgs& a, int q, int64_t pos) {
    if (pos < a.L) return a.past + pos * a.D;
    const int64_t g = pos - a.L;
    const int64_t i = 8 * g + 7 < q ? 8 * g + 7 : q;
    return a.new_keys + i * a.D;
}

// grid (ceil(max positions / 256), nq): thread = position
template <int MODE>
__global__ void __launch_bounds__(IX_THREADS) indexer_kernel(const IxArgs a) {
    __shared__ __align__(16) int16_t qs[IX_MAX_D];
    const int q = blockIdx.y;
    const int64_t ns = a.L + q / 8 + 1;                  // visible positions
    const int64_t pos = (int64_t)blockIdx.x * IX_THREADS + threadIdx.x;
    for (int d = threadIdx.x; d < a.D; d += IX_THREADS) qs[d] = a.queries[(int64_t)q * a.D + d];
    __syncthreads();
    if ((int64_t)blockIdx.x * IX_THREADS >= ns) {
        if (MODE == IX_BUDGET && threadIdx.x == 0 && blockIdx.x == 0) a.counts[q] = 0;
        return;   // the whole block is past this query's window
    }
    long long dot = 0;
    const bool vis = pos < ns;
    if (vis) {
        const int16_t* k = key_at(a, q, pos);
        for (int d = 0; d < a.D; d += 2) {
            const int kk = *reinterpret_cast<const int*>(k + d);
            const int qq = *reinterpret_cast<const int*>(qs + d);
            dot += (long long)((int)(short)(kk & 0xffff) * (int)(short)(qq & 0xffff));
            dot += (long long)((kk >> 16) * (qq >> 16));
        }
    }
    if (MODE == IX_THRESHOLD) {
        // bit p % 64 of word p / 64: dot > threshold (strict), visible only
        const unsigned m = __ballot_sync(0xffffffffu, vis && dot > a.threshold);
        if ((threadIdx.x & 31) == 0 && pos < ns) {   // this warp sees a position
            uint32_t* w = reinterpret_cast<uint32_t*>(a.bitmap + (int64_t)q * a.wpq);
            w[pos >> 5] = m;   // little-endian halves of the 64-bit words
        }
    } else if (MODE == IX_BUDGET) {
        if (vis) a.cand[(int64_t)q * a.cap + pos] = make_cand(f32_key((float)dot), (uint32_t)pos);
        if (blockIdx.x == 0 && threadIdx.x == 0) a.counts[q] = (int)ns;
    } else {
        // LServe: max over the positions of each block (block | 32), strict >
        // from -1e30f as the reference does; blocks are aligned to lanes
        float s = vis ? (float)dot : -1e30f;
        for (int o = a.block >> 1; o > 0; o >>= 1)
            s = fmaxf(s, __shfl_xor_sync(0xffffffffu, s, o));
        const int64_t b = pos / a.block;
        const int64_t nblk = (ns + a.block - 1) / a.block;
        if ((threadIdx.x % a.block) == 0 && b < nblk)
            a.cand[(int64_t)q * a.cap + b] = make_cand(f32_key(s), (uint32_t)b);
        if (blockIdx.x == 0 && threadIdx.x == 0) a.counts[q] = (int)nblk;
    }
}

}  // namespace
}  // namespace hmm

using namespace hmm;

namespace {
hmm_status_t ix_common(const int16_t* past, int64_t L, const int16_t* queries,
                       const int16_t* new_keys, int64_t nq, int64_t D) {
    HMM_REQUIRE(L >= 0 && L < (int64_t(1) << 30), "L out of range");
    HMM_REQUIRE(nq >= 0 && nq <= 65535, "n_queries must be in [0, 65535]");
    HMM_REQUIRE(D >= 2 && D <= IX_MAX_D && D % 2 == 0, "D must be even and in [2, %d]",
                IX_MAX_D);
    HMM_REQUIRE(nq == 0 || (queries && new_keys), "null query / new-key pointer");
    HMM_REQUIRE(L == 0 || past, "past is null");
    HMM_REQUIRE((reinterpret_cast<uintptr_t>(past) % 4) == 0 &&
                    (reinterpret_cast<uintptr_t>(new_keys) % 4) == 0,
                "key arrays must be 4-byte aligned");
    return HMM_OK;
}
int64_t max_positions(int64_t L, int64_t nq) { return L + (nq > 0 ? (nq - 1) / 8 : 0) + 1; }
}  // namespace

extern "C" int64_t hmm_seer_words_per_query(int64_t L, int64_t n_queries) {
    if (L < 0 || n_queries < 0) return 0;
    return ((max_positions(L, n_queries) - 1 + 128) / 128) * 2;
}

extern "C" hmm_status_t hmm_seer_threshold_i16(const int16_t* past, int64_t L,
                                               const int16_t* queries, const int16_t* new_keys,
                                               int64_t n_queries, int64_t D, int64_t threshold,
                                               uint64_t* out_bitmap, void* stream) {
    hmm_status_t s = ix_common(past, L, queries, new_keys, n_queries, D);
    if (s != HMM_OK) return s;
    if (n_queries == 0) return HMM_OK;
    HMM_REQUIRE(out_bitmap, "out_bitmap is null");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int64_t wpq = hmm_seer_words_per_query(L, n_queries);
    HMM_CUDA_TRY(cudaMemsetAsync(out_bitmap, 0, sizeof(uint64_t) * wpq * n_queries, st));
    IxArgs a{};
    a.past = past; a.queries = queries; a.new_keys = new_keys;
    a.L = L; a.nq = (int)n_queries; a.D = (int)D; a.threshold = threshold;
    a.bitmap = out_bitmap; a.wpq = wpq;
    const int64_t mp = max_positions(L, n_queries);
    indexer_kernel<IX_THRESHOLD><<<dim3((unsigned)((mp + IX_THREADS - 1) / IX_THREADS),
                                        (unsigned)n_queries), IX_THREADS, 0, st>>>(a);
    return check_launch("indexer_kernel<threshold>");
}

extern "C" size_t hmm_indexer_workspace_size(int64_t L, int64_t n_queries) {
    if (L < 0 || n_queries < 0) return 0;
    const size_t cap = (size_t)max_positions(L, n_queries);
    return ((sizeof(uint64_t) * cap * n_queries + 255) & ~size_t(255)) +
           sizeof(int) * n_queries + 256;
}

namespace {
template <int MODE>
hmm_status_t run_topk_indexer(const int16_t* past, int64_t L, const int16_t* queries,
                              const int16_t* new_keys, int64_t nq, int64_t D, int64_t topk,
                              int64_t block, int32_t* out, void* ws, size_t ws_bytes,
                              void* stream) {
    hmm_status_t s = ix_common(past, L, queries, new_keys, nq, D);
    if (s != HMM_OK) return s;
    HMM_REQUIRE(topk >= 1 && topk <= 4096, "topk must be in [1, 4096]");
    if (nq == 0) return HMM_OK;
    HMM_REQUIRE(out, "out is null");
    const int64_t mp = max_positions(L, nq);
    HMM_REQUIRE(mp < (int64_t(1) << 31), "too many positions");
    const size_t need = hmm_indexer_workspace_size(L, nq);
    if (!ws || ws_bytes < need)
        return set_error(HMM_ERR_OOM, "workspace too small: %zu < %zu", ws_bytes, need);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    unsigned char* w = static_cast<unsigned char*>(ws);
    IxArgs a{};
    a.past = past; a.queries = queries; a.new_keys = new_keys;
    a.L = L; a.nq = (int)nq; a.D = (int)D; a.block = (int)block;
    a.cap = MODE == IX_LSERVE ? (mp + block - 1) / block : mp;
    a.cand = reinterpret_cast<uint64_t*>(w);
    a.counts = reinterpret_cast<int*>(w + ((sizeof(uint64_t) * mp * nq + 255) & ~size_t(255)));
    indexer_kernel<MODE><<<dim3((unsigned)((mp + IX_THREADS - 1) / IX_THREADS), (unsigned)nq),
                           IX_THREADS, 0, st>>>(a);
    s = check_launch(MODE == IX_LSERVE ? "indexer_kernel<lserve>" : "indexer_kernel<budget>");
    if (s != HMM_OK) return s;
    return launch_cand_merge_i32(a.cand, a.cap, a.counts, (int)nq, (int)topk, out, nullptr, st);
}
}  // namespace

extern "C" hmm_status_t hmm_seer_budget_i16(const int16_t* past, int64_t L,
                                            const int16_t* queries, const int16_t* new_keys,
                                            int64_t n_queries, int64_t D, int64_t topk,
                                            int32_t* out, void* workspace,
                                            size_t workspace_bytes, void* stream) {
    return run_topk_indexer<IX_BUDGET>(past, L, queries, new_keys, n_queries, D, topk, 1, out,
                                       workspace, workspace_bytes, stream);
}

extern "C" hmm_status_t hmm_lserve_topk_i16(const int16_t* past, int64_t L,
                                            const int16_t* queries, const int16_t* new_keys,
                                            int64_t n_queries, int64_t D, int64_t topk,
                                            int64_t block, int32_t* out, void* workspace,
                                            size_t workspace_bytes, void* stream) {
    HMM_REQUIRE(block == 1 || block == 2 || block == 4 || block == 8 || block == 16 ||
                    block == 32,
                "block must be a power of two <= 32, got %lld", (long long)block);
    return run_topk_indexer<IX_LSERVE>(past, L, queries, new_keys, n_queries, D, topk, block,
                                       out, workspace, workspace_bytes, stream);
}
