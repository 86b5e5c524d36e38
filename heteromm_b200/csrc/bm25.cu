// bm25.cu — BM25 fused score + top-k over a CSR inverted index.
//
// Reference: FusedBM25Retrieval::run_cpu_kernel
// (steps/example_kernel/bm25_fpga_retrieval.cpp:143-205): fp64 BM25 with
// k1 = 1.2, b = 0.75, idf = log((N - df + 0.5) / (df + 0.5) + 1.0),
// per matching (term, doc): idf * (tf * (k1 + 1)) / (tf + k1 * (1 - b + b * dl / avg_dl)),
// summed over the query's terms, then the top-k documents.
//
// Index layout (CSR): postings of term t are [term_ptr[t], term_ptr[t+1]) with
// ascending doc ids (post_doc int32) and term frequencies (post_tf uint16);
// doc_len[d] = sum of the doc's term frequencies.
//
// Design: documents are cut into ranges of BM_RANGE docs.  One block per
// (range, query) keeps that range's fp64 scores in shared memory, adds the
// query's terms one after another in ascending term order (a barrier between
// terms, so every document's sum has the same order as the oracle's), then
// keeps the range's top-k; a second kernel merges the ranges.  Postings are
// read once per query from HBM; the per-term range boundaries (skips) and the
// per-document length factor k1 * (1 - b + b * dl / avg_dl) are built once per
// index by hmm_bm25_prepare.  Every fp64 operation is an explicit IEEE
// round-to-nearest intrinsic, in the reference's order, so scores are
// bit-identical to the reference's x86-64 (SSE2, no FMA) doubles.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <vector>

#include "heteromm_cuda.h"
#include "hmm_common.cuh"

namespace hmm {
namespace {

constexpr int BM_RANGE = HMM_BM25_RANGE_DOCS;   // docs per block: 32 KB of fp64 scores
constexpr int BM_THREADS = 256;
constexpr int BM_MAX_QLEN = 64;
constexpr int BM_KMAX = 128;
constexpr double BM_K1 = 1.2;
constexpr double BM_B = 0.75;

// Orderable 64-bit key of a double: larger key = larger value; NaN -> 0,
// -0.0 -> key of +0.0 (the reference's `>` comparator).
__device__ __forceinline__ uint64_t f64_key(double x) {
    if (x != x) return 0ull;
    if (x == 0.0) x = 0.0;
    const uint64_t b = (uint64_t)__double_as_longlong(x);
    return (b >> 63) ? ~b : (b | 0x8000000000000000ull);
}

__device__ __forceinline__ double key_to_f64(uint64_t k) {
    const uint64_t b = (k >> 63) ? (k & 0x7fffffffffffffffull) : ~k;
    return __longlong_as_double((long long)b);
}

// (key desc, doc asc) is the ranking; `better` is strict.
__device__ __forceinline__ bool better(uint64_t ka, uint32_t da, uint64_t kb, uint32_t db) {
    return ka > kb || (ka == kb && da < db);
}

// ---------------------------------------------------------- index prep
// skips[t][r] = first posting of term t whose doc is >= r * BM_RANGE.
__global__ void bm25_skips_kernel(const int64_t* __restrict__ term_ptr,
                                  const int32_t* __restrict__ post_doc, int64_t n_terms,
                                  int n_ranges, int32_t* __restrict__ skips) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_terms * (n_ranges + 1)) return;
    const int64_t t = i / (n_ranges + 1);
    const int r = (int)(i % (n_ranges + 1));
    const int64_t target = (int64_t)r * BM_RANGE;
    int64_t lo = term_ptr[t], hi = term_ptr[t + 1];   // first p in [lo, hi) with doc >= target
    while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if (post_doc[mid] < target) lo = mid + 1; else hi = mid;
    }
    skips[i] = (int32_t)lo;
}

// impact[p] = idf * (tf * (k1 + 1.0)) / (tf + k1 * (1.0 - b + b * dl / avg_dl)),
// the amount :186 adds to document post_doc[p] for term t, with the
// reference's operation order.  It depends on (term, document) and corpus
// statistics only (the query's own term frequency is not used), so it is
// computed once per index.  One block per term.
__global__ void bm25_impact_kernel(const int64_t* __restrict__ term_ptr,
                                   const int32_t* __restrict__ post_doc,
                                   const uint16_t* __restrict__ post_tf,
                                   const int32_t* __restrict__ doc_len, int64_t n_docs,
                                   const double* __restrict__ idf, double avg_dl,
                                   double* __restrict__ impact, int* status) {
    const int64_t t = blockIdx.x;
    const double w = idf[t];
    const double k1p1 = BM_K1 + 1.0;
    for (int64_t p = term_ptr[t] + threadIdx.x; p < term_ptr[t + 1]; p += blockDim.x) {
        const int32_t d = post_doc[p];
        if (d < 0 || d >= n_docs) {
            atomicOr(status, 1);
            impact[p] = 0.0;
            continue;
        }
        const double tf = (double)post_tf[p];
        const double dl = (double)doc_len[d];
        const double x = __dadd_rn(1.0 - BM_B, __ddiv_rn(__dmul_rn(BM_B, dl), avg_dl));
        const double den = __dadd_rn(tf, __dmul_rn(BM_K1, x));
        impact[p] = __ddiv_rn(__dmul_rn(w, __dmul_rn(tf, k1p1)), den);
    }
}

// ------------------------------------------------------------- scoring
struct BmArgs {
    const int32_t* post_doc;
    const double* impact;     // [n_postings]
    const int32_t* skips;     // [n_terms][n_ranges + 1]
    const int32_t* qterms;    // [nq][qlen]
    int64_t n_terms;
    int64_t n_docs;
    int n_ranges;
    int qlen;
    int k;
    uint64_t* cand_key;       // [nq][n_ranges][k]
    int32_t* cand_doc;
};

constexpr int BM_PER_THREAD = BM_RANGE / BM_THREADS;   // 16 contiguous docs per thread

// Bitonic sort, descending by (key, then lower index), of n (power of two)
// pairs in shared memory.
__device__ __forceinline__ void sort_pairs_desc(uint64_t* key, int32_t* idx, int n) {
    for (int size = 2; size <= n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            __syncthreads();
            for (int i = threadIdx.x; i < n / 2; i += blockDim.x) {
                const int lo = 2 * i - (i & (stride - 1));
                const int hi = lo + stride;
                const bool desc = ((lo & size) == 0);
                const bool hi_better =
                    better(key[hi], (uint32_t)idx[hi], key[lo], (uint32_t)idx[lo]);
                if (hi_better == desc) {
                    const uint64_t tk = key[lo]; key[lo] = key[hi]; key[hi] = tk;
                    const int32_t ti = idx[lo]; idx[lo] = idx[hi]; idx[hi] = ti;
                }
            }
        }
    }
    __syncthreads();
}

// 5 CTAs per SM: the extra latency hiding outweighs a few spilled registers
__global__ void __launch_bounds__(BM_THREADS, 5) bm25_range_kernel(const BmArgs a) {
    // fp64 scores of the range; reused as the candidate scratch afterwards
    __shared__ __align__(16) unsigned char arena[BM_RANGE * sizeof(double)];
    __shared__ uint64_t tmax[BM_THREADS];
    __shared__ unsigned tie_cnt[BM_PER_THREAD * (BM_THREADS / 32)];
    __shared__ int32_t terms[BM_MAX_QLEN];
    __shared__ int span[BM_MAX_QLEN][2];
    __shared__ int n_terms_q;
    __shared__ unsigned wt[8];
    __shared__ uint64_t tau_s;
    double* sc = reinterpret_cast<double*>(arena);
    // queries vary fastest across the grid, so the blocks in flight share one
    // doc range and its slice of the index stays in L2 across queries
    const int q = blockIdx.x, r = blockIdx.y;
    const int64_t d0 = (int64_t)r * BM_RANGE;
    const int nd = (int)min((int64_t)BM_RANGE, a.n_docs - d0);

    for (int i = threadIdx.x; i < BM_RANGE; i += BM_THREADS) sc[i] = 0.0;
    __shared__ int32_t raw[BM_MAX_QLEN];
    if (threadIdx.x < a.qlen) raw[threadIdx.x] = __ldg(a.qterms + (int64_t)q * a.qlen + threadIdx.x);
    __syncthreads();
    if (threadIdx.x == 0) {
        // the query's distinct in-vocabulary terms, ascending
        int n = 0;
        for (int i = 0; i < a.qlen; ++i) {
            const int32_t t = raw[i];
            if (t < 0 || t >= a.n_terms) continue;
            int j = n;
            while (j > 0 && terms[j - 1] > t) { terms[j] = terms[j - 1]; --j; }
            if (j > 0 && terms[j - 1] == t) {          // duplicate: undo the shift
                for (int m = j; m < n; ++m) terms[m] = terms[m + 1];
                continue;
            }
            terms[j] = t;
            ++n;
        }
        n_terms_q = n;
    }
    __syncthreads();
    // every term's posting span in this range, loaded in parallel
    if (threadIdx.x < 2 * n_terms_q) {
        const int i = threadIdx.x >> 1, e = threadIdx.x & 1;
        span[i][e] = __ldg(a.skips + (int64_t)terms[i] * (a.n_ranges + 1) + r + e);
    }
    __syncthreads();

    constexpr int U = 8;   // postings in flight per thread
    for (int i = 0; i < n_terms_q; ++i) {
        const int p0 = span[i][0], p1 = span[i][1];
        for (int pb = p0 + threadIdx.x; pb < p1; pb += BM_THREADS * U) {
            int li[U];
            double w[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int p = pb + u * BM_THREADS;
                li[u] = p < p1 ? __ldg(a.post_doc + p) - (int)d0 : -1;
                w[u] = p < p1 ? __ldg(a.impact + p) : 0.0;
            }
#pragma unroll
            for (int u = 0; u < U; ++u)
                if ((unsigned)li[u] < (unsigned)nd)   // (also drops postings outside the range)
                    sc[li[u]] = __dadd_rn(sc[li[u]], w[u]);
        }
        __syncthreads();   // the next term adds to the same documents
    }

    // ---- top-k of the range.  Thread t owns docs t + 256 j (j < 16), so the
    // reads below are conflict-free and doc order is (j, t); key 0 marks a
    // slot past the range (every real score has a key >= 2^63).
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint64_t key[BM_PER_THREAD];
    uint64_t mx = 0ull;
#pragma unroll
    for (int j = 0; j < BM_PER_THREAD; ++j) {
        const int i = threadIdx.x + BM_THREADS * j;
        key[j] = i < nd ? f64_key(sc[i]) : 0ull;
        mx = key[j] > mx ? key[j] : mx;
    }
    // tau = the k-th largest of the thread maxima: at least k documents have a
    // key >= tau, and only the (fewer than k) threads whose maximum exceeds tau
    // hold documents above it, so at most 16 (k - 1) documents do.  Each warp
    // sorts its 32 maxima with shuffles; warp 0 merges the 8 sorted lists.
#pragma unroll
    for (int size = 2; size <= 32; size <<= 1)
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            const uint64_t o = __shfl_xor_sync(0xffffffffu, mx, stride);
            const bool keep_max = ((lane & stride) == 0) == ((lane & size) == 0);
            mx = keep_max ? (o > mx ? o : mx) : (o < mx ? o : mx);
        }
    tmax[warp * 32 + lane] = mx;   // warp w's maxima, descending
    __syncthreads();               // also: every read of the scores is done
    const int kk = min(a.k, nd);
    if (kk <= 32) {
        // merge tree: pairs of descending lists -> the top 32 of their union
        // (the larger of a[l] and b[31 - l] is a bitonic sequence holding it),
        // sorted again with shuffles; three rounds leave the top 32 in list 0
        for (int span_w = 1; span_w < 8; span_w <<= 1) {
            uint64_t v = 0ull;
            const bool act = (warp % (2 * span_w)) == 0;
            if (act) {
                const uint64_t x = tmax[warp * 32 + lane];
                const uint64_t y = tmax[(warp + span_w) * 32 + (31 - lane)];
                v = x > y ? x : y;
#pragma unroll
                for (int stride = 16; stride > 0; stride >>= 1) {
                    const uint64_t o = __shfl_xor_sync(0xffffffffu, v, stride);
                    const bool keep_max = (lane & stride) == 0;
                    v = keep_max ? (o > v ? o : v) : (o < v ? o : v);
                }
            }
            __syncthreads();
            if (act) tmax[warp * 32 + lane] = v;
            __syncthreads();
        }
        if (threadIdx.x == 0) tau_s = kk > 0 ? tmax[kk - 1] : 0ull;
    } else if (warp == 0) {
        // larger k: warp 0 merges the 8 sorted lists one element at a time
        int ptr = 0;
        uint64_t head = lane < 8 ? tmax[lane * 32] : 0ull, t = 0ull;
        for (int i = 0; i < kk; ++i) {
            uint64_t best = head;
            int bl = lane;
#pragma unroll
            for (int o = 4; o > 0; o >>= 1) {   // lanes 0-7 form their own group
                const uint64_t ob = __shfl_xor_sync(0xffffffffu, best, o);
                const int obl = __shfl_xor_sync(0xffffffffu, bl, o);
                if (ob > best || (ob == best && obl < bl)) { best = ob; bl = obl; }
            }
            t = __shfl_sync(0xffffffffu, best, 0);
            const int win = __shfl_sync(0xffffffffu, bl, 0);
            if (lane == win) {
                ++ptr;
                head = ptr < 32 ? tmax[lane * 32 + ptr] : 0ull;
            }
        }
        if (lane == 0) tau_s = t;
    }
    __syncthreads();
    const uint64_t tau = tau_s;
    // candidates: the documents at or above tau (at least kk of them).  When
    // there are few, ranking them by (key desc, doc asc) settles ties at tau
    // too; otherwise only those above tau are candidates and the ties at tau
    // are filled in document order below.
    unsigned g = 0;
#pragma unroll
    for (int j = 0; j < BM_PER_THREAD; ++j) g += key[j] >= tau && key[j] != 0ull;
    unsigned g_incl = block_scan_incl_256(g, wt);
    unsigned G = wt[7];
    const bool with_ties = G <= BM_THREADS;
    if (!with_ties) {
        __syncthreads();   // every read of wt[7] is done before the scan reuses it
        g = 0;
#pragma unroll
        for (int j = 0; j < BM_PER_THREAD; ++j) g += key[j] > tau;
        g_incl = block_scan_incl_256(g, wt);
        G = wt[7];
    }
    uint64_t* ck = reinterpret_cast<uint64_t*>(arena);
    int32_t* cdoc = reinterpret_cast<int32_t*>(arena + 2048 * sizeof(uint64_t));
    {
        unsigned pos = g_incl - g;
#pragma unroll
        for (int j = 0; j < BM_PER_THREAD; ++j)
            if (with_ties ? (key[j] >= tau && key[j] != 0ull) : key[j] > tau) {
                ck[pos] = key[j];
                cdoc[pos] = threadIdx.x + BM_THREADS * j;
                ++pos;
            }
    }
    __syncthreads();
    uint64_t* ok = a.cand_key + ((int64_t)q * a.n_ranges + r) * a.k;
    int32_t* od = a.cand_doc + ((int64_t)q * a.n_ranges + r) * a.k;
    if ((int)G <= kk) {
        // all of them (the merge orders candidates)
        for (int i = threadIdx.x; i < (int)G; i += BM_THREADS) {
            ok[i] = ck[i];
            od[i] = (int32_t)(d0 + cdoc[i]);
        }
    } else if (G <= BM_THREADS) {
        // rank each candidate against the others; ranks < k are the top-k
        if (threadIdx.x < G) {
            const uint64_t mk = ck[threadIdx.x];
            const uint32_t md = (uint32_t)cdoc[threadIdx.x];
            int rank = 0;
            for (int j = 0; j < (int)G; ++j) rank += better(ck[j], (uint32_t)cdoc[j], mk, md);
            if (rank < kk) {
                ok[rank] = mk;
                od[rank] = (int32_t)(d0 + md);
            }
        }
    } else {
        const int n2 = next_pow2((int)G);
        for (int i = (int)G + threadIdx.x; i < n2; i += BM_THREADS) {
            ck[i] = 0ull;
            cdoc[i] = 0x7fffffff;
        }
        sort_pairs_desc(ck, cdoc, n2);
        for (int i = threadIdx.x; i < kk; i += BM_THREADS) {
            ok[i] = ck[i];
            od[i] = (int32_t)(d0 + cdoc[i]);
        }
    }
    if (!with_ties && (int)G < kk) {
        // the rest from the documents tied at tau, lowest doc first: rank =
        // ties in earlier rows + ties earlier in this row (warp ballots)
        unsigned* cnt = tie_cnt;   // [16 rows][8 warps]
        unsigned m[BM_PER_THREAD];
#pragma unroll
        for (int j = 0; j < BM_PER_THREAD; ++j) {
            m[j] = __ballot_sync(0xffffffffu, key[j] == tau && key[j] != 0ull);
            if (lane == 0) cnt[j * (BM_THREADS / 32) + warp] = __popc(m[j]);
        }
        __syncthreads();
        unsigned before = 0;
#pragma unroll
        for (int j = 0; j < BM_PER_THREAD; ++j) {
            unsigned row_before = 0, row_total = 0;
            for (int w = 0; w < BM_THREADS / 32; ++w) {
                const unsigned c = cnt[j * (BM_THREADS / 32) + w];
                row_total += c;
                if (w < warp) row_before += c;
            }
            if ((m[j] >> lane) & 1u) {
                const unsigned rank = G + before + row_before + __popc(m[j] & ((1u << lane) - 1u));
                if (rank < (unsigned)kk) {
                    ok[rank] = tau;
                    od[rank] = (int32_t)(d0 + threadIdx.x + BM_THREADS * j);
                }
            }
            before += row_total;
        }
    }
    for (int i = kk + threadIdx.x; i < a.k; i += BM_THREADS) { ok[i] = 0ull; od[i] = -1; }
}

// Per query: the best k of the ranges' candidates (key desc, doc asc).
__global__ void __launch_bounds__(BM_THREADS) bm25_merge_kernel(const uint64_t* __restrict__ ck,
                                                                const int32_t* __restrict__ cd,
                                                                int n_cand, int k,
                                                                int32_t* __restrict__ out_idx,
                                                                double* __restrict__ out_scores) {
    extern __shared__ unsigned char msm[];
    const int n2 = next_pow2(n_cand);
    uint64_t* key = reinterpret_cast<uint64_t*>(msm);
    int32_t* doc = reinterpret_cast<int32_t*>(key + n2);
    const int q = blockIdx.x;
    for (int i = threadIdx.x; i < n2; i += BM_THREADS) {
        const bool in = i < n_cand && cd[(int64_t)q * n_cand + i] >= 0;
        key[i] = in ? ck[(int64_t)q * n_cand + i] : 0ull;
        doc[i] = in ? cd[(int64_t)q * n_cand + i] : 0x7fffffff;
    }
    sort_pairs_desc(key, doc, n2);
    for (int j = threadIdx.x; j < k; j += BM_THREADS) {
        const bool ok = j < n2 && key[j] != 0ull;
        out_idx[(int64_t)q * k + j] = ok ? doc[j] : -1;
        if (out_scores) out_scores[(int64_t)q * k + j] = ok ? key_to_f64(key[j]) : 0.0;
    }
}

int bm25_ranges(int64_t n_docs) { return (int)((n_docs + BM_RANGE - 1) / BM_RANGE); }

}  // namespace
}  // namespace hmm

using namespace hmm;

extern "C" hmm_status_t hmm_bm25_stats_host(const int64_t* term_ptr, int64_t n_terms,
                                            const int32_t* doc_len, int64_t n_docs, double* idf,
                                            double* avg_dl) {
    HMM_REQUIRE(n_terms >= 0 && n_docs >= 0, "negative sizes");
    HMM_REQUIRE((term_ptr || n_terms == 0) && (doc_len || n_docs == 0), "null input");
    HMM_REQUIRE((idf || n_terms == 0) && avg_dl, "null output");
    const double N = (double)n_docs;
    for (int64_t t = 0; t < n_terms; ++t) {
        const double df = (double)(term_ptr[t + 1] - term_ptr[t]);
        idf[t] = df > 0 ? std::log((N - df + 0.5) / (df + 0.5) + 1.0) : 0.0;
    }
    double s = 0.0;
    for (int64_t d = 0; d < n_docs; ++d) s += (double)doc_len[d];
    *avg_dl = n_docs ? s / N : 0.0;
    return HMM_OK;
}

extern "C" size_t hmm_bm25_skips_count(int64_t n_terms, int64_t n_docs) {
    if (n_terms < 0 || n_docs < 0) return 0;
    return (size_t)n_terms * (size_t)(bm25_ranges(n_docs) + 1);
}

extern "C" hmm_status_t hmm_bm25_prepare(const int64_t* term_ptr, const int32_t* post_doc,
                                         const uint16_t* post_tf, int64_t n_terms,
                                         const int32_t* doc_len, int64_t n_docs,
                                         const double* idf, double avg_dl, int32_t* skips,
                                         double* impact, void* workspace, size_t workspace_bytes,
                                         void* stream) {
    HMM_REQUIRE(n_terms >= 0 && n_docs >= 0 && n_docs < (int64_t(1) << 31), "bad sizes");
    HMM_REQUIRE(n_terms <= 2147483647, "too many terms");
    HMM_REQUIRE(workspace && workspace_bytes >= 256, "workspace must hold >= 256 bytes");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int nr = bm25_ranges(n_docs);
    const int64_t ns = n_terms * (int64_t)(nr + 1);
    if (ns == 0) return HMM_OK;
    HMM_REQUIRE(term_ptr && skips && idf && impact, "null pointer");
    HMM_REQUIRE(n_docs == 0 || (post_doc && post_tf && doc_len), "null pointer");
    int* status = static_cast<int*>(workspace);
    HMM_CUDA_TRY(cudaMemsetAsync(status, 0, sizeof(int), st));
    bm25_skips_kernel<<<(unsigned)((ns + 255) / 256), 256, 0, st>>>(term_ptr, post_doc, n_terms,
                                                                   nr, skips);
    hmm_status_t s = check_launch("bm25_skips_kernel");
    if (s != HMM_OK) return s;
    bm25_impact_kernel<<<(unsigned)n_terms, 256, 0, st>>>(term_ptr, post_doc, post_tf, doc_len,
                                                          n_docs, idf, avg_dl, impact, status);
    s = check_launch("bm25_impact_kernel");
    if (s != HMM_OK) return s;
    int h = 0;
    HMM_CUDA_TRY(cudaMemcpyAsync(&h, status, sizeof(int), cudaMemcpyDeviceToHost, st));
    HMM_CUDA_TRY(cudaStreamSynchronize(st));
    if (h) return set_error(HMM_ERR_BOUNDS, "hmm_bm25_prepare: a posting's doc id is outside [0, n_docs)");
    return HMM_OK;
}

extern "C" size_t hmm_bm25_topk_workspace_size(int64_t n_docs, int64_t n_queries, int64_t k) {
    if (n_docs < 0 || n_queries < 0 || k < 1) return 0;
    const size_t n = (size_t)n_queries * bm25_ranges(n_docs) * (size_t)k;
    return ((n * 8 + 255) & ~size_t(255)) + n * 4 + 256;
}

extern "C" hmm_status_t hmm_bm25_topk_csr(const int32_t* post_doc, const double* impact,
                                          int64_t n_postings, int64_t n_terms, int64_t n_docs,
                                          const int32_t* skips, const int32_t* qterms,
                                          int64_t n_queries, int64_t qlen, int64_t k,
                                          int32_t* out_idx, double* out_scores, void* workspace,
                                          size_t workspace_bytes, void* stream) {
    HMM_REQUIRE(n_terms >= 0 && n_docs >= 0 && n_docs < (int64_t(1) << 31), "bad sizes");
    HMM_REQUIRE(n_postings >= 0 && n_postings < (int64_t(1) << 31),
                "n_postings must be < 2^31 (int32 skips)");
    HMM_REQUIRE(n_queries >= 0 && n_queries <= 2147483647, "n_queries out of range");
    HMM_REQUIRE(n_docs <= (int64_t)65535 * BM_RANGE, "n_docs must be <= %lld",
                (long long)65535 * BM_RANGE);
    HMM_REQUIRE(qlen >= 0 && qlen <= BM_MAX_QLEN, "qlen must be in [0, %d]", BM_MAX_QLEN);
    HMM_REQUIRE(k >= 1 && k <= BM_KMAX, "k must be in [1, %d]", BM_KMAX);
    if (n_queries == 0) return HMM_OK;
    HMM_REQUIRE(out_idx, "out_idx is null");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (n_docs == 0) {   // the reference returns an empty index (:148-151)
        HMM_CUDA_TRY(cudaMemsetAsync(out_idx, 0xff, sizeof(int32_t) * n_queries * k, st));
        if (out_scores)
            HMM_CUDA_TRY(cudaMemsetAsync(out_scores, 0, sizeof(double) * n_queries * k, st));
        return HMM_OK;
    }
    HMM_REQUIRE((qterms || qlen == 0) && (n_terms == 0 || skips), "null input pointer");
    HMM_REQUIRE(n_postings == 0 || (post_doc && impact), "null postings");
    const int nr = bm25_ranges(n_docs);
    const int n_cand = nr * (int)k;
    const size_t msm = (size_t)next_pow2(n_cand) * 12;
    if (msm > 200 * 1024)
        return set_error(HMM_ERR_UNSUPPORTED,
                         "ceil(n_docs / %d) * k = %d range candidates per query; at most 16384",
                         BM_RANGE, n_cand);
    const size_t need = hmm_bm25_topk_workspace_size(n_docs, n_queries, k);
    if (!workspace || workspace_bytes < need)
        return set_error(HMM_ERR_OOM, "workspace too small: %zu < %zu", workspace_bytes, need);
    const size_t n = (size_t)n_queries * nr * (size_t)k;
    unsigned char* w = static_cast<unsigned char*>(workspace);
    BmArgs a;
    a.post_doc = post_doc;
    a.impact = impact;
    a.skips = skips;
    a.qterms = qterms;
    a.n_terms = n_terms;
    a.n_docs = n_docs;
    a.n_ranges = nr;
    a.qlen = (int)qlen;
    a.k = (int)k;
    a.cand_key = reinterpret_cast<uint64_t*>(w);
    a.cand_doc = reinterpret_cast<int32_t*>(w + ((n * 8 + 255) & ~size_t(255)));
    const ProfileMark pm = profile_begin(st);
    bm25_range_kernel<<<dim3((unsigned)n_queries, (unsigned)nr), BM_THREADS, 0, st>>>(a);
    hmm_status_t s = check_launch("bm25_range_kernel");
    profile_end(pm, st);
    if (s != HMM_OK) return s;
    HMM_CUDA_TRY(cudaFuncSetAttribute(bm25_merge_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)msm));
    bm25_merge_kernel<<<(unsigned)n_queries, BM_THREADS, msm, st>>>(
        a.cand_key, a.cand_doc, n_cand, (int)k, out_idx, out_scores);
    return check_launch("bm25_merge_kernel");
}
