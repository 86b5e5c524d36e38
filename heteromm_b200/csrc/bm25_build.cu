// bm25_build.cu — the BM25 inverted index built on the GPU from per-document
// term counts: the layout of the reference's term_freq.bin export
// (toolchain/rag_test/export_bm25_data.py:13-27, 230-263: for each document its
// (vocab index, count) pairs) and of BM25IndexMemory's per-document maps
// (types/memory.h:232-301), transposed into the term-major CSR the BM25
// kernels read: term_ptr [V+1], post_doc (ascending within each term),
// post_tf, plus doc_len (sum of the document's counts, the reference's dl,
// bm25_fpga_retrieval.cpp:158-169).
//
// The transpose is a two-level counting sort that keeps document order:
//   1. per chunk of BC documents, a histogram of its terms;
//   2. per term, an exclusive scan down the chunks (where each chunk's
//      postings of the term start), and the term totals;
//   3. term_ptr = exclusive scan of the totals;
//   4. per chunk, one warp walks its documents in order and writes each
//      (document, count) to term_ptr[t] + the chunk's running slot of t.
// Within a document every term occurs at most once (term_freq.bin stores a
// map per document), so the lanes of one document never share a slot.
#include <cuda_runtime.h>

#include <cstdint>

#include "heteromm_cuda.h"
#include "hmm_common.cuh"

namespace hmm {
namespace {

constexpr int BC = 1024;   // documents per chunk

__global__ void bm25_doclen_kernel(const int64_t* __restrict__ doc_ptr,
                                   const int32_t* __restrict__ terms,
                                   const uint32_t* __restrict__ counts, int64_t n_docs,
                                   int64_t n_terms, int32_t* __restrict__ doc_len,
                                   int* __restrict__ status) {
    const int lane = threadIdx.x & 31;
    const int64_t d = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (d >= n_docs) return;
    const int64_t e0 = doc_ptr[d], e1 = doc_ptr[d + 1];
    if (e1 < e0 || (d == 0 && e0 < 0)) {
        if (lane == 0) atomicOr(&status[0], 4);
        return;
    }
    unsigned long long sum = 0;
    int bad = 0;
    for (int64_t e = e0 + lane; e < e1; e += 32) {
        const int32_t t = terms[e];
        const uint32_t c = counts[e];
        bad |= (t < 0 || t >= n_terms) ? 1 : 0;
        bad |= (c == 0u || c > 65535u) ? 2 : 0;
        sum += c;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        sum += __shfl_xor_sync(0xffffffffu, sum, o);
        bad |= __shfl_xor_sync(0xffffffffu, bad, o);
    }
    if (lane == 0) {
        if (sum > 0x7fffffffull) bad |= 8;
        if (bad) atomicOr(&status[0], bad);
        doc_len[d] = (int32_t)(sum > 0x7fffffffull ? 0x7fffffffull : sum);
    }
}

// hist [n_chunks][n_terms]: postings of term t in chunk c
__global__ void bm25_chunk_hist_kernel(const int64_t* __restrict__ doc_ptr,
                                       const int32_t* __restrict__ terms, int64_t n_docs,
                                       int64_t n_terms, int32_t* __restrict__ hist) {
    const int64_t c = blockIdx.x;
    const int64_t d0 = c * BC, d1 = min(n_docs, d0 + BC);
    const int64_t e0 = doc_ptr[d0], e1 = doc_ptr[d1];
    int32_t* h = hist + c * n_terms;
    for (int64_t e = e0 + threadIdx.x; e < e1; e += blockDim.x) {
        const int32_t t = terms[e];
        if (t >= 0 && t < n_terms) atomicAdd(&h[t], 1);
    }
}

// per term: hist column -> exclusive running offsets, and the total
__global__ void bm25_col_scan_kernel(int32_t* __restrict__ hist, int64_t n_chunks,
                                     int64_t n_terms, int64_t* __restrict__ total) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n_terms) return;
    int64_t run = 0;
    for (int64_t c = 0; c < n_chunks; ++c) {
        const int32_t v = hist[c * n_terms + t];
        hist[c * n_terms + t] = (int32_t)run;
        run += v;
    }
    total[t] = run;
}

// term_ptr[0..V]: exclusive scan of the totals (one block of 1024 threads)
__global__ void __launch_bounds__(1024) bm25_term_ptr_kernel(const int64_t* __restrict__ total,
                                                             int64_t n_terms,
                                                             int64_t* __restrict__ term_ptr) {
    __shared__ int64_t warp_sum[32];
    __shared__ int64_t carry;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int64_t base = 0; base < n_terms; base += 1024) {
        const int64_t i = base + threadIdx.x;
        const int64_t v = i < n_terms ? total[i] : 0;
        int64_t incl = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int64_t u = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += u;
        }
        if (lane == 31) warp_sum[w] = incl;
        __syncthreads();
        if (w == 0) {
            int64_t s = warp_sum[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int64_t u = __shfl_up_sync(0xffffffffu, s, o);
                if (lane >= o) s += u;
            }
            warp_sum[lane] = s;
        }
        __syncthreads();
        const int64_t excl = carry + incl - v + (w > 0 ? warp_sum[w - 1] : 0);
        if (i < n_terms) term_ptr[i] = excl;
        __syncthreads();
        if (threadIdx.x == 1023) carry = excl + v;
        __syncthreads();
    }
    if (threadIdx.x == 0) term_ptr[n_terms] = carry;
}

// one warp per chunk, documents in order
__global__ void bm25_scatter_kernel(const int64_t* __restrict__ doc_ptr,
                                    const int32_t* __restrict__ terms,
                                    const uint32_t* __restrict__ counts, int64_t n_docs,
                                    int64_t n_terms, int64_t n_chunks, int32_t* __restrict__ hist,
                                    const int64_t* __restrict__ term_ptr,
                                    int32_t* __restrict__ post_doc, uint16_t* __restrict__ post_tf) {
    const int lane = threadIdx.x & 31;
    const int64_t c = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (c >= n_chunks) return;
    int32_t* h = hist + c * n_terms;
    const int64_t d0 = c * BC, d1 = min(n_docs, d0 + BC);
    for (int64_t d = d0; d < d1; ++d) {
        const int64_t e0 = doc_ptr[d], e1 = doc_ptr[d + 1];
        for (int64_t e = e0 + lane; e < e1; e += 32) {
            const int32_t t = terms[e];
            if (t < 0 || t >= n_terms) continue;   // reported by bm25_doclen_kernel
            const int32_t slot = h[t];
            h[t] = slot + 1;   // the term occurs once in this document
            const int64_t p = term_ptr[t] + slot;
            post_doc[p] = (int32_t)d;
            post_tf[p] = (uint16_t)min(counts[e], 65535u);
        }
        __syncwarp();   // this document's slot updates before the next document's reads
    }
}

size_t up256(size_t v) { return (v + 255) & ~size_t(255); }

}  // namespace
}  // namespace hmm

using namespace hmm;

extern "C" size_t hmm_bm25_csr_workspace_size(int64_t n_docs, int64_t n_terms) {
    if (n_docs < 0 || n_terms < 0) return 0;
    const int64_t n_chunks = (n_docs + BC - 1) / BC;
    return up256(sizeof(int32_t) * (size_t)n_chunks * (size_t)n_terms) +
           up256(sizeof(int64_t) * (size_t)(n_terms + 1)) + 256;
}

extern "C" hmm_status_t hmm_bm25_csr_from_docs(const int64_t* doc_ptr, const int32_t* terms,
                                               const uint32_t* counts, int64_t n_docs,
                                               int64_t n_terms, int64_t* term_ptr,
                                               int32_t* post_doc, uint16_t* post_tf,
                                               int32_t* doc_len, void* workspace,
                                               size_t workspace_bytes, void* stream) {
    HMM_REQUIRE(n_docs >= 0 && n_docs < (int64_t(1) << 31), "n_docs out of range");
    HMM_REQUIRE(n_terms >= 1 && n_terms < (int64_t(1) << 31), "n_terms out of range");
    HMM_REQUIRE(doc_ptr && term_ptr && (n_docs == 0 || doc_len), "null pointer");
    const size_t need = hmm_bm25_csr_workspace_size(n_docs, n_terms);
    if (!workspace || workspace_bytes < need)
        return set_error(HMM_ERR_OOM, "workspace too small: %zu < %zu", workspace_bytes, need);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int64_t n_chunks = (n_docs + BC - 1) / BC;
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    int32_t* hist = reinterpret_cast<int32_t*>(ws);
    int64_t* total = reinterpret_cast<int64_t*>(ws + up256(sizeof(int32_t) * (size_t)n_chunks *
                                                            (size_t)n_terms));
    int* status = reinterpret_cast<int*>(reinterpret_cast<unsigned char*>(total) +
                                         up256(sizeof(int64_t) * (size_t)(n_terms + 1)));
    HMM_CUDA_TRY(cudaMemsetAsync(status, 0, sizeof(int), st));
    HMM_CUDA_TRY(cudaMemsetAsync(hist, 0, sizeof(int32_t) * (size_t)n_chunks * (size_t)n_terms, st));
    hmm_status_t s = HMM_OK;
    if (n_docs > 0) {
        HMM_REQUIRE(terms && counts && post_doc && post_tf, "null pointer");
        bm25_doclen_kernel<<<(unsigned)((n_docs + 7) / 8), 256, 0, st>>>(
            doc_ptr, terms, counts, n_docs, n_terms, doc_len, status);
        if ((s = check_launch("bm25_doclen_kernel")) != HMM_OK) return s;
        int h = 0;
        HMM_CUDA_TRY(cudaMemcpyAsync(&h, status, sizeof(int), cudaMemcpyDeviceToHost, st));
        HMM_CUDA_TRY(cudaStreamSynchronize(st));
        if (h & 4) return set_error(HMM_ERR_INVALID, "doc_ptr must start at >= 0 and not decrease");
        if (h & 1) return set_error(HMM_ERR_BOUNDS, "a term index is outside [0, n_terms)");
        if (h & 2) return set_error(HMM_ERR_INVALID, "term counts must be in [1, 65535]");
        if (h & 8) return set_error(HMM_ERR_INVALID, "a document length exceeds 2^31 - 1");
        bm25_chunk_hist_kernel<<<(unsigned)n_chunks, 256, 0, st>>>(doc_ptr, terms, n_docs, n_terms,
                                                                   hist);
        if ((s = check_launch("bm25_chunk_hist_kernel")) != HMM_OK) return s;
    }
    bm25_col_scan_kernel<<<(unsigned)((n_terms + 255) / 256), 256, 0, st>>>(hist, n_chunks, n_terms,
                                                                            total);
    if ((s = check_launch("bm25_col_scan_kernel")) != HMM_OK) return s;
    bm25_term_ptr_kernel<<<1, 1024, 0, st>>>(total, n_terms, term_ptr);
    if ((s = check_launch("bm25_term_ptr_kernel")) != HMM_OK) return s;
    if (n_docs > 0) {
        bm25_scatter_kernel<<<(unsigned)((n_chunks + 7) / 8), 256, 0, st>>>(
            doc_ptr, terms, counts, n_docs, n_terms, n_chunks, hist, term_ptr, post_doc, post_tf);
        if ((s = check_launch("bm25_scatter_kernel")) != HMM_OK) return s;
    }
    return HMM_OK;
}
