// packed.h — the GPU work of the step adapters on contiguous row-major host
// arrays: what an adapter has after packing a vector-of-vectors, and what the
// Python bindings (src/py) already hold as NumPy arrays, so they skip the
// packing copies.  Synchronous, on the legacy default stream, per-thread
// device scratch (device.h); failures throw std::runtime_error.
#ifndef HETEROMM_B200_SRC_PACKED_H_
#define HETEROMM_B200_SRC_PACKED_H_

#include <cstddef>
#include <cstdint>
#include <vector>

namespace heteromm {
namespace gpu {

// n fp32 inner products of rows[n][d] with q[d], index order (zeros if n or d is 0).
std::vector<float> ip_scores(const float* rows, size_t n, size_t d, const float* q);

// Indices of the min(k, n) best inner products, best first, ties to the lowest
// index (0, 1, ... if d is 0: every score is 0).
std::vector<int> ip_topk(const float* rows, size_t n, size_t d, const float* q, size_t k);

// The same two with the rows already on the device (n, d > 0).
std::vector<float> ip_scores_dev(const float* d_rows, size_t n, size_t d, const float* q);
std::vector<int> ip_topk_dev(const float* d_rows, size_t n, size_t d, const float* q, size_t k);

// Page summaries [ceil(L/page)][out_dim] (flat) of keys[L][D] projected by
// weight[out_dim][D]; the caller has checked L, D, out_dim and page > 0.
std::vector<float> paged_summary(const float* keys, size_t L, size_t D, const float* weight,
                                 size_t out_dim, int page);

// The same with the keys on the device; the summaries stay on the device
// (this thread's output scratch, valid until its next GPU call) and the
// returned pointer addresses them.
const float* paged_summary_dev(const float* d_keys, size_t L, size_t D, const float* weight,
                               size_t out_dim, int page);

// Attention output [D] of q over the tokens of the selected blocks of `page`
// tokens of keys/values [L][D]; the caller has checked L, D, nb and page > 0.
std::vector<float> block_sparse_attention(const float* keys, const float* values, size_t L,
                                          size_t D, const float* q, const int* blocks, size_t nb,
                                          size_t page);

// The same with keys, values and the block ids on the device.
std::vector<float> block_sparse_attention_dev(const float* d_keys, const float* d_values,
                                              size_t L, size_t D, const float* q,
                                              const int32_t* d_blocks, size_t nb, size_t page);

}  // namespace gpu
}  // namespace heteromm

#endif  // HETEROMM_B200_SRC_PACKED_H_
