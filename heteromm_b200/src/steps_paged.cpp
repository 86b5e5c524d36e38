// steps_paged.cpp — PagedKVIndexBuilder and BlockSparseAttention: CPU bodies
// (the reference's arithmetic, steps/example_kernel/paged_kv_index_builder.cpp:18-85
// and block_sparse_attention.cpp:21-126) and GPU adapters onto
// hmm_paged_kv_summary_f32 / hmm_block_sparse_attention_f32, reading the KV
// cache through the per-thread device mirrors (device.h).
#include <algorithm>
#include <cmath>
#include <iostream>

#include "device.h"
#include "packed.h"
#include "heteromm/dev/steps/apply_memory.h"
#include "heteromm/dev/steps/build_memory.h"

namespace heteromm {
namespace step {

namespace {
void fpga_stub(const char* step) {
    std::clog << "[" << step << "] FPGA kernel not implemented. exiting." << std::endl;
}

// The checks that make the builder return an empty memory (:30-44).
bool builder_input_ok(const std::vector<std::vector<float>>& keys,
                      const std::vector<std::vector<float>>& weight, int page_size) {
    const size_t L = keys.size(), D = keys.empty() ? 0 : keys[0].size();
    if (L == 0 || D == 0) {
        std::clog << "[PagedKVIndexBuilder] Warning: Empty KV cache data." << std::endl;
        return false;
    }
    if (weight.empty() || weight[0].size() != D) {
        std::clog << "[PagedKVIndexBuilder] Warning: Weight matrix dimension mismatch." << std::endl;
        return false;
    }
    if (page_size <= 0) {
        std::clog << "[PagedKVIndexBuilder] Warning: page_size must be positive." << std::endl;
        return false;
    }
    return true;
}
}  // namespace

// ------------------------------------------------------- PagedKVIndexBuilder
void PagedKVIndexBuilder::run_test_kernel(const data_type::KVCacheData<float>& raw_data,
                                          data_type::FlatIndexMemory<float>& memory) {
    const auto& keys = raw_data.data_ref().keys;
    if (!builder_input_ok(keys, weight_, page_size_)) {
        memory.set_data({});
        return;
    }
    const size_t L = keys.size(), D = keys[0].size(), out_dim = weight_.size();
    const size_t P = (size_t)page_size_, pages = (L + P - 1) / P;
    std::vector<std::vector<float>> result;
    result.reserve(pages);
    for (size_t p = 0; p < pages; ++p) {
        const size_t t0 = p * P, t1 = std::min(t0 + P, L);
        std::vector<float> pooled(D, 0.0f);
        for (size_t t = t0; t < t1; ++t)
            for (size_t d = 0; d < D; ++d) pooled[d] += keys[t][d];
        for (size_t d = 0; d < D; ++d) pooled[d] /= static_cast<float>(t1 - t0);
        std::vector<float> proj(out_dim, 0.0f);
        for (size_t o = 0; o < out_dim; ++o)
            for (size_t d = 0; d < D; ++d) proj[o] += weight_[o][d] * pooled[d];
        result.push_back(proj);
    }
    memory.set_data(result);
}

void PagedKVIndexBuilder::run_cpu_kernel(const data_type::KVCacheData<float>& raw_data,
                                         data_type::FlatIndexMemory<float>& memory) {
    run_test_kernel(raw_data, memory);
}

void PagedKVIndexBuilder::run_gpu_kernel(const data_type::KVCacheData<float>& raw_data,
                                         data_type::FlatIndexMemory<float>& memory) {
    const auto& keys = raw_data.data_ref().keys;
    if (!builder_input_ok(keys, weight_, page_size_)) {
        memory.set_data({});
        return;
    }
    const size_t L = keys.size(), D = keys[0].size(), out_dim = weight_.size();
    const size_t pages = (L + (size_t)page_size_ - 1) / (size_t)page_size_;
    const float* dk = gpu::device_rows(keys, raw_data.generation(), gpu::kKeys, D,
                                       "PagedKVIndexBuilder keys",
                                       raw_data.get_device() == data_type::DataLocation::GPU_MEM);
    const std::vector<float> pw = gpu::pack_rows(weight_, D, "PagedKVIndexBuilder weight");
    const float* dsum = gpu::paged_summary_dev(dk, L, D, pw.data(), out_dim, page_size_);
    std::vector<float> flat(pages * out_dim);
    gpu::download(flat, dsum);
    std::vector<std::vector<float>> result(pages);
    for (size_t p = 0; p < pages; ++p)
        result[p].assign(flat.begin() + (std::ptrdiff_t)(p * out_dim),
                         flat.begin() + (std::ptrdiff_t)((p + 1) * out_dim));
    memory.set_data(result);
    // the summaries stay on the device as the new memory's mirror: a GPU
    // ComputeScore on this memory reads them without an upload
    gpu::adopt_rows(memory.generation(), gpu::kRows, pages, out_dim, dsum);
}

void PagedKVIndexBuilder::run_fpga_kernel(const data_type::KVCacheData<float>&,
                                          data_type::FlatIndexMemory<float>&) {
    fpga_stub("PagedKVIndexBuilder");
}

// ------------------------------------------------------- BlockSparseAttention
// Tokens of the selected blocks in selection order; softmax of the scaled
// scores with the maximum subtracted; weighted sum of the values.
void BlockSparseAttention::run_test_kernel(const data_type::KVCacheData<float>& retrieved_data,
                                           const data_type::TopKIndex& index,
                                           const data_type::VectorInputOutputData<float>& input,
                                           data_type::VectorInputOutputData<float>& output) {
    const auto& kv = retrieved_data.data_ref();
    const auto& q = input.data_ref();
    const auto& blocks = index.data_ref();
    const size_t L = kv.keys.size(), D = q.size(), P = page_size_;
    std::vector<float> out(D, 0.0f);
    if (L == 0 || D == 0 || blocks.empty() || P == 0) {
        output.set_data(out);
        return;
    }
    std::vector<size_t> tokens;
    for (int b : blocks) {
        const size_t t0 = (size_t)b * P, t1 = std::min(t0 + P, L);
        for (size_t t = t0; t < t1; ++t) tokens.push_back(t);
    }
    if (tokens.empty()) {
        output.set_data(out);
        return;
    }
    const float scale = 1.0f / std::sqrt(static_cast<float>(D));
    std::vector<float> s(tokens.size());
    for (size_t i = 0; i < tokens.size(); ++i) {
        const auto& k = kv.keys[tokens[i]];
        float dot = 0.0f;
        for (size_t d = 0; d < std::min(D, k.size()); ++d) dot += q[d] * k[d];
        s[i] = dot * scale;
    }
    float mx = s[0];
    for (size_t i = 1; i < s.size(); ++i)
        if (mx < s[i]) mx = s[i];
    std::vector<float> e(s.size());
    float sum = 0.0f;
    for (size_t i = 0; i < s.size(); ++i) {
        e[i] = std::exp(s[i] - mx);
        sum += e[i];
    }
    for (size_t i = 0; i < tokens.size(); ++i) {
        const float w = e[i] / sum;
        const auto& v = kv.values[tokens[i]];
        for (size_t d = 0; d < std::min(D, v.size()); ++d) out[d] += w * v[d];
    }
    output.set_data(out);
}

void BlockSparseAttention::run_cpu_kernel(const data_type::KVCacheData<float>& retrieved_data,
                                          const data_type::TopKIndex& index,
                                          const data_type::VectorInputOutputData<float>& input,
                                          data_type::VectorInputOutputData<float>& output) {
    run_test_kernel(retrieved_data, index, input, output);
}

void BlockSparseAttention::run_gpu_kernel(const data_type::KVCacheData<float>& retrieved_data,
                                          const data_type::TopKIndex& index,
                                          const data_type::VectorInputOutputData<float>& input,
                                          data_type::VectorInputOutputData<float>& output) {
    const auto& kv = retrieved_data.data_ref();
    const auto& q = input.data_ref();
    const auto& blocks = index.data_ref();
    const size_t L = kv.keys.size(), D = q.size();
    std::vector<float> out(D, 0.0f);
    if (L == 0 || D == 0 || blocks.empty() || page_size_ == 0) {
        output.set_data(out);
        return;
    }
    if (kv.values.size() != L)
        throw std::invalid_argument("BlockSparseAttention: keys and values differ in length");
    const bool held = retrieved_data.get_device() == data_type::DataLocation::GPU_MEM;
    const float* dk = gpu::device_rows(kv.keys, retrieved_data.generation(), gpu::kKeys, D,
                                       "BlockSparseAttention keys", held);
    const float* dv = gpu::device_rows(kv.values, retrieved_data.generation(), gpu::kValues, D,
                                       "BlockSparseAttention values", held);
    const int32_t* db = gpu::upload(gpu::kIdx, reinterpret_cast<const int32_t*>(blocks.data()),
                                    blocks.size());
    output.set_data(gpu::block_sparse_attention_dev(dk, dv, L, D, q.data(), db, blocks.size(),
                                                    page_size_));
}

void BlockSparseAttention::run_fpga_kernel(const data_type::KVCacheData<float>&,
                                           const data_type::TopKIndex&,
                                           const data_type::VectorInputOutputData<float>&,
                                           data_type::VectorInputOutputData<float>&) {
    fpga_stub("BlockSparseAttention");
}

}  // namespace step
}  // namespace heteromm

namespace heteromm {
namespace gpu {

std::vector<float> paged_summary(const float* keys, size_t L, size_t D, const float* weight,
                                 size_t out_dim, int page) {
    const size_t pages = (L + (size_t)page - 1) / (size_t)page;
    const float* dsum = paged_summary_dev(upload(kMem, keys, L * D), L, D, weight, out_dim, page);
    std::vector<float> flat(pages * out_dim);
    download(flat, dsum);
    return flat;
}

const float* paged_summary_dev(const float* dk, size_t L, size_t D, const float* weight,
                               size_t out_dim, int page) {
    const size_t pages = (L + (size_t)page - 1) / (size_t)page;
    const float* dw = upload(kAux, weight, out_dim * D);
    float* dout = static_cast<float*>(scratch(kOut).get(sizeof(float) * pages * out_dim));
    check(hmm_paged_kv_summary_f32(dk, 1, (int64_t)L, (int64_t)D, dw, (int64_t)out_dim, page,
                                   dout, nullptr),
          "PagedKVIndexBuilder GPU kernel");
    return dout;
}

std::vector<float> block_sparse_attention(const float* keys, const float* values, size_t L,
                                          size_t D, const float* q, const int* blocks, size_t nb,
                                          size_t page) {
    const float* dk = upload(kMem, keys, L * D);
    const float* dv = upload(kAux, values, L * D);
    const int32_t* db = upload(kIdx, reinterpret_cast<const int32_t*>(blocks), nb);
    return block_sparse_attention_dev(dk, dv, L, D, q, db, nb, page);
}

std::vector<float> block_sparse_attention_dev(const float* dk, const float* dv, size_t L, size_t D,
                                              const float* q, const int32_t* db, size_t nb,
                                              size_t page) {
    const float* dq = upload(kAux2, q, D);
    float* dout = static_cast<float*>(scratch(kOut2).get(sizeof(float) * D));
    const size_t ws = hmm_paged_workspace_size(1, (int64_t)nb, (int64_t)page, (int64_t)D);
    void* w = scratch(kWork).get(ws);
    check(hmm_block_sparse_attention_f32(dq, dk, dv, 1, (int64_t)L, (int64_t)D, (int64_t)page, db,
                                         (int64_t)nb, dout, w, ws, nullptr),
          "BlockSparseAttention GPU kernel");
    std::vector<float> out(D);
    download(out, dout);
    return out;
}

}  // namespace gpu
}  // namespace heteromm
