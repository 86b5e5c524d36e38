// steps_flat.cpp — InnerProductCompute, TopKRetrieval, ThresholdRetrieval and
// InnerProductTopKRetrieval: CPU bodies (the reference's arithmetic,
// steps/example_kernel/inner_product_compute.cpp:11-31,
// topk_retrieval.cpp:13-31, threshold_retrieval.cpp:11-32) and GPU adapters
// onto hmm_ip_score_f32 / hmm_topk_f32 / hmm_threshold_bitmap_f32 /
// hmm_ip_topk_f32.
#include <algorithm>
#include <cmath>
#include <iostream>
#include <numeric>

#include "device.h"
#include "packed.h"
#include "heteromm/dev/steps/compute_score.h"
#include "heteromm/dev/steps/fused_steps/template.h"
#include "heteromm/dev/steps/memory_retrieval.h"

namespace heteromm {
namespace step {

namespace {
// fp32 dot products in index order, each product rounded before the add.
std::vector<float> cpu_scores(const std::vector<std::vector<float>>& mem,
                              const std::vector<float>& q) {
    std::vector<float> s(mem.size(), 0.0f);
    for (size_t i = 0; i < mem.size(); ++i) {
        float dot = 0.0f;
        for (size_t j = 0; j < q.size(); ++j) dot += mem[i][j] * q[j];   // built without contraction
        s[i] = dot;
    }
    return s;
}

// Indices of the min(k, n) best scores, best first, ties to the lowest index
// (the reference's partial_sort by `>`, with its tie order pinned).
std::vector<int> cpu_topk(const std::vector<float>& s, size_t k) {
    const size_t n = s.size(), m = std::min(k, n);
    std::vector<int> idx(n);
    std::iota(idx.begin(), idx.end(), 0);
    std::partial_sort(idx.begin(), idx.begin() + (std::ptrdiff_t)m, idx.end(), [&](int a, int b) {
        const bool an = s[a] != s[a], bn = s[b] != s[b];
        if (an || bn) return an != bn ? bn : a < b;   // NaN ranks below every number
        return s[a] != s[b] ? s[a] > s[b] : a < b;
    });
    idx.resize(m);
    return idx;
}

std::vector<unsigned long long> cpu_bitmap(const std::vector<float>& s, float thr) {
    std::vector<unsigned long long> bm((s.size() + 63) / 64, 0ULL);
    for (size_t i = 0; i < s.size(); ++i)
        if (s[i] >= thr) bm[i / 64] |= 1ULL << (i % 64);
    return bm;
}

// The memory's first d columns on the device: its cached mirror when the
// memory is unchanged since an earlier call on this thread, or that mirror
// brought up to date from the memory's row log after inserts and deletes.
const float* device_rows(const data_type::FlatIndexMemory<float>& memory, size_t d,
                         const char* what) {
    return gpu::device_flat_rows(memory, d, what);
}

void fpga_stub(const char* step) {
    std::clog << "[" << step << "] FPGA kernel not implemented. exiting." << std::endl;
}
}  // namespace

// ------------------------------------------------------------ InnerProduct
void InnerProductCompute::run_test_kernel(const data_type::FlatIndexMemory<float>& memory,
                                          const data_type::VectorQuery<float>& query,
                                          data_type::VectorScore<float>& score) {
    score.set_data(cpu_scores(memory.data_ref(), query.data_ref()));
}

void InnerProductCompute::run_cpu_kernel(const data_type::FlatIndexMemory<float>& memory,
                                         const data_type::VectorQuery<float>& query,
                                         data_type::VectorScore<float>& score) {
    run_test_kernel(memory, query, score);
}

void InnerProductCompute::run_gpu_kernel(const data_type::FlatIndexMemory<float>& memory,
                                         const data_type::VectorQuery<float>& query,
                                         data_type::VectorScore<float>& score) {
    const auto& rows = memory.data_ref();
    const auto& q = query.data_ref();
    const size_t n = rows.size(), d = q.size();
    if (n == 0 || d == 0) {
        score.set_data(std::vector<float>(n, 0.0f));
        return;
    }
    score.set_data(gpu::ip_scores_dev(device_rows(memory, d, "InnerProductCompute"), n, d, q.data()));
}

void InnerProductCompute::run_fpga_kernel(const data_type::FlatIndexMemory<float>&,
                                          const data_type::VectorQuery<float>&,
                                          data_type::VectorScore<float>&) {
    fpga_stub("InnerProductCompute");
}

// ------------------------------------------------------------------ TopK
void TopKRetrieval::run_test_kernel(const data_type::VectorScore<float>& score,
                                    data_type::TopKIndex& index) {
    index.set_data(cpu_topk(score.data_ref(), k_));
}

void TopKRetrieval::run_cpu_kernel(const data_type::VectorScore<float>& score,
                                   data_type::TopKIndex& index) {
    run_test_kernel(score, index);
}

void TopKRetrieval::run_gpu_kernel(const data_type::VectorScore<float>& score,
                                   data_type::TopKIndex& index) {
    const auto& s = score.data_ref();
    const size_t n = s.size(), m = std::min(k_, n);
    std::vector<int> out(m);
    if (m > 0) {
        const float* ds = gpu::upload(gpu::kQuery, s);
        int32_t* di = static_cast<int32_t*>(gpu::scratch(gpu::kIdx).get(sizeof(int32_t) * m));
        const size_t ws = hmm_topk_f32_workspace_size((int64_t)n, 1, (int64_t)m);
        void* w = gpu::scratch(gpu::kWork).get(ws);
        gpu::check(hmm_topk_f32(ds, (int64_t)n, 1, (int64_t)m, di, nullptr, w, ws, nullptr),
                   "TopKRetrieval GPU kernel");
        gpu::download(out, di);
    }
    index.set_data(out);
}

void TopKRetrieval::run_fpga_kernel(const data_type::VectorScore<float>&, data_type::TopKIndex&) {
    fpga_stub("TopKRetrieval");
}

// ------------------------------------------------------------- Threshold
void ThresholdRetrieval::run_test_kernel(const data_type::VectorScore<float>& score,
                                         data_type::ThresholdBitmapIndex& index) {
    const auto& s = score.data_ref();
    index = data_type::ThresholdBitmapIndex(cpu_bitmap(s, threshold_), s.size());
}

void ThresholdRetrieval::run_cpu_kernel(const data_type::VectorScore<float>& score,
                                        data_type::ThresholdBitmapIndex& index) {
    run_test_kernel(score, index);
}

void ThresholdRetrieval::run_gpu_kernel(const data_type::VectorScore<float>& score,
                                        data_type::ThresholdBitmapIndex& index) {
    const auto& s = score.data_ref();
    const size_t n = s.size();
    std::vector<unsigned long long> bm((n + 63) / 64);
    if (n > 0) {
        const float* ds = gpu::upload(gpu::kQuery, s);
        auto* db = static_cast<uint64_t*>(gpu::scratch(gpu::kOut).get(sizeof(uint64_t) * bm.size()));
        gpu::check(hmm_threshold_bitmap_f32(ds, (int64_t)n, 1, threshold_, db, nullptr),
                   "ThresholdRetrieval GPU kernel");
        gpu::download(bm, reinterpret_cast<const unsigned long long*>(db));
    }
    index = data_type::ThresholdBitmapIndex(bm, n);
}

void ThresholdRetrieval::run_fpga_kernel(const data_type::VectorScore<float>&,
                                         data_type::ThresholdBitmapIndex&) {
    fpga_stub("ThresholdRetrieval");
}

// ------------------------------------------------- fused inner product top-k
void InnerProductTopKRetrieval::run_test_kernel(const data_type::FlatIndexMemory<float>& memory,
                                                const data_type::VectorQuery<float>& query,
                                                data_type::TopKIndex& index) {
    index.set_data(cpu_topk(cpu_scores(memory.data_ref(), query.data_ref()), k_));
}

void InnerProductTopKRetrieval::run_cpu_kernel(const data_type::FlatIndexMemory<float>& memory,
                                               const data_type::VectorQuery<float>& query,
                                               data_type::TopKIndex& index) {
    run_test_kernel(memory, query, index);
}

void InnerProductTopKRetrieval::run_gpu_kernel(const data_type::FlatIndexMemory<float>& memory,
                                               const data_type::VectorQuery<float>& query,
                                               data_type::TopKIndex& index) {
    const auto& rows = memory.data_ref();
    const auto& q = query.data_ref();
    const size_t n = rows.size(), d = q.size();
    if (std::min(k_, n) == 0 || d == 0) {
        index.set_data(gpu::ip_topk(nullptr, n, d, q.data(), k_));   // no device work
        return;
    }
    index.set_data(gpu::ip_topk_dev(device_rows(memory, d, "InnerProductTopK"), n, d, q.data(), k_));
}

void InnerProductTopKRetrieval::run_fpga_kernel(const data_type::FlatIndexMemory<float>&,
                                                const data_type::VectorQuery<float>&,
                                                data_type::TopKIndex&) {
    fpga_stub("InnerProductTopKRetrieval");
}

}  // namespace step
}  // namespace heteromm

namespace heteromm {
namespace gpu {

std::vector<float> ip_scores(const float* rows, size_t n, size_t d, const float* q) {
    if (n == 0 || d == 0) return std::vector<float>(n, 0.0f);
    return ip_scores_dev(upload(kMem, rows, n * d), n, d, q);
}

std::vector<float> ip_scores_dev(const float* dm, size_t n, size_t d, const float* q) {
    std::vector<float> out(n, 0.0f);
    const float* dq = upload(kQuery, q, d);
    float* ds = static_cast<float*>(scratch(kOut).get(sizeof(float) * n));
    check(hmm_ip_score_f32(dm, (int64_t)n, (int64_t)d, dq, 1, ds, nullptr),
          "InnerProductCompute GPU kernel");
    download(out, ds);
    return out;
}

std::vector<int> ip_topk(const float* rows, size_t n, size_t d, const float* q, size_t k) {
    if (std::min(k, n) > 0 && d > 0) return ip_topk_dev(upload(kMem, rows, n * d), n, d, q, k);
    std::vector<int> out(std::min(k, n));
    std::iota(out.begin(), out.end(), 0);   // all scores 0: the lowest indices
    return out;
}

std::vector<int> ip_topk_dev(const float* dm, size_t n, size_t d, const float* q, size_t k) {
    const size_t m = std::min(k, n);
    std::vector<int> out(m);
    {
        const float* dq = upload(kQuery, q, d);
        int32_t* di = static_cast<int32_t*>(scratch(kIdx).get(sizeof(int32_t) * m));
        const size_t ws = hmm_ip_topk_f32_workspace_size((int64_t)n, (int64_t)d, 1, (int64_t)m);
        void* w = scratch(kWork).get(ws);
        check(hmm_ip_topk_f32(dm, (int64_t)n, (int64_t)d, dq, 1, (int64_t)m, di, nullptr, 0.0f,
                              nullptr, w, ws, nullptr),
              "InnerProductTopKRetrieval GPU kernel");
        download(out, di);
    }
    return out;
}

}  // namespace gpu
}  // namespace heteromm
