// deploy_chain.cpp — the device-resident pass of the PagedAttention pipeline
// (include/heteromm/deploy/device_chain.h): InnerProductCompute ->
// TopKRetrieval -> BlockSparseAttention with the scores and block ids kept on
// the device, the page summaries and the KV cache read from this thread's
// device mirrors.  Each branch returns what the three steps' GPU arms
// (steps_flat.cpp, steps_paged.cpp) return when run one after another on the
// same objects.
#include <algorithm>
#include <numeric>
#include <stdexcept>

#include "device.h"
#include "packed.h"
#include "heteromm/deploy/device_chain.h"

namespace heteromm {
namespace gpu {

namespace {
// Three events on the legacy default stream, per thread and device.
struct ChainEvents {
    cudaEvent_t e[3] = {nullptr, nullptr, nullptr};
    ChainEvents() {
        for (auto& x : e) check_cuda(cudaEventCreate(&x), "cudaEventCreate");
    }
    ~ChainEvents() {
        for (auto& x : e)
            if (x) cudaEventDestroy(x);
    }
};

ChainEvents& chain_events() { return per_device<ChainEvents>(); }

float elapsed_ms(cudaEvent_t a, cudaEvent_t b) {
    float ms = 0.0f;
    check_cuda(cudaEventElapsedTime(&ms, a, b), "cudaEventElapsedTime");
    return ms;
}
}  // namespace

std::vector<float> paged_attention_chain(const data_type::KVCacheData<float>& kv,
                                         const data_type::FlatIndexMemory<float>& memory,
                                         const std::vector<float>& query, size_t k,
                                         const std::vector<float>& input, size_t page,
                                         ChainTimes* times) {
    ChainEvents& ev = chain_events();
    check_cuda(cudaEventRecord(ev.e[0], nullptr), "cudaEventRecord");

    // InnerProductCompute + TopKRetrieval: the min(k, n) best summaries.
    const auto& rows = memory.data_ref();
    const size_t n = rows.size(), d = query.size(), m = std::min(k, n);
    int32_t* dblocks = static_cast<int32_t*>(scratch(kIdx).get(sizeof(int32_t) * (m ? m : 1)));
    if (m > 0 && d > 0) {
        const float* dm = device_flat_rows(memory, d, "InnerProductCompute");
        const float* dq = upload(kQuery, query.data(), d);
        const size_t ws = hmm_ip_topk_f32_workspace_size((int64_t)n, (int64_t)d, 1, (int64_t)m);
        void* w = scratch(kWork).get(ws);
        check(hmm_ip_topk_f32(dm, (int64_t)n, (int64_t)d, dq, 1, (int64_t)m, dblocks, nullptr,
                              0.0f, nullptr, w, ws, nullptr),
              "InnerProductTopKRetrieval GPU kernel");
    } else if (m > 0) {
        // no query dimensions: every score is 0, the lowest block ids win
        std::vector<int32_t> first(m);
        std::iota(first.begin(), first.end(), 0);
        copy_h2d(dblocks, first.data(), sizeof(int32_t) * m);
    }
    check_cuda(cudaEventRecord(ev.e[1], nullptr), "cudaEventRecord");

    // BlockSparseAttention on the device-resident block ids.
    const auto& keys = kv.data_ref().keys;
    const auto& values = kv.data_ref().values;
    const size_t L = keys.size(), D = input.size();
    std::vector<float> out(D, 0.0f);
    if (m > 0 && L > 0 && D > 0 && page > 0) {
        if (values.size() != L)
            throw std::invalid_argument("BlockSparseAttention: keys and values differ in length");
        const bool held = kv.get_device() == data_type::DataLocation::GPU_MEM;
        const float* dk =
            device_rows(keys, kv.generation(), kKeys, D, "BlockSparseAttention keys", held);
        const float* dv =
            device_rows(values, kv.generation(), kValues, D, "BlockSparseAttention values", held);
        out = block_sparse_attention_dev(dk, dv, L, D, input.data(), dblocks, m, page);
    }
    check_cuda(cudaEventRecord(ev.e[2], nullptr), "cudaEventRecord");
    check_cuda(cudaEventSynchronize(ev.e[2]), "cudaEventSynchronize");
    if (times) {
        times->score_topk_ms = elapsed_ms(ev.e[0], ev.e[1]);
        times->apply_ms = elapsed_ms(ev.e[1], ev.e[2]);
    }
    return out;
}

}  // namespace gpu
}  // namespace heteromm
