// template.h — fused ComputeScore + MemoryRetrieval steps (B200 build).
// Interface of the reference's steps/fused_steps/template.h:21-200
// (set_kernel / get_kernel, as the reference names them for fused steps).
//   FusedBM25Retrieval         BM25 top-64 (GPU arm: hmm_bm25_topk_csr)
//   InnerProductTopKRetrieval  flat fp32 inner product + top-k in one pass
//                              (GPU arm: hmm_ip_topk_f32); an addition of
//                              this build, the fused form of
//                              InnerProductCompute -> TopKRetrieval
#ifndef HETEROMM_B200_DEV_STEPS_FUSED_STEPS_TEMPLATE_H_
#define HETEROMM_B200_DEV_STEPS_FUSED_STEPS_TEMPLATE_H_

#include <cstddef>
#include <string>
#include <type_traits>

#include "../../types/memory.h"
#include "../../types/query.h"
#include "../../types/retrieved_index.h"
#include "../util.h"

namespace heteromm {
namespace step {

template <typename MemoryType, typename QueryType, typename IndexType>
class FusedComputeScoreAndRetrieval {
    static_assert(std::is_base_of<data_type::Memory<typename MemoryType::content_type>,
                                  MemoryType>::value,
                  "MemoryType must derive from data_type::Memory");
    static_assert(std::is_base_of<data_type::Query<typename QueryType::content_type>,
                                  QueryType>::value,
                  "QueryType must derive from data_type::Query");
    static_assert(std::is_base_of<data_type::RetrievedIndex<typename IndexType::content_type>,
                                  IndexType>::value,
                  "IndexType must derive from data_type::RetrievedIndex");

public:
    FusedComputeScoreAndRetrieval() = default;
    virtual ~FusedComputeScoreAndRetrieval() = default;

    int execute(const MemoryType& memory, const QueryType& query, IndexType& index,
                bool run_functional_test = false, bool verbose = false) {
        if (run_functional_test)
            return detail::functional_test("FusedComputeScoreAndRetrieval", index, verbose,
                                           [&] { run_test_kernel(memory, query, index); });
        detail::log_kernel("FusedComputeScoreAndRetrieval", kernel_, verbose, false);
        switch (kernel_) {
            case KernelType::CPU: run_cpu_kernel(memory, query, index); break;
            case KernelType::GPU: run_gpu_kernel(memory, query, index); break;
            case KernelType::FPGA: run_fpga_kernel(memory, query, index); break;
        }
        detail::log_kernel("FusedComputeScoreAndRetrieval", kernel_, verbose, true);
        return 0;
    }

    void set_kernel(KernelType kernel) { kernel_ = kernel; }
    KernelType get_kernel() const { return kernel_; }

protected:
    virtual void run_test_kernel(const MemoryType&, const QueryType&, IndexType&) = 0;
    virtual void run_cpu_kernel(const MemoryType&, const QueryType&, IndexType&) = 0;
    virtual void run_gpu_kernel(const MemoryType&, const QueryType&, IndexType&) = 0;
    virtual void run_fpga_kernel(const MemoryType&, const QueryType&, IndexType&) = 0;

private:
    KernelType kernel_ = KernelType::CPU;
};

// BM25 (k1 = 1.2, b = 0.75) top-64 documents of a BM25 index.  The GPU arm
// sums the query's tokens in ascending token-id order.
class FusedBM25Retrieval
    : public FusedComputeScoreAndRetrieval<data_type::BM25IndexMemory, data_type::BM25Query,
                                           data_type::TopKIndex> {
public:
    FusedBM25Retrieval(void* fpga_setup_object = nullptr,
                       const std::string& python_module_path = ".")
        : fpga_setup_object_(fpga_setup_object), python_module_path_(python_module_path) {}
    ~FusedBM25Retrieval() override;
    void set_fpga_setup(void* fpga_setup) { fpga_setup_object_ = fpga_setup; }

protected:
    void run_fpga_kernel(const data_type::BM25IndexMemory& memory,
                         const data_type::BM25Query& query, data_type::TopKIndex& index) override;
    void run_cpu_kernel(const data_type::BM25IndexMemory& memory,
                        const data_type::BM25Query& query, data_type::TopKIndex& index) override;
    void run_gpu_kernel(const data_type::BM25IndexMemory& memory,
                        const data_type::BM25Query& query, data_type::TopKIndex& index) override;
    void run_test_kernel(const data_type::BM25IndexMemory& memory,
                         const data_type::BM25Query& query, data_type::TopKIndex& index) override;

private:
    void* fpga_setup_object_;
    std::string python_module_path_;
};

class InnerProductTopKRetrieval
    : public FusedComputeScoreAndRetrieval<data_type::FlatIndexMemory<float>,
                                           data_type::VectorQuery<float>, data_type::TopKIndex> {
public:
    explicit InnerProductTopKRetrieval(size_t k) : k_(k) {}
    ~InnerProductTopKRetrieval() override = default;
    size_t k() const { return k_; }
    void set_k(size_t k) { k_ = k; }

protected:
    void run_test_kernel(const data_type::FlatIndexMemory<float>& memory,
                         const data_type::VectorQuery<float>& query,
                         data_type::TopKIndex& index) override;
    void run_cpu_kernel(const data_type::FlatIndexMemory<float>& memory,
                        const data_type::VectorQuery<float>& query,
                        data_type::TopKIndex& index) override;
    void run_gpu_kernel(const data_type::FlatIndexMemory<float>& memory,
                        const data_type::VectorQuery<float>& query,
                        data_type::TopKIndex& index) override;
    void run_fpga_kernel(const data_type::FlatIndexMemory<float>& memory,
                         const data_type::VectorQuery<float>& query,
                         data_type::TopKIndex& index) override;

private:
    size_t k_;
};

}  // namespace step
}  // namespace heteromm

#endif  // HETEROMM_B200_DEV_STEPS_FUSED_STEPS_TEMPLATE_H_
