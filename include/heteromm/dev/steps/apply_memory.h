// apply_memory.h — ApplyMemory step: (RetrievedData, RetrievedIndex, Input)
// -> Output (B200 build).  Interface of the reference's
// steps/apply_memory.h:46-213; the KernelType::GPU arm of
// BlockSparseAttention runs hmm_block_sparse_attention_f32.
#ifndef HETEROMM_B200_DEV_STEPS_APPLY_MEMORY_H_
#define HETEROMM_B200_DEV_STEPS_APPLY_MEMORY_H_

#include <cstddef>
#include <type_traits>

#include "../types/retrieved_data.h"
#include "../types/retrieved_index.h"
#include "../types/target_data.h"
#include "util.h"

namespace heteromm {
namespace step {

template <typename RetDataType, typename IndexType, typename InputType, typename OutputType>
class ApplyMemory {
    static_assert(std::is_base_of<data_type::RetrievedData<typename RetDataType::content_type>,
                                  RetDataType>::value,
                  "RetDataType must derive from data_type::RetrievedData");
    static_assert(std::is_base_of<data_type::RetrievedIndex<typename IndexType::content_type>,
                                  IndexType>::value,
                  "IndexType must derive from data_type::RetrievedIndex");
    static_assert(std::is_base_of<data_type::TargetData<typename InputType::content_type>,
                                  InputType>::value,
                  "InputType must derive from data_type::TargetData");
    static_assert(std::is_base_of<data_type::TargetData<typename OutputType::content_type>,
                                  OutputType>::value,
                  "OutputType must derive from data_type::TargetData");

public:
    ApplyMemory() = default;
    virtual ~ApplyMemory() = default;

    int execute(const RetDataType& retrieved_data, const IndexType& index, const InputType& input,
                OutputType& output, bool run_functional_test = false, bool verbose = false) {
        if (run_functional_test)
            return detail::functional_test("ApplyMemory", output, verbose, [&] {
                run_test_kernel(retrieved_data, index, input, output);
            });
        detail::log_kernel("ApplyMemory", current_kernel_, verbose, false);
        switch (current_kernel_) {
            case KernelType::CPU: run_cpu_kernel(retrieved_data, index, input, output); break;
            case KernelType::GPU: run_gpu_kernel(retrieved_data, index, input, output); break;
            case KernelType::FPGA: run_fpga_kernel(retrieved_data, index, input, output); break;
        }
        detail::log_kernel("ApplyMemory", current_kernel_, verbose, true);
        return 0;
    }

    KernelType current_kernel() const { return current_kernel_; }
    void set_current_kernel(KernelType type) { current_kernel_ = type; }

protected:
    virtual void run_test_kernel(const RetDataType&, const IndexType&, const InputType&,
                                 OutputType&) = 0;
    virtual void run_cpu_kernel(const RetDataType&, const IndexType&, const InputType&,
                                OutputType&) = 0;
    virtual void run_gpu_kernel(const RetDataType&, const IndexType&, const InputType&,
                                OutputType&) = 0;
    virtual void run_fpga_kernel(const RetDataType&, const IndexType&, const InputType&,
                                 OutputType&) = 0;

private:
    KernelType current_kernel_ = KernelType::CPU;
};

// Softmax attention of the input query over the tokens of the selected
// blocks of `page_size` tokens, scaled by 1/sqrt(head_dim).
class BlockSparseAttention
    : public ApplyMemory<data_type::KVCacheData<float>, data_type::TopKIndex,
                         data_type::VectorInputOutputData<float>,
                         data_type::VectorInputOutputData<float>> {
public:
    BlockSparseAttention() = default;
    BlockSparseAttention(size_t page_size) : page_size_(page_size) {}
    ~BlockSparseAttention() override = default;

    // Tokens per block (an accessor of this build; the device-resident
    // pipeline of deploy/paged_attention.h reads it).
    size_t page_size() const { return page_size_; }

protected:
    void run_test_kernel(const data_type::KVCacheData<float>& retrieved_data,
                         const data_type::TopKIndex& index,
                         const data_type::VectorInputOutputData<float>& input,
                         data_type::VectorInputOutputData<float>& output) override;
    void run_cpu_kernel(const data_type::KVCacheData<float>& retrieved_data,
                        const data_type::TopKIndex& index,
                        const data_type::VectorInputOutputData<float>& input,
                        data_type::VectorInputOutputData<float>& output) override;
    void run_gpu_kernel(const data_type::KVCacheData<float>& retrieved_data,
                        const data_type::TopKIndex& index,
                        const data_type::VectorInputOutputData<float>& input,
                        data_type::VectorInputOutputData<float>& output) override;
    void run_fpga_kernel(const data_type::KVCacheData<float>& retrieved_data,
                         const data_type::TopKIndex& index,
                         const data_type::VectorInputOutputData<float>& input,
                         data_type::VectorInputOutputData<float>& output) override;

private:
    size_t page_size_ = 0;
};

}  // namespace step
}  // namespace heteromm

#endif  // HETEROMM_B200_DEV_STEPS_APPLY_MEMORY_H_
