// build_memory.h — BuildMemory step: RetrievedData -> Memory (B200 build).
// Interface of the reference's steps/build_memory.h:44-182; the
// KernelType::GPU arm of PagedKVIndexBuilder runs hmm_paged_kv_summary_f32.
#ifndef HETEROMM_B200_DEV_STEPS_BUILD_MEMORY_H_
#define HETEROMM_B200_DEV_STEPS_BUILD_MEMORY_H_

#include <type_traits>
#include <vector>

#include "../types/memory.h"
#include "../types/retrieved_data.h"
#include "util.h"

namespace heteromm {
namespace step {

template <typename RetDataType, typename MemoryType>
class BuildMemory {
    static_assert(std::is_base_of<data_type::RetrievedData<typename RetDataType::content_type>,
                                  RetDataType>::value,
                  "RetDataType must derive from data_type::RetrievedData");
    static_assert(std::is_base_of<data_type::Memory<typename MemoryType::content_type>,
                                  MemoryType>::value,
                  "MemoryType must derive from data_type::Memory");

public:
    BuildMemory() = default;
    virtual ~BuildMemory() = default;

    int execute(const RetDataType& raw_data, MemoryType& memory, bool run_functional_test = false,
                bool verbose = false) {
        if (run_functional_test)
            return detail::functional_test("BuildMemory", memory, verbose,
                                           [&] { run_test_kernel(raw_data, memory); });
        detail::log_kernel("BuildMemory", current_kernel_, verbose, false);
        switch (current_kernel_) {
            case KernelType::CPU: run_cpu_kernel(raw_data, memory); break;
            case KernelType::GPU: run_gpu_kernel(raw_data, memory); break;
            case KernelType::FPGA: run_fpga_kernel(raw_data, memory); break;
        }
        detail::log_kernel("BuildMemory", current_kernel_, verbose, true);
        return 0;
    }

    KernelType current_kernel() const { return current_kernel_; }
    void set_current_kernel(KernelType type) { current_kernel_ = type; }

protected:
    virtual void run_test_kernel(const RetDataType&, MemoryType&) = 0;
    virtual void run_cpu_kernel(const RetDataType&, MemoryType&) = 0;
    virtual void run_gpu_kernel(const RetDataType&, MemoryType&) = 0;
    virtual void run_fpga_kernel(const RetDataType&, MemoryType&) = 0;

private:
    KernelType current_kernel_ = KernelType::CPU;
};

// Page summaries of a key cache: page p pools tokens [p*P, min(p*P+P, L))
// (fp32 mean), projected by weight [out_dim][D].
class PagedKVIndexBuilder
    : public BuildMemory<data_type::KVCacheData<float>, data_type::FlatIndexMemory<float>> {
public:
    PagedKVIndexBuilder() = default;
    PagedKVIndexBuilder(const std::vector<std::vector<float>>& weight, int page_size)
        : weight_(weight), page_size_(page_size) {}
    ~PagedKVIndexBuilder() override = default;

protected:
    void run_test_kernel(const data_type::KVCacheData<float>& raw_data,
                         data_type::FlatIndexMemory<float>& memory) override;
    void run_cpu_kernel(const data_type::KVCacheData<float>& raw_data,
                        data_type::FlatIndexMemory<float>& memory) override;
    void run_gpu_kernel(const data_type::KVCacheData<float>& raw_data,
                        data_type::FlatIndexMemory<float>& memory) override;
    void run_fpga_kernel(const data_type::KVCacheData<float>& raw_data,
                         data_type::FlatIndexMemory<float>& memory) override;

private:
    std::vector<std::vector<float>> weight_;
    int page_size_ = 0;
};

}  // namespace step
}  // namespace heteromm

#endif  // HETEROMM_B200_DEV_STEPS_BUILD_MEMORY_H_
