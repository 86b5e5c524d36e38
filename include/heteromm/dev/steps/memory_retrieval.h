// memory_retrieval.h — MemoryRetrieval step: Score -> RetrievedIndex (B200
// build).  Interface of the reference's steps/memory_retrieval.h:39-234; the
// KernelType::GPU arms run hmm_topk_f32 and hmm_threshold_bitmap_f32.
#ifndef HETEROMM_B200_DEV_STEPS_MEMORY_RETRIEVAL_H_
#define HETEROMM_B200_DEV_STEPS_MEMORY_RETRIEVAL_H_

#include <cstddef>
#include <type_traits>

#include "../types/retrieved_index.h"
#include "../types/score.h"
#include "util.h"

namespace heteromm {
namespace step {

template <typename ScoreType, typename IndexType>
class MemoryRetrieval {
    static_assert(std::is_base_of<data_type::Score<typename ScoreType::content_type>,
                                  ScoreType>::value,
                  "ScoreType must derive from data_type::Score");
    static_assert(std::is_base_of<data_type::RetrievedIndex<typename IndexType::content_type>,
                                  IndexType>::value,
                  "IndexType must derive from data_type::RetrievedIndex");

public:
    MemoryRetrieval() = default;
    virtual ~MemoryRetrieval() = default;

    int execute(const ScoreType& score, IndexType& index, bool run_functional_test = false,
                bool verbose = false) {
        if (run_functional_test)
            return detail::functional_test("MemoryRetrieval", index, verbose,
                                           [&] { run_test_kernel(score, index); });
        detail::log_kernel("MemoryRetrieval", current_kernel_, verbose, false);
        switch (current_kernel_) {
            case KernelType::CPU: run_cpu_kernel(score, index); break;
            case KernelType::GPU: run_gpu_kernel(score, index); break;
            case KernelType::FPGA: run_fpga_kernel(score, index); break;
        }
        detail::log_kernel("MemoryRetrieval", current_kernel_, verbose, true);
        return 0;
    }

    KernelType current_kernel() const { return current_kernel_; }
    void set_current_kernel(KernelType type) { current_kernel_ = type; }

protected:
    virtual void run_test_kernel(const ScoreType&, IndexType&) = 0;
    virtual void run_gpu_kernel(const ScoreType&, IndexType&) = 0;
    virtual void run_fpga_kernel(const ScoreType&, IndexType&) = 0;
    virtual void run_cpu_kernel(const ScoreType&, IndexType&) = 0;

private:
    KernelType current_kernel_ = KernelType::CPU;
};

// The min(k, n) best scores' indices, best first, ties to the lowest index.
class TopKRetrieval
    : public MemoryRetrieval<data_type::VectorScore<float>, data_type::TopKIndex> {
public:
    explicit TopKRetrieval(size_t k) : k_(k) {}
    ~TopKRetrieval() override = default;
    size_t k() const { return k_; }
    void set_k(size_t k) { k_ = k; }

protected:
    void run_test_kernel(const data_type::VectorScore<float>& score,
                         data_type::TopKIndex& index) override;
    void run_cpu_kernel(const data_type::VectorScore<float>& score,
                        data_type::TopKIndex& index) override;
    void run_gpu_kernel(const data_type::VectorScore<float>& score,
                        data_type::TopKIndex& index) override;
    void run_fpga_kernel(const data_type::VectorScore<float>& score,
                         data_type::TopKIndex& index) override;

private:
    size_t k_;
};

// Bitmap of the scores >= threshold.
class ThresholdRetrieval
    : public MemoryRetrieval<data_type::VectorScore<float>, data_type::ThresholdBitmapIndex> {
public:
    explicit ThresholdRetrieval(float threshold) : threshold_(threshold) {}
    ~ThresholdRetrieval() override = default;
    float threshold() const { return threshold_; }
    void set_threshold(float threshold) { threshold_ = threshold; }

protected:
    void run_test_kernel(const data_type::VectorScore<float>& score,
                         data_type::ThresholdBitmapIndex& index) override;
    void run_cpu_kernel(const data_type::VectorScore<float>& score,
                        data_type::ThresholdBitmapIndex& index) override;
    void run_gpu_kernel(const data_type::VectorScore<float>& score,
                        data_type::ThresholdBitmapIndex& index) override;
    void run_fpga_kernel(const data_type::VectorScore<float>& score,
                         data_type::ThresholdBitmapIndex& index) override;

private:
    float threshold_;
};

}  // namespace step
}  // namespace heteromm

#endif  // HETEROMM_B200_DEV_STEPS_MEMORY_RETRIEVAL_H_
