// compute_score.h — ComputeScore step: (Memory, Query) -> Score (B200 build).
// Interface of the reference's steps/compute_score.h:41-205; the
// KernelType::GPU arm of InnerProductCompute runs hmm_ip_score_f32.
#ifndef HETEROMM_B200_DEV_STEPS_COMPUTE_SCORE_H_
#define HETEROMM_B200_DEV_STEPS_COMPUTE_SCORE_H_

#include <type_traits>

#include "../types/memory.h"
#include "../types/query.h"
#include "../types/score.h"
#include "util.h"

namespace heteromm {
namespace step {

template <typename MemoryType, typename QueryType, typename ScoreType>
class ComputeScore {
    static_assert(std::is_base_of<data_type::Memory<typename MemoryType::content_type>,
                                  MemoryType>::value,
                  "MemoryType must derive from data_type::Memory");
    static_assert(std::is_base_of<data_type::Query<typename QueryType::content_type>,
                                  QueryType>::value,
                  "QueryType must derive from data_type::Query");
    static_assert(std::is_base_of<data_type::Score<typename ScoreType::content_type>,
                                  ScoreType>::value,
                  "ScoreType must derive from data_type::Score");

public:
    ComputeScore() = default;
    virtual ~ComputeScore() = default;

    int execute(const MemoryType& memory, const QueryType& query, ScoreType& score,
                bool run_functional_test = false, bool verbose = false) {
        if (run_functional_test)
            return detail::functional_test("ComputeScore", score, verbose,
                                           [&] { run_test_kernel(memory, query, score); });
        detail::log_kernel("ComputeScore", current_kernel_, verbose, false);
        switch (current_kernel_) {
            case KernelType::CPU: run_cpu_kernel(memory, query, score); break;
            case KernelType::GPU: run_gpu_kernel(memory, query, score); break;
            case KernelType::FPGA: run_fpga_kernel(memory, query, score); break;
        }
        detail::log_kernel("ComputeScore", current_kernel_, verbose, true);
        return 0;
    }

    KernelType current_kernel() const { return current_kernel_; }
    void set_current_kernel(KernelType type) { current_kernel_ = type; }

protected:
    virtual void run_test_kernel(const MemoryType&, const QueryType&, ScoreType&) = 0;
    virtual void run_gpu_kernel(const MemoryType&, const QueryType&, ScoreType&) = 0;
    virtual void run_fpga_kernel(const MemoryType&, const QueryType&, ScoreType&) = 0;
    virtual void run_cpu_kernel(const MemoryType&, const QueryType&, ScoreType&) = 0;

private:
    KernelType current_kernel_ = KernelType::CPU;
};

// score[i] = sum_j memory[i][j] * query[j] in fp32, j ascending.
class InnerProductCompute
    : public ComputeScore<data_type::FlatIndexMemory<float>, data_type::VectorQuery<float>,
                          data_type::VectorScore<float>> {
public:
    InnerProductCompute() = default;
    ~InnerProductCompute() override = default;

protected:
    void run_test_kernel(const data_type::FlatIndexMemory<float>& memory,
                         const data_type::VectorQuery<float>& query,
                         data_type::VectorScore<float>& score) override;
    void run_cpu_kernel(const data_type::FlatIndexMemory<float>& memory,
                        const data_type::VectorQuery<float>& query,
                        data_type::VectorScore<float>& score) override;
    void run_gpu_kernel(const data_type::FlatIndexMemory<float>& memory,
                        const data_type::VectorQuery<float>& query,
                        data_type::VectorScore<float>& score) override;
    void run_fpga_kernel(const data_type::FlatIndexMemory<float>& memory,
                         const data_type::VectorQuery<float>& query,
                         data_type::VectorScore<float>& score) override;
};

}  // namespace step
}  // namespace heteromm

#endif  // HETEROMM_B200_DEV_STEPS_COMPUTE_SCORE_H_
