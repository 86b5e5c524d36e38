// memory_manager.h — the MemoryManager pipeline of the heteromm deploy layer
// (B200 build).
//
// Interface of the reference's deploy/memory_manager.h: a MemoryManager over
// seven data types runs build_memory (RetrievedData -> Memory), then
// compute_score -> memory_retrieval -> apply_memory, with the kernel of each
// step (CPU / GPU / FPGA) taken from the first matching rule of a schedule file
// (utils.h), and reports per-step times in an ExecutionResult.
//
// The reference's header does not compile; this one fixes it where it fails:
//   - ret_data_size / memory_size take const references (the reference
//     declares them non-const, :277-278, and calls them on const data,
//     :302, :360, so PagedAttention's const overloads never override and the
//     class stays abstract);
//   - build_memory looks its rule up by the one size the rule has (:304);
//   - build_and_apply_memory declares its memory before use and calls the
//     schedule lookup that exists (:451-452).
// Two choices where the reference's intent and its body disagree:
//   - with no rule for an entry point (no schedule file), the kernels set by
//     set_kernel_config / set_*_kernel run, as the reference's comments say
//     (its body would throw "No matching ... rule");
//   - build_and_apply_memory's own rule sets all four kernels (the reference's
//     body re-resolves the nested entry points' rules, which would override
//     the build_and_apply_memory entries of its schedule file).
// An addition: when compute_score, memory_retrieval and apply_memory all run on
// the GPU, a subclass may run the three as one device-resident pass
// (run_device_chain) so scores and indices never return to the host;
// set_device_chain(false) keeps the step-by-step route.
#ifndef HETEROMM_B200_DEPLOY_MEMORY_MANAGER_H_
#define HETEROMM_B200_DEPLOY_MEMORY_MANAGER_H_

#include <chrono>
#include <iostream>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "../dev/steps/apply_memory.h"
#include "../dev/steps/build_memory.h"
#include "../dev/steps/compute_score.h"
#include "../dev/steps/memory_retrieval.h"
#include "../dev/steps/util.h"
#include "../dev/types/base_types.h"
#include "../dev/types/memory.h"
#include "../dev/types/query.h"
#include "../dev/types/retrieved_data.h"
#include "../dev/types/retrieved_index.h"
#include "../dev/types/score.h"
#include "../dev/types/target_data.h"
#include "utils.h"

namespace heteromm {
namespace deploy {

// Kernel of each pipeline step (reference memory_manager.h:41-54).
struct PipelineKernelConfig {
    step::KernelType build_memory = step::KernelType::CPU;
    step::KernelType compute_score = step::KernelType::CPU;
    step::KernelType memory_retrieval = step::KernelType::CPU;
    step::KernelType apply_memory = step::KernelType::CPU;

    PipelineKernelConfig() = default;
    PipelineKernelConfig(step::KernelType build, step::KernelType compute,
                         step::KernelType retrieval, step::KernelType apply)
        : build_memory(build), compute_score(compute), memory_retrieval(retrieval),
          apply_memory(apply) {}
};

// Outcome and per-step host times of a pipeline call (reference :58-85).
struct ExecutionResult {
    bool success = false;
    std::string error_message;
    double total_time_ms = 0.0;

    double build_memory_time_ms = 0.0;
    double compute_score_time_ms = 0.0;
    double retrieval_time_ms = 0.0;
    double apply_memory_time_ms = 0.0;

    static ExecutionResult Success(double time_ms = 0.0) {
        ExecutionResult r;
        r.success = true;
        r.total_time_ms = time_ms;
        return r;
    }
    static ExecutionResult Failure(const std::string& msg) {
        ExecutionResult r;
        r.success = false;
        r.error_message = msg;
        return r;
    }
};

template <typename RetDataT, typename MemoryT, typename QueryT, typename ScoreT, typename IndexT,
          typename InputT, typename OutputT>
class MemoryManager {
public:
    using RetrievedData = RetDataT;
    using Memory = MemoryT;
    using Query = QueryT;
    using Score = ScoreT;
    using Index = IndexT;
    using Input = InputT;
    using Output = OutputT;

    using BuildMemoryStepT = step::BuildMemory<RetDataT, MemoryT>;
    using ComputeScoreStepT = step::ComputeScore<MemoryT, QueryT, ScoreT>;
    using MemoryRetrievalStepT = step::MemoryRetrieval<ScoreT, IndexT>;
    using ApplyMemoryStepT = step::ApplyMemory<RetDataT, IndexT, InputT, OutputT>;

    explicit MemoryManager(const std::string& schedule_path = "") : kernel_config_() {
        if (!schedule_path.empty()) schedule_config_ = ScheduleConfig::load_from_file(schedule_path);
    }
    MemoryManager(const std::string& schedule_path, const PipelineKernelConfig& config)
        : kernel_config_(config) {
        if (!schedule_path.empty()) schedule_config_ = ScheduleConfig::load_from_file(schedule_path);
    }
    virtual ~MemoryManager() = default;

    // ----- kernel configuration
    void set_kernel_config(const PipelineKernelConfig& config) { kernel_config_ = config; }
    void set_build_memory_kernel(step::KernelType type) { kernel_config_.build_memory = type; }
    void set_compute_score_kernel(step::KernelType type) { kernel_config_.compute_score = type; }
    void set_memory_retrieval_kernel(step::KernelType type) {
        kernel_config_.memory_retrieval = type;
    }
    void set_apply_memory_kernel(step::KernelType type) { kernel_config_.apply_memory = type; }
    const PipelineKernelConfig& get_kernel_config() const { return kernel_config_; }
    const ScheduleConfig& get_schedule_config() const { return schedule_config_; }
    // Rules in place of a schedule file (an addition of this build).
    void set_schedule_config(const ScheduleConfig& config) { schedule_config_ = config; }

    // Whether an all-GPU manage_memory_and_apply may run as one
    // device-resident pass (default on; an addition of this build).
    void set_device_chain(bool enabled) { device_chain_ = enabled; }
    bool device_chain() const { return device_chain_; }

    // ----- step handlers
    void set_build_memory_step(std::shared_ptr<BuildMemoryStepT> step) {
        build_memory_step_ = std::move(step);
    }
    void set_compute_score_step(std::shared_ptr<ComputeScoreStepT> step) {
        compute_score_step_ = std::move(step);
    }
    void set_memory_retrieval_step(std::shared_ptr<MemoryRetrievalStepT> step) {
        memory_retrieval_step_ = std::move(step);
    }
    void set_apply_memory_step(std::shared_ptr<ApplyMemoryStepT> step) {
        apply_memory_step_ = std::move(step);
    }

    // ----- factories (override to provide the steps)
    virtual std::shared_ptr<BuildMemoryStepT> create_build_memory_step() { return nullptr; }
    virtual std::shared_ptr<ComputeScoreStepT> create_compute_score_step() { return nullptr; }
    virtual std::shared_ptr<MemoryRetrievalStepT> create_memory_retrieval_step() {
        return nullptr;
    }
    virtual std::shared_ptr<ApplyMemoryStepT> create_apply_memory_step() { return nullptr; }

    // Sizes the schedule rules are matched on.
    virtual int ret_data_size(const RetDataT& retrieved_data) = 0;
    virtual int memory_size(const MemoryT& memory) = 0;

    // ----- entry points (reference :297-480)

    // retrieved_data -> memory.
    ExecutionResult build_memory(const RetDataT& retrieved_data, MemoryT& memory,
                                 bool verbose = false) {
        if (!schedule_config_.build_memory_rules.empty())
            set_build_memory_kernel(step::string_to_kernel_type(
                schedule_config_.get_build_memory_config(ret_data_size(retrieved_data))));
        return run_build(retrieved_data, memory, verbose);
    }

    // (memory, query) -> scores -> indices -> (retrieved_data, indices, input) -> output.
    ExecutionResult manage_memory_and_apply(const RetDataT& retrieved_data, const MemoryT& memory,
                                            const QueryT& query, const InputT& input,
                                            OutputT& output, bool verbose = false) {
        if (!schedule_config_.manage_memory_and_apply_rules.empty()) {
            const auto config = schedule_config_.get_manage_memory_and_apply_config(
                ret_data_size(retrieved_data), memory_size(memory));
            set_compute_score_kernel(step::string_to_kernel_type(config[0]));
            set_memory_retrieval_kernel(step::string_to_kernel_type(config[1]));
            set_apply_memory_kernel(step::string_to_kernel_type(config[2]));
        }
        return run_manage(retrieved_data, memory, query, input, output, verbose);
    }

    // build_memory, then manage_memory_and_apply on the memory it built.
    ExecutionResult build_and_apply_memory(const RetDataT& retrieved_data, const QueryT& query,
                                           const InputT& input, OutputT& output,
                                           bool verbose = false) {
        if (!schedule_config_.build_and_apply_memory_rules.empty()) {
            const auto config =
                schedule_config_.get_build_and_apply_memory_config(ret_data_size(retrieved_data));
            set_build_memory_kernel(step::string_to_kernel_type(config[0]));
            set_compute_score_kernel(step::string_to_kernel_type(config[1]));
            set_memory_retrieval_kernel(step::string_to_kernel_type(config[2]));
            set_apply_memory_kernel(step::string_to_kernel_type(config[3]));
        }
        MemoryT memory;
        ExecutionResult build_result = run_build(retrieved_data, memory, verbose);
        if (!build_result.success) return build_result;
        ExecutionResult result = run_manage(retrieved_data, memory, query, input, output, verbose);
        if (!result.success) return result;
        result.build_memory_time_ms = build_result.build_memory_time_ms;
        result.total_time_ms = build_result.total_time_ms + result.total_time_ms;
        return result;
    }

    // Each configured step's functional test against the given expected
    // outputs (reference :496-555).
    bool run_functional_tests(const RetDataT& retrieved_data, MemoryT& expected_memory,
                              const QueryT& query, ScoreT& expected_scores,
                              IndexT& expected_indices, const InputT& input,
                              OutputT& expected_output, bool verbose = false) {
        bool all_passed = true;
        auto report = [&](const char* name, int status) {
            if (status != 0) {
                if (verbose) std::clog << "[MemoryManager] " << name << " test FAILED" << std::endl;
                all_passed = false;
            } else if (verbose) {
                std::clog << "[MemoryManager] " << name << " test PASSED" << std::endl;
            }
        };
        if (auto s = get_or_create_build_memory_step())
            report("BuildMemory", s->execute(retrieved_data, expected_memory, true, verbose));
        if (auto s = get_or_create_compute_score_step())
            report("ComputeScore", s->execute(expected_memory, query, expected_scores, true, verbose));
        if (auto s = get_or_create_memory_retrieval_step())
            report("MemoryRetrieval", s->execute(expected_scores, expected_indices, true, verbose));
        if (auto s = get_or_create_apply_memory_step())
            report("ApplyMemory", s->execute(retrieved_data, expected_indices, input,
                                             expected_output, true, verbose));
        return all_passed;
    }

protected:
    // compute_score -> memory_retrieval -> apply_memory as one pass on the
    // device, called when all three kernels are GPU and the device chain is
    // enabled.  Returns false to take the step-by-step route; on true it has
    // written `output` and the step times of `result`.
    virtual bool run_device_chain(const RetDataT&, const MemoryT&, const QueryT&, const InputT&,
                                  OutputT&, ExecutionResult&, bool /*verbose*/) {
        return false;
    }

    std::shared_ptr<BuildMemoryStepT> build_memory_step_;
    std::shared_ptr<ComputeScoreStepT> compute_score_step_;
    std::shared_ptr<MemoryRetrievalStepT> memory_retrieval_step_;
    std::shared_ptr<ApplyMemoryStepT> apply_memory_step_;

    PipelineKernelConfig kernel_config_;
    ScheduleConfig schedule_config_;
    bool device_chain_ = true;

    std::shared_ptr<BuildMemoryStepT> get_or_create_build_memory_step() {
        if (!build_memory_step_) build_memory_step_ = create_build_memory_step();
        if (build_memory_step_) build_memory_step_->set_current_kernel(kernel_config_.build_memory);
        return build_memory_step_;
    }
    std::shared_ptr<ComputeScoreStepT> get_or_create_compute_score_step() {
        if (!compute_score_step_) compute_score_step_ = create_compute_score_step();
        if (compute_score_step_)
            compute_score_step_->set_current_kernel(kernel_config_.compute_score);
        return compute_score_step_;
    }
    std::shared_ptr<MemoryRetrievalStepT> get_or_create_memory_retrieval_step() {
        if (!memory_retrieval_step_) memory_retrieval_step_ = create_memory_retrieval_step();
        if (memory_retrieval_step_)
            memory_retrieval_step_->set_current_kernel(kernel_config_.memory_retrieval);
        return memory_retrieval_step_;
    }
    std::shared_ptr<ApplyMemoryStepT> get_or_create_apply_memory_step() {
        if (!apply_memory_step_) apply_memory_step_ = create_apply_memory_step();
        if (apply_memory_step_) apply_memory_step_->set_current_kernel(kernel_config_.apply_memory);
        return apply_memory_step_;
    }

private:
    using Clock = std::chrono::high_resolution_clock;
    static double ms_since(Clock::time_point t0) {
        return std::chrono::duration<double, std::milli>(Clock::now() - t0).count();
    }

    ExecutionResult run_build(const RetDataT& retrieved_data, MemoryT& memory, bool verbose) {
        auto step = get_or_create_build_memory_step();
        if (!step) return ExecutionResult::Failure("BuildMemory step not configured");
        const auto t0 = Clock::now();
        const int status = step->execute(retrieved_data, memory, false, verbose);
        const double time_ms = ms_since(t0);
        if (status != 0) return ExecutionResult::Failure("BuildMemory execution failed");
        ExecutionResult result = ExecutionResult::Success(time_ms);
        result.build_memory_time_ms = time_ms;
        return result;
    }

    ExecutionResult run_manage(const RetDataT& retrieved_data, const MemoryT& memory,
                               const QueryT& query, const InputT& input, OutputT& output,
                               bool verbose) {
        ExecutionResult result;
        result.success = true;
        const bool all_gpu = kernel_config_.compute_score == step::KernelType::GPU &&
                             kernel_config_.memory_retrieval == step::KernelType::GPU &&
                             kernel_config_.apply_memory == step::KernelType::GPU;
        if (all_gpu && device_chain_ &&
            run_device_chain(retrieved_data, memory, query, input, output, result, verbose)) {
            result.total_time_ms =
                result.compute_score_time_ms + result.retrieval_time_ms + result.apply_memory_time_ms;
            return result;
        }

        auto score_step = get_or_create_compute_score_step();
        if (!score_step) return ExecutionResult::Failure("ComputeScore step not configured");
        ScoreT scores;
        auto t0 = Clock::now();
        if (score_step->execute(memory, query, scores, false, verbose) != 0)
            return ExecutionResult::Failure("ComputeScore execution failed");
        result.compute_score_time_ms = ms_since(t0);

        auto retrieval_step = get_or_create_memory_retrieval_step();
        if (!retrieval_step) return ExecutionResult::Failure("MemoryRetrieval step not configured");
        IndexT indices;
        t0 = Clock::now();
        if (retrieval_step->execute(scores, indices, false, verbose) != 0)
            return ExecutionResult::Failure("MemoryRetrieval execution failed");
        result.retrieval_time_ms = ms_since(t0);

        auto apply_step = get_or_create_apply_memory_step();
        if (!apply_step) return ExecutionResult::Failure("ApplyMemory step not configured");
        t0 = Clock::now();
        if (apply_step->execute(retrieved_data, indices, input, output, false, verbose) != 0)
            return ExecutionResult::Failure("ApplyMemory execution failed");
        result.apply_memory_time_ms = ms_since(t0);

        result.total_time_ms =
            result.compute_score_time_ms + result.retrieval_time_ms + result.apply_memory_time_ms;
        return result;
    }
};

}  // namespace deploy
}  // namespace heteromm

#endif  // HETEROMM_B200_DEPLOY_MEMORY_MANAGER_H_
