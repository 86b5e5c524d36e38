// util.h — kernel-type selection of the heteromm steps (B200 build);
// interface of the reference's steps/util.h (the conversion is `inline` here:
// the reference defines it non-inline in a header, :30).
#ifndef HETEROMM_B200_DEV_STEPS_UTIL_H_
#define HETEROMM_B200_DEV_STEPS_UTIL_H_

#include <iostream>
#include <string>

namespace heteromm {
namespace step {

enum class KernelType { CPU, GPU, FPGA };

inline std::string kernel_type_to_string(KernelType type) {
    switch (type) {
        case KernelType::CPU: return "CPU";
        case KernelType::GPU: return "GPU";
        case KernelType::FPGA: return "FPGA";
    }
    return "UNKNOWN";
}

inline KernelType string_to_kernel_type(const std::string& device) {
    if (device == "gpu") return KernelType::GPU;
    if (device == "fpga") return KernelType::FPGA;
    return KernelType::CPU;
}

namespace detail {
// Runs the functional test of a step: keep the caller's expected output,
// compute into `out` with the test kernel, compare.  0 on a match, 1 otherwise
// (the contract of every reference step's execute(..., true, ...)).
template <typename Out, typename Run>
int functional_test(const char* step, Out& out, bool verbose, Run&& run) {
    Out expected = out;
    if (verbose) std::clog << "[" << step << "] Running functional test kernel." << std::endl;
    run();
    const bool ok = out.is_equal(expected);
    if (verbose)
        std::clog << "[" << step << "] Functional test " << (ok ? "passed" : "failed") << "."
                  << std::endl;
    return ok ? 0 : 1;
}

inline void log_kernel(const char* step, KernelType k, bool verbose, bool done) {
    if (verbose)
        std::clog << "[" << step << "] " << (done ? "" : "Running ") << kernel_type_to_string(k)
                  << (done ? " kernel completed." : " kernel.") << std::endl;
}
}  // namespace detail

}  // namespace step
}  // namespace heteromm

#endif  // HETEROMM_B200_DEV_STEPS_UTIL_H_
