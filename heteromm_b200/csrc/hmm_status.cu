// hmm_status.cu — thread-local last-error message, version, device queries.
#include <stdarg.h>
#include <stdio.h>

#include <atomic>
#include <mutex>
#include <vector>

#include "hmm_common.cuh"

namespace hmm {

static thread_local char g_last_error[512] = "";
// Kernels launched by this library since load (every launch site calls
// check_launch exactly once).
static std::atomic<int64_t> g_launches{0};

// Event pairs recorded around the dominant scoring kernel while profiling is on.
struct ProfileState {
    std::mutex mu;
    bool on = false;
    std::vector<cudaEvent_t> free_events;
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> pending;
};
static ProfileState g_prof;

static cudaEvent_t take_event() {
    cudaEvent_t e = nullptr;
    if (!g_prof.free_events.empty()) {
        e = g_prof.free_events.back();
        g_prof.free_events.pop_back();
    } else if (cudaEventCreate(&e) != cudaSuccess) {
        e = nullptr;
    }
    return e;
}

ProfileMark profile_begin(cudaStream_t st) {
    std::lock_guard<std::mutex> lk(g_prof.mu);
    ProfileMark m{nullptr, nullptr};
    if (!g_prof.on) return m;
    m.start = take_event();
    m.stop = take_event();
    if (m.start) cudaEventRecord(m.start, st);
    return m;
}

void profile_end(const ProfileMark& m, cudaStream_t st) {
    if (!m.start || !m.stop) return;
    std::lock_guard<std::mutex> lk(g_prof.mu);
    cudaEventRecord(m.stop, st);
    g_prof.pending.emplace_back(m.start, m.stop);
}

hmm_status_t set_error(hmm_status_t st, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return st;
}

hmm_status_t check_launch(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return set_error(HMM_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return HMM_OK;
}

int device_sm_count() {
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (cache[dev] == 0) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            v <= 0)
            v = 148;
        cache[dev] = v;
    }
    return cache[dev];
}

constexpr int64_t DEFAULT_WAIT_NS = 2000000000ll;   // far above any legitimate wait
std::atomic<int64_t> g_wait_ns{DEFAULT_WAIT_NS};

uint64_t wait_limit_ns() { return (uint64_t)g_wait_ns.load(std::memory_order_relaxed); }

}  // namespace hmm

extern "C" hmm_status_t hmm_debug_set_wait_limit_ns(int64_t ns) {
    hmm::g_wait_ns.store(ns < 0 ? hmm::DEFAULT_WAIT_NS : ns, std::memory_order_relaxed);
    return HMM_OK;
}

extern "C" const char* hmm_last_error(void) { return hmm::g_last_error; }

extern "C" const char* hmm_version(void) { return "heteromm-b200 0.1.0 sm_100a"; }

extern "C" int64_t hmm_kernel_launches(void) {
    return hmm::g_launches.load(std::memory_order_relaxed);
}

extern "C" hmm_status_t hmm_profile_enable(int enable) {
    std::lock_guard<std::mutex> lk(hmm::g_prof.mu);
    hmm::g_prof.on = enable != 0;
    return HMM_OK;
}

extern "C" hmm_status_t hmm_profile_read(double* total_ms, int64_t* launches) {
    if (!total_ms || !launches) return hmm::set_error(HMM_ERR_INVALID, "null output pointer");
    std::lock_guard<std::mutex> lk(hmm::g_prof.mu);
    double sum = 0.0;
    int64_t n = 0;
    hmm_status_t st = HMM_OK;
    for (auto& pr : hmm::g_prof.pending) {
        float ms = 0.f;
        if (st == HMM_OK) {
            cudaError_t e = cudaEventSynchronize(pr.second);
            if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, pr.first, pr.second);
            if (e != cudaSuccess)
                st = hmm::set_error(HMM_ERR_CUDA, "profile events: %s", cudaGetErrorString(e));
        }
        sum += ms;
        ++n;
        hmm::g_prof.free_events.push_back(pr.first);
        hmm::g_prof.free_events.push_back(pr.second);
    }
    hmm::g_prof.pending.clear();
    *total_ms = sum;
    *launches = n;
    return st;
}
