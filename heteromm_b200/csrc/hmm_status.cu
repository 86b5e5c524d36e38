// hmm_status.cu — thread-local last-error message, version, device queries.
#include <stdarg.h>
#include <stdio.h>

#include "hmm_common.cuh"

namespace hmm {

static thread_local char g_last_error[512] = "";

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

}  // namespace hmm

extern "C" const char* hmm_last_error(void) { return hmm::g_last_error; }

extern "C" const char* hmm_version(void) { return "heteromm-b200 0.1.0 sm_100a"; }
