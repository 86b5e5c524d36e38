// device.h — shared plumbing of the GPU adapters behind the step classes:
// status -> exception mapping, a grow-only per-thread device scratch and
// per-thread device mirrors of unchanged host rows.
// Adapters are synchronous, like the reference steps: upload, run on the
// legacy default stream, copy results back.
#ifndef HETEROMM_B200_SRC_DEVICE_H_
#define HETEROMM_B200_SRC_DEVICE_H_

#include <cuda_runtime_api.h>

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include "heteromm_cuda.h"

namespace heteromm {
namespace gpu {

// Nonzero status -> std::runtime_error carrying hmm_last_error(), the
// reference's way of failing a kernel (exceptions out of run_*_kernel).
inline void check(hmm_status_t st, const char* what) {
    if (st != HMM_OK) throw std::runtime_error(std::string(what) + ": " + hmm_last_error());
}

inline void check_cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess)
        throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// A device allocation reused across calls (grows, never shrinks).
class DeviceBuffer {
public:
    DeviceBuffer() = default;
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
    ~DeviceBuffer() {
        if (p_) cudaFree(p_);
    }
    void* get(size_t bytes) {
        if (bytes > n_) {
            if (p_) cudaFree(p_);
            p_ = nullptr;
            n_ = 0;
            check_cuda(cudaMalloc(&p_, bytes < 256 ? 256 : bytes), "cudaMalloc");
            n_ = bytes < 256 ? 256 : bytes;
        }
        return p_;
    }
    size_t size() const { return n_; }

private:
    void* p_ = nullptr;
    size_t n_ = 0;
};

// Named scratch slots of the calling thread.
enum Slot { kMem, kQuery, kOut, kOut2, kIdx, kWork, kAux, kAux2, kAux3, kSlots };
inline DeviceBuffer& scratch(Slot s) {
    thread_local DeviceBuffer buf[kSlots];
    return buf[s];
}

// Bytes this thread has copied host -> device through the adapters (read by
// h2d_bytes(), deploy/device_chain.h).
inline uint64_t& h2d_counter() {
    thread_local uint64_t n = 0;
    return n;
}

inline void copy_h2d(void* dev, const void* host, size_t bytes) {
    if (!bytes) return;
    check_cuda(cudaMemcpy(dev, host, bytes, cudaMemcpyHostToDevice), "cudaMemcpy H2D");
    h2d_counter() += bytes;
}

template <typename T>
T* upload(Slot s, const std::vector<T>& host) {
    T* d = static_cast<T*>(scratch(s).get(sizeof(T) * (host.empty() ? 1 : host.size())));
    copy_h2d(d, host.data(), sizeof(T) * host.size());
    return d;
}

template <typename T>
T* upload(Slot s, const T* host, size_t n) {
    T* d = static_cast<T*>(scratch(s).get(sizeof(T) * (n ? n : 1)));
    copy_h2d(d, host, sizeof(T) * n);
    return d;
}

template <typename T>
void download(std::vector<T>& host, const T* dev) {
    if (!host.empty())
        check_cuda(cudaMemcpy(host.data(), dev, sizeof(T) * host.size(), cudaMemcpyDeviceToHost),
                   "cudaMemcpy D2H");
}

// Device copies of recently used row arrays, per thread: up to kMirrors,
// keyed by the owning object's generation (renewed by every change of its
// contents), which of its arrays it is (tag) and the packed shape; the least
// recently used is replaced.  A hit skips the packing and the upload of
// unchanged rows.
enum MirrorTag { kRows = 1, kKeys = 2, kValues = 3 };
struct Mirror {
    uint64_t gen = 0;
    int tag = 0;
    size_t n = 0, d = 0;
    uint64_t used = 0;
    DeviceBuffer buf;
};
constexpr int kMirrors = 8;

// The mirror of (gen, tag, n, d); *hit tells whether it already holds the data.
inline Mirror& mirror(uint64_t gen, int tag, size_t n, size_t d, bool* hit) {
    thread_local Mirror m[kMirrors];
    thread_local uint64_t clock = 0;
    ++clock;
    for (auto& x : m)
        if (x.gen != 0 && x.gen == gen && x.tag == tag && x.n == n && x.d == d) {
            x.used = clock;
            *hit = true;
            return x;
        }
    Mirror* lru = &m[0];
    for (auto& x : m)
        if (x.used < lru->used) lru = &x;
    lru->gen = 0;   // claimed; valid once the caller has filled it
    lru->used = clock;
    *hit = false;
    return *lru;
}

// Rows of a vector-of-vectors packed into one row-major array; every row
// must have `cols` values.
template <typename T>
std::vector<T> pack_rows(const std::vector<std::vector<T>>& rows, size_t cols, const char* what) {
    std::vector<T> out;
    out.reserve(rows.size() * cols);
    for (const auto& r : rows) {
        if (r.size() < cols)
            throw std::invalid_argument(std::string(what) + ": a row is shorter than the query");
        out.insert(out.end(), r.begin(), r.begin() + (std::ptrdiff_t)cols);
    }
    return out;
}

// The first d columns of `rows` (owned by an object of generation `gen`) on
// the device: the cached mirror when it is still valid, else packed and
// uploaded into one.  n = rows.size() > 0 and d > 0.
inline const float* device_rows(const std::vector<std::vector<float>>& rows, uint64_t gen,
                                int tag, size_t d, const char* what) {
    const size_t n = rows.size();
    bool hit = false;
    Mirror& m = mirror(gen, tag, n, d, &hit);
    float* dev = static_cast<float*>(m.buf.get(sizeof(float) * n * d));
    if (!hit) {
        const std::vector<float> packed = pack_rows(rows, d, what);
        copy_h2d(dev, packed.data(), sizeof(float) * n * d);
        m.gen = gen;
        m.tag = tag;
        m.n = n;
        m.d = d;
    }
    return dev;
}

// Registers n x d device rows (already computed on the device) as the mirror
// of an object of generation `gen`, so the next step that reads that object
// finds them resident.
inline void adopt_rows(uint64_t gen, int tag, size_t n, size_t d, const float* src) {
    if (!n || !d) return;
    bool hit = false;
    Mirror& m = mirror(gen, tag, n, d, &hit);
    float* dev = static_cast<float*>(m.buf.get(sizeof(float) * n * d));
    check_cuda(cudaMemcpy(dev, src, sizeof(float) * n * d, cudaMemcpyDeviceToDevice),
               "cudaMemcpy D2D");
    m.gen = gen;
    m.tag = tag;
    m.n = n;
    m.d = d;
}

}  // namespace gpu
}  // namespace heteromm

#endif  // HETEROMM_B200_SRC_DEVICE_H_
