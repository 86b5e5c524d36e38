// device.h — shared plumbing of the GPU adapters behind the step classes:
// status -> exception mapping, a grow-only device scratch and device mirrors
// of unchanged host rows, both per thread and GPU.
// Adapters are synchronous, like the reference steps: upload, run on the
// legacy default stream, copy results back.
#ifndef HETEROMM_B200_SRC_DEVICE_H_
#define HETEROMM_B200_SRC_DEVICE_H_

#include <cuda_runtime_api.h>

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <memory>
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
    // Grows to at least `bytes` (by half again at least, so appends amortise),
    // keeping the first `keep` bytes.
    void* grow_keep(size_t bytes, size_t keep) {
        if (bytes <= n_) return p_;
        const size_t cap = bytes > n_ + n_ / 2 ? bytes : n_ + n_ / 2;
        void* q = nullptr;
        check_cuda(cudaMalloc(&q, cap), "cudaMalloc");
        if (keep && p_) {
            const cudaError_t e = cudaMemcpy(q, p_, keep, cudaMemcpyDeviceToDevice);
            if (e != cudaSuccess) {
                cudaFree(q);
                check_cuda(e, "cudaMemcpy D2D");
            }
        }
        if (p_) cudaFree(p_);
        p_ = q;
        n_ = cap;
        return p_;
    }
    void* ptr() const { return p_; }
    size_t size() const { return n_; }

private:
    void* p_ = nullptr;
    size_t n_ = 0;
};

// The calling thread's instance of T for the current device, created on
// first use there.  Device buffers, the events recorded on a device's streams
// and the copies of data held on a device live in these, so a thread that
// moves between GPUs (cudaSetDevice) never hands one device's memory or
// events to another's kernels.
inline int current_device() {
    int d = 0;
    check_cuda(cudaGetDevice(&d), "cudaGetDevice");
    return d;
}
template <typename T>
T& per_device() {
    thread_local std::vector<std::unique_ptr<T>> v;
    const int d = current_device();
    if ((size_t)d >= v.size()) v.resize((size_t)d + 1);
    if (!v[(size_t)d]) v[(size_t)d] = std::make_unique<T>();
    return *v[(size_t)d];
}

// Named scratch slots of the calling thread on the current device.
enum Slot { kMem, kQuery, kOut, kOut2, kIdx, kWork, kAux, kAux2, kAux3, kSlots };
struct ScratchSet {
    DeviceBuffer buf[kSlots];
};
inline DeviceBuffer& scratch(Slot s) { return per_device<ScratchSet>().buf[s]; }

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

// Device copies of recently used row arrays, per thread and device: up to kMirrors,
// keyed by the owning object's generation (renewed by every change of its
// contents), which of its arrays it is (tag) and the packed shape.  A hit skips
// the packing and the upload of unchanged rows.  A new copy replaces the least
// recently used one, among copies not held if there are any: copies of objects
// tagged DataLocation::GPU_MEM are held.
enum MirrorTag { kRows = 1, kKeys = 2, kValues = 3 };
struct Mirror {
    uint64_t gen = 0;
    int tag = 0;
    size_t n = 0, d = 0;
    uint64_t used = 0;
    bool held = false;
    DeviceBuffer buf;
};
constexpr int kMirrors = 8;
struct MirrorTable {
    Mirror m[kMirrors];
    uint64_t clock = 0;
};
inline MirrorTable& mirror_table() { return per_device<MirrorTable>(); }

inline Mirror* find_mirror(uint64_t gen, int tag, size_t n, size_t d) {
    MirrorTable& t = mirror_table();
    for (auto& x : t.m)
        if (x.gen != 0 && x.gen == gen && x.tag == tag && x.n == n && x.d == d) {
            x.used = ++t.clock;
            return &x;
        }
    return nullptr;
}

// A slot for a new copy, emptied (gen 0) until the caller fills it.
inline Mirror& claim_mirror() {
    MirrorTable& t = mirror_table();
    Mirror* lru = nullptr;
    for (int pass = 0; pass < 2 && !lru; ++pass)   // pass 0: copies not held
        for (auto& x : t.m)
            if ((pass == 1 || !x.held || x.gen == 0) && (!lru || x.used < lru->used)) lru = &x;
    lru->gen = 0;
    lru->held = false;
    lru->used = ++t.clock;
    return *lru;
}

// The mirror of (gen, tag, n, d); *hit tells whether it already holds the data.
inline Mirror& mirror(uint64_t gen, int tag, size_t n, size_t d, bool* hit) {
    if (Mirror* x = find_mirror(gen, tag, n, d)) {
        *hit = true;
        return *x;
    }
    *hit = false;
    return claim_mirror();
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

// Two pinned host buffers of kStageBytes per thread and GPU, with an event each: a
// full upload packs the next chunk of rows into one while the copy from the
// other runs, so packing and the host->device transfer overlap, and the copies
// run from pinned memory at full link speed.
constexpr size_t kStageBytes = size_t(8) << 20;
struct PinnedStage {
    void* buf[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    bool pending[2] = {false, false};
    PinnedStage() {
        for (int i = 0; i < 2; ++i) {
            check_cuda(cudaMallocHost(&buf[i], kStageBytes), "cudaMallocHost");
            check_cuda(cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming), "cudaEventCreate");
        }
    }
    ~PinnedStage() {
        for (int i = 0; i < 2; ++i) {
            if (done[i]) {
                if (pending[i]) cudaEventSynchronize(done[i]);
                cudaEventDestroy(done[i]);
            }
            if (buf[i]) cudaFreeHost(buf[i]);
        }
    }
    void wait(int i) {
        if (pending[i]) check_cuda(cudaEventSynchronize(done[i]), "cudaEventSynchronize");
        pending[i] = false;
    }
};
inline PinnedStage& pinned_stage() { return per_device<PinnedStage>(); }

// The first d columns of rows[0..n) into dev (n x d floats); every row must
// have d values (checked before anything is copied).
inline void upload_rows(float* dev, const std::vector<std::vector<float>>& rows, size_t d,
                        const char* what) {
    const size_t n = rows.size();
    for (const auto& r : rows)
        if (r.size() < d)
            throw std::invalid_argument(std::string(what) + ": a row is shorter than the query");
    const size_t row_bytes = sizeof(float) * d;
    if (row_bytes > kStageBytes) {   // rows wider than a stage: one packed pageable copy
        const std::vector<float> packed = pack_rows(rows, d, what);
        copy_h2d(dev, packed.data(), sizeof(float) * n * d);
        return;
    }
    PinnedStage& st = pinned_stage();
    const size_t per = kStageBytes / row_bytes;
    int b = 0;
    for (size_t r0 = 0; r0 < n; r0 += per, b ^= 1) {
        const size_t r1 = r0 + per < n ? r0 + per : n;
        st.wait(b);
        float* h = static_cast<float*>(st.buf[b]);
        for (size_t r = r0; r < r1; ++r) std::memcpy(h + (r - r0) * d, rows[r].data(), row_bytes);
        check_cuda(cudaMemcpyAsync(dev + r0 * d, h, (r1 - r0) * row_bytes, cudaMemcpyHostToDevice,
                                   nullptr),
                   "cudaMemcpyAsync H2D");
        check_cuda(cudaEventRecord(st.done[b], nullptr), "cudaEventRecord");
        st.pending[b] = true;
    }
    st.wait(0);
    st.wait(1);
    h2d_counter() += sizeof(float) * n * d;
}

// The first d columns of `rows` (owned by an object of generation `gen`) on
// the device: the cached mirror when it is still valid, else uploaded into
// one.  n = rows.size() > 0 and d > 0; `held` marks the copy as held.
inline const float* device_rows(const std::vector<std::vector<float>>& rows, uint64_t gen,
                                int tag, size_t d, const char* what, bool held = false) {
    const size_t n = rows.size();
    bool hit = false;
    Mirror& m = mirror(gen, tag, n, d, &hit);
    float* dev = static_cast<float*>(m.buf.get(sizeof(float) * n * d));
    if (!hit) {
        upload_rows(dev, rows, d, what);
        m.gen = gen;
        m.tag = tag;
        m.n = n;
        m.d = d;
    }
    m.held = m.held || held;
    return dev;
}

// Replays the row log of a flat memory from entry k onto mirror x (its rows as
// of log[k].from): appended rows are copied up in one transfer per run of
// appends, erased rows close up on the device.  False if the log does not fit
// the mirror (the caller then uploads in full).
template <typename Log>
bool replay_rows(Mirror& x, const Log& log, size_t k, size_t d) {
    size_t cur = x.n;
    std::vector<float> pend;   // a run of appended rows awaiting one copy
    size_t pend_at = 0;
    auto flush = [&]() {
        if (pend.empty()) return;
        const size_t rows_after = pend_at + pend.size() / d;
        float* base = static_cast<float*>(
            x.buf.grow_keep(sizeof(float) * rows_after * d, sizeof(float) * pend_at * d));
        copy_h2d(base + pend_at * d, pend.data(), sizeof(float) * pend.size());
        pend.clear();
    };
    for (; k < log.size(); ++k) {
        const auto& e = log[k];
        switch (e.kind) {
            case Log::value_type::Append:
                if (e.index != cur || e.row.size() < d) return false;
                if (pend.empty()) pend_at = cur;
                pend.insert(pend.end(), e.row.begin(), e.row.begin() + (std::ptrdiff_t)d);
                ++cur;
                break;
            case Log::value_type::PopLast:
                flush();
                if (cur == 0) return false;
                --cur;
                break;
            case Log::value_type::Erase: {
                flush();
                if (e.index >= cur) return false;
                const size_t tail = cur - e.index - 1;
                if (tail) {
                    float* base = static_cast<float*>(x.buf.ptr());
                    float* tmp = static_cast<float*>(scratch(kAux3).get(sizeof(float) * tail * d));
                    check_cuda(cudaMemcpy(tmp, base + (e.index + 1) * d, sizeof(float) * tail * d,
                                          cudaMemcpyDeviceToDevice),
                               "cudaMemcpy D2D");
                    check_cuda(cudaMemcpy(base + e.index * d, tmp, sizeof(float) * tail * d,
                                          cudaMemcpyDeviceToDevice),
                               "cudaMemcpy D2D");
                }
                --cur;
                break;
            }
        }
    }
    flush();
    x.n = cur;
    return true;
}

// The first d columns of a flat memory's rows on the device (n, d > 0): the
// mirror of its current generation; else a mirror of an earlier generation
// brought up to date from the memory's row log; else a full upload.
template <typename Mem>
const float* device_flat_rows(const Mem& memory, size_t d, const char* what) {
    const auto& rows = memory.data_ref();
    const size_t n = rows.size();
    const uint64_t gen = memory.generation();
    const bool held = memory.get_device() == decltype(memory.get_device())::GPU_MEM;
    if (Mirror* x = find_mirror(gen, kRows, n, d)) {
        x->held = x->held || held;
        return static_cast<const float*>(x->buf.ptr());
    }
    const auto& log = memory.row_deltas();
    if (!log.empty() && log.back().to == gen) {
        size_t j = log.size() - 1;   // start of the unbroken run of changes ending at gen
        while (j > 0 && log[j - 1].to == log[j].from) --j;
        MirrorTable& t = mirror_table();
        for (auto& x : t.m) {
            if (x.gen == 0 || x.tag != kRows || x.d != d) continue;
            size_t k = j;
            while (k < log.size() && log[k].from != x.gen) ++k;
            if (k == log.size()) continue;
            x.gen = 0;   // invalid until the replay completes
            if (replay_rows(x, log, k, d) && x.n == n) {
                x.gen = gen;
                x.used = ++t.clock;
                x.held = x.held || held;
                return static_cast<const float*>(x.buf.ptr());
            }
        }
    }
    return device_rows(rows, gen, kRows, d, what, held);
}

// Registers n x d device rows (already computed on the device) as the mirror
// of an object of generation `gen`, so the next step that reads that object
// finds them resident.
inline void adopt_rows(uint64_t gen, int tag, size_t n, size_t d, const float* src) {
    if (!n || !d) return;
    Mirror& m = claim_mirror();
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
