// base_types.h — data-type base of the heteromm step API (B200 build).
//
// Same interface as the reference's toolchain/frontend/dev/types/base_types.h:
// every datum carries its device location and exposes its contents by copy
// (export_data) and replacement (set_data).  data_ref() is an addition of this
// build: a const reference to the contents for the GPU adapters, which read
// large memories without the deep copy export_data makes, and generation(): a
// process-unique number that every construction, copy and mutation renews, so
// the GPU adapters can keep device copies of unchanged contents across calls.
#ifndef HETEROMM_B200_DEV_TYPES_BASE_TYPES_H_
#define HETEROMM_B200_DEV_TYPES_BASE_TYPES_H_

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <string>
#include <type_traits>
#include <vector>

namespace heteromm {
namespace data_type {

enum class DataLocation { SYS_DRAM, GPU_MEM, FPGA_MEM };

// Next value of the process-wide generation counter (never 0).
inline uint64_t next_generation() {
    static std::atomic<uint64_t> counter{0};
    return counter.fetch_add(1, std::memory_order_relaxed) + 1;
}

template <typename T>
class BaseType {
public:
    BaseType() = default;
    BaseType(const BaseType& o) : device_(o.device_), data(o.data) {}
    BaseType& operator=(const BaseType& o) {
        device_ = o.device_;
        data = o.data;
        touch();
        return *this;
    }
    virtual ~BaseType() = default;
    virtual std::string type_name() const = 0;
    virtual size_t get_size() const = 0;

    DataLocation get_device() const { return device_; }
    void set_device(DataLocation device) { device_ = device; }

    T export_data() const { return data; }
    void set_data(const T& new_data) {
        data = new_data;
        touch();
    }
    const T& data_ref() const { return data; }
    // Changes whenever the contents may have changed (and differs between
    // objects), so (generation, shape) identifies the contents.
    uint64_t generation() const { return generation_; }

protected:
    void touch() { generation_ = next_generation(); }

    DataLocation device_ = DataLocation::SYS_DRAM;
    T data;

private:
    uint64_t generation_ = next_generation();
};

}  // namespace data_type
}  // namespace heteromm

#endif  // HETEROMM_B200_DEV_TYPES_BASE_TYPES_H_
