// base_types.h — data-type base of the heteromm step API (B200 build).
//
// Same interface as the reference's toolchain/frontend/dev/types/base_types.h:
// every datum carries its device location and exposes its contents by copy
// (export_data) and replacement (set_data).  data_ref() is an addition of this
// build: a const reference to the contents for the GPU adapters, which read
// large memories without the deep copy export_data makes.
#ifndef HETEROMM_B200_DEV_TYPES_BASE_TYPES_H_
#define HETEROMM_B200_DEV_TYPES_BASE_TYPES_H_

#include <cstddef>
#include <cstdint>
#include <string>
#include <type_traits>
#include <vector>

namespace heteromm {
namespace data_type {

enum class DataLocation { SYS_DRAM, GPU_MEM, FPGA_MEM };

template <typename T>
class BaseType {
public:
    virtual ~BaseType() = default;
    virtual std::string type_name() const = 0;
    virtual size_t get_size() const = 0;

    DataLocation get_device() const { return device_; }
    void set_device(DataLocation device) { device_ = device; }

    T export_data() const { return data; }
    void set_data(const T& new_data) { data = new_data; }
    const T& data_ref() const { return data; }

protected:
    DataLocation device_ = DataLocation::SYS_DRAM;
    T data;
};

}  // namespace data_type
}  // namespace heteromm

#endif  // HETEROMM_B200_DEV_TYPES_BASE_TYPES_H_
