// target_data.h — inputs / outputs a memory is applied to (B200 build);
// interface of the reference's types/target_data.h: VectorInputOutputData<S>
// (:38-67, exact element-wise is_equal).
#ifndef HETEROMM_B200_DEV_TYPES_TARGET_DATA_H_
#define HETEROMM_B200_DEV_TYPES_TARGET_DATA_H_

#include <vector>

#include "base_types.h"

namespace heteromm {
namespace data_type {

template <typename T>
class TargetData : public BaseType<T> {
public:
    TargetData() = default;
    virtual ~TargetData() = default;
    virtual bool is_equal(const TargetData<T>& other) = 0;
    std::string type_name() const override { return "TargetData"; }
};

template <typename S>
class VectorInputOutputData : public TargetData<std::vector<S>> {
public:
    using content_type = std::vector<S>;
    VectorInputOutputData() = default;
    VectorInputOutputData(const std::vector<S>& v) : vector_size_(v.size()) { this->data = v; }
    std::string type_name() const override { return "VectorInputOutputData"; }
    size_t get_size() const override { return this->data.size() * sizeof(S); }
    bool is_equal(const TargetData<std::vector<S>>& other) override {
        const auto* o = dynamic_cast<const VectorInputOutputData<S>*>(&other);
        if (!o || o->data.size() != this->data.size()) return false;
        for (size_t i = 0; i < this->data.size(); ++i)
            if (this->data[i] != o->data[i]) return false;
        return true;
    }

private:
    size_t vector_size_ = 0;
};

}  // namespace data_type
}  // namespace heteromm

#endif  // HETEROMM_B200_DEV_TYPES_TARGET_DATA_H_
