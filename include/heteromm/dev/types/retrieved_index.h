// retrieved_index.h — selection results (B200 build); interface of the
// reference's types/retrieved_index.h: TopKIndex (:43-74, order-sensitive
// is_equal) and ThresholdBitmapIndex (:80-139: 64-bit words, bit i % 64 of
// word i / 64, plus the list of selected indices rebuilt from the bitmap).
#ifndef HETEROMM_B200_DEV_TYPES_RETRIEVED_INDEX_H_
#define HETEROMM_B200_DEV_TYPES_RETRIEVED_INDEX_H_

#include <vector>

#include "base_types.h"

namespace heteromm {
namespace data_type {

template <typename T>
class RetrievedIndex : public BaseType<T> {
public:
    RetrievedIndex() = default;
    virtual ~RetrievedIndex() = default;
    std::string type_name() const override { return "RetrievedIndex"; }
    virtual bool is_equal(const RetrievedIndex<T>& other) = 0;
};

class TopKIndex : public RetrievedIndex<std::vector<int>> {
public:
    using content_type = std::vector<int>;
    TopKIndex() = default;
    TopKIndex(const std::vector<int>& idx) { this->data = idx; }
    std::string type_name() const override { return "TopKIndex"; }
    size_t get_size() const override { return this->data.size() * sizeof(int); }
    bool is_equal(const RetrievedIndex<std::vector<int>>& other) override {
        const auto& o = static_cast<const TopKIndex&>(other).data_ref();
        return o == this->data;
    }
};

class ThresholdBitmapIndex : public RetrievedIndex<std::vector<unsigned long long>> {
public:
    using content_type = std::vector<unsigned long long>;
    ThresholdBitmapIndex() = default;
    ThresholdBitmapIndex(const std::vector<unsigned long long>& bitmap, size_t total_len)
        : total_length_(total_len) {
        this->data = bitmap;
        for (size_t i = 0; i < total_len; ++i)
            if (i / 64 < bitmap.size() && ((bitmap[i / 64] >> (i % 64)) & 1ULL))
                selected_.push_back((int)i);
    }
    std::string type_name() const override { return "ThresholdBitmapIndex"; }
    size_t get_size() const override { return this->data.size() * sizeof(unsigned long long); }
    const std::vector<int>& get_selected_indices() const { return selected_; }
    size_t get_total_length() const { return total_length_; }
    bool is_equal(const RetrievedIndex<std::vector<unsigned long long>>& other) override {
        const auto& o = static_cast<const ThresholdBitmapIndex&>(other).data_ref();
        return o == this->data;
    }

private:
    size_t total_length_ = 0;
    std::vector<int> selected_;
};

}  // namespace data_type
}  // namespace heteromm

#endif  // HETEROMM_B200_DEV_TYPES_RETRIEVED_INDEX_H_
