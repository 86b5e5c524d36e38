// retrieved_data.h — raw data a memory is built from or applied with (B200
// build); interface of the reference's types/retrieved_data.h: KVCache<S>
// (keys and values, one row per token) and KVCacheData<S> (:38-73).
#ifndef HETEROMM_B200_DEV_TYPES_RETRIEVED_DATA_H_
#define HETEROMM_B200_DEV_TYPES_RETRIEVED_DATA_H_

#include <vector>

#include "base_types.h"

namespace heteromm {
namespace data_type {

template <typename T>
class RetrievedData : public BaseType<T> {
public:
    RetrievedData() = default;
    virtual ~RetrievedData() = default;
    std::string type_name() const override { return "RetrievedData"; }
};

template <typename S>
struct KVCache {
    std::vector<std::vector<S>> keys;
    std::vector<std::vector<S>> values;
};

template <typename S>
class KVCacheData : public RetrievedData<KVCache<S>> {
public:
    using content_type = KVCache<S>;
    KVCacheData() = default;
    KVCacheData(const KVCache<S>& kv)
        : context_length_(kv.keys.size()), head_dim_(kv.keys.empty() ? 0 : kv.keys[0].size()) {
        this->data = kv;
    }
    std::string type_name() const override { return "KVCacheData"; }
    size_t get_size() const override { return 2 * context_length_ * head_dim_ * sizeof(S); }
    size_t get_context_length() const { return context_length_; }
    size_t get_head_dim() const { return head_dim_; }

private:
    size_t context_length_ = 0;
    size_t head_dim_ = 0;
};

}  // namespace data_type
}  // namespace heteromm

#endif  // HETEROMM_B200_DEV_TYPES_RETRIEVED_DATA_H_
