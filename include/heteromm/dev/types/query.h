// query.h — query types (B200 build); interface of the reference's
// types/query.h: VectorQuery<S> (:46-65) and BM25Query (:101-119).
#ifndef HETEROMM_B200_DEV_TYPES_QUERY_H_
#define HETEROMM_B200_DEV_TYPES_QUERY_H_

#include <unordered_map>
#include <vector>

#include "base_types.h"

namespace heteromm {
namespace data_type {

using BM25QueryType = std::unordered_map<int, int>;   // token id -> frequency

template <typename T>
class Query : public BaseType<T> {
public:
    Query() = default;
    virtual ~Query() = default;
    std::string type_name() const override { return "Query"; }
};

template <typename S>
class VectorQuery : public Query<std::vector<S>> {
public:
    using content_type = std::vector<S>;
    VectorQuery() = default;
    VectorQuery(const std::vector<S>& v) : vector_size_(v.size()) { this->data = v; }
    std::string type_name() const override { return "VectorQuery"; }
    size_t get_size() const override { return vector_size_ * sizeof(S); }
    size_t get_vector_size() const { return vector_size_; }

private:
    size_t vector_size_ = 0;
};

class BM25Query : public Query<BM25QueryType> {
public:
    using content_type = BM25QueryType;
    BM25Query() = default;
    BM25Query(const BM25QueryType& token_freq) {
        this->data = token_freq;
        for (const auto& p : token_freq) num_tokens_ += (size_t)p.second;
    }
    std::string type_name() const override { return "BM25Query"; }
    size_t get_size() const override { return this->data.size() * 2 * sizeof(int); }
    size_t get_num_tokens() const { return num_tokens_; }

private:
    size_t num_tokens_ = 0;
};

}  // namespace data_type
}  // namespace heteromm

#endif  // HETEROMM_B200_DEV_TYPES_QUERY_H_
