// score.h — score types (B200 build); interface of the reference's
// types/score.h: VectorScore<S> (:40-74), exact element-wise is_equal.
#ifndef HETEROMM_B200_DEV_TYPES_SCORE_H_
#define HETEROMM_B200_DEV_TYPES_SCORE_H_

#include <vector>

#include "base_types.h"

namespace heteromm {
namespace data_type {

template <typename T>
class Score : public BaseType<T> {
public:
    Score() = default;
    virtual ~Score() = default;
    virtual bool is_equal(const Score<T>& other) = 0;
    std::string type_name() const override { return "Score"; }
};

template <typename S>
class VectorScore : public Score<std::vector<S>> {
public:
    using content_type = std::vector<S>;
    VectorScore() = default;
    VectorScore(const std::vector<S>& s) : num_scores_(s.size()) { this->data = s; }
    std::string type_name() const override { return "VectorScore"; }
    size_t get_size() const override { return this->data.size() * sizeof(S); }
    size_t get_num_scores() const { return this->data.size(); }
    bool is_equal(const Score<std::vector<S>>& other) override {
        const auto* o = dynamic_cast<const VectorScore<S>*>(&other);
        if (!o || o->data.size() != this->data.size()) return false;
        for (size_t i = 0; i < this->data.size(); ++i)
            if (this->data[i] != o->data[i]) return false;
        return true;
    }

private:
    size_t num_scores_ = 0;
};

}  // namespace data_type
}  // namespace heteromm

#endif  // HETEROMM_B200_DEV_TYPES_SCORE_H_
