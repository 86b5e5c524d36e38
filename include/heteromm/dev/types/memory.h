// memory.h — memory types on the score -> select path (B200 build).
//
// Interface of the reference's types/memory.h for the types this path uses:
// FlatIndexMemory<S> (types/memory.h:46-126) and BM25IndexMemory
// (:232-301).  BM25IndexMemory declares the `content_type` alias the step
// templates require (the reference omits it at :240).
#ifndef HETEROMM_B200_DEV_TYPES_MEMORY_H_
#define HETEROMM_B200_DEV_TYPES_MEMORY_H_

#include <deque>
#include <stdexcept>
#include <unordered_map>
#include <vector>

#include "base_types.h"

namespace heteromm {
namespace data_type {

template <typename T>
class Memory : public BaseType<T> {
public:
    virtual ~Memory() = default;
    virtual bool is_equal(const Memory<T>& other) = 0;
    std::string type_name() const override { return "Memory"; }
};

// num_entries rows of memory_size values each.
template <typename S>
class FlatIndexMemory : public Memory<std::vector<std::vector<S>>> {
public:
    using content_type = std::vector<std::vector<S>>;

    FlatIndexMemory() = default;
    FlatIndexMemory(const content_type& rows)
        : num_entries_(rows.size()), memory_size_(rows.empty() ? 0 : rows[0].size()) {
        this->data = rows;
    }

    std::string type_name() const override { return "FlatIndexMemory"; }
    size_t get_size() const override { return num_entries_ * memory_size_ * sizeof(S); }

    // Replaces the rows and keeps num_entries / memory_size in step with them
    // (the reference's set_data is the base's, which leaves the counts of the
    // previous contents, types/base_types.h:68-70 and memory.h:78).
    void set_data(const content_type& rows) {
        Memory<content_type>::set_data(rows);
        num_entries_ = rows.size();
        memory_size_ = rows.empty() ? 0 : rows[0].size();
        deltas_.clear();
    }

    // Row changes made by insert_memory / pop_last_memory / delete_memory,
    // oldest first, at most kMaxRowDeltas (an addition of this build).  Each
    // names the generation it was made on and the one it produced, so a copy of
    // the rows taken at generation `from` (a device copy, say) can be brought up
    // to date by replaying the changes after it instead of being taken again.
    // set_data clears the log; a copy of the memory has a generation of its own,
    // so the log it inherits never ends at it and is never replayed for it.
    struct RowDelta {
        enum Kind { Append, PopLast, Erase };
        uint64_t from, to;
        Kind kind;
        size_t index;          // Append: the new row's position; Erase: the erased row's
        std::vector<S> row;    // Append: the appended row
    };
    static constexpr size_t kMaxRowDeltas = 1024;
    const std::deque<RowDelta>& row_deltas() const { return deltas_; }
    size_t get_num_entries() const { return num_entries_; }
    size_t get_memory_size() const { return memory_size_; }

    // Element-wise equality of the stored rows (`==` per value, as `!=` is
    // the reference's mismatch test, so NaN never matches).
    bool is_equal(const Memory<content_type>& other) override {
        const auto* o = dynamic_cast<const FlatIndexMemory<S>*>(&other);
        return o && o->data == this->data;
    }

    void insert_memory(const std::vector<S>& row) {
        if (num_entries_ == 0 && memory_size_ == 0) memory_size_ = row.size();
        if (row.size() != memory_size_)
            throw std::invalid_argument("FlatIndexMemory: row size does not match memory_size");
        this->data.push_back(row);
        record(RowDelta::Append, num_entries_, &row);
        ++num_entries_;
    }
    void pop_last_memory() {
        if (num_entries_ == 0) throw std::out_of_range("FlatIndexMemory: memory is empty");
        this->data.pop_back();
        record(RowDelta::PopLast, num_entries_ - 1, nullptr);
        --num_entries_;
    }
    void delete_memory(size_t idx) {
        if (idx >= num_entries_) throw std::out_of_range("FlatIndexMemory: index out of range");
        this->data.erase(this->data.begin() + (std::ptrdiff_t)idx);
        record(RowDelta::Erase, idx, nullptr);
        --num_entries_;
    }
    std::vector<S> get_memory(size_t idx) const {
        if (idx >= num_entries_) throw std::out_of_range("FlatIndexMemory: index out of range");
        return this->data[idx];
    }

private:
    // Renews the generation and logs the change that produced it.
    void record(typename RowDelta::Kind kind, size_t index, const std::vector<S>* row) {
        const uint64_t from = this->generation();
        this->touch();
        deltas_.push_back(RowDelta{from, this->generation(), kind, index,
                                   row ? *row : std::vector<S>()});
        if (deltas_.size() > kMaxRowDeltas) deltas_.pop_front();
    }

    size_t num_entries_ = 0;
    size_t memory_size_ = 0;
    std::deque<RowDelta> deltas_;
};

// Inverted BM25 statistics: document frequency per token and the token
// frequencies of every document.
struct BM25IndexData {
    std::unordered_map<int, int> df_map;
    std::vector<std::unordered_map<int, int>> doc_freqs;
};

class BM25IndexMemory : public Memory<BM25IndexData> {
public:
    using content_type = BM25IndexData;

    BM25IndexMemory() = default;
    BM25IndexMemory(const BM25IndexData& d) : num_documents_(d.doc_freqs.size()) {
        this->data = d;
        for (const auto& doc : d.doc_freqs)
            for (const auto& tf : doc) num_tokens_ += (size_t)tf.second;
    }

    std::string type_name() const override { return "BM25IndexMemory"; }
    size_t get_size() const override {
        size_t n = this->data.df_map.size();
        for (const auto& doc : this->data.doc_freqs) n += doc.size();
        return n * 2 * sizeof(int);
    }
    size_t get_num_documents() const { return num_documents_; }
    size_t get_num_tokens() const { return num_tokens_; }

    bool is_equal(const Memory<BM25IndexData>& other) override {
        const auto* o = dynamic_cast<const BM25IndexMemory*>(&other);
        return o && o->data.doc_freqs == this->data.doc_freqs && o->data.df_map == this->data.df_map;
    }

    void insert_document(const std::unordered_map<int, int>& doc) {
        this->data.doc_freqs.push_back(doc);
        this->touch();
        for (const auto& tf : doc) {
            ++this->data.df_map[tf.first];
            num_tokens_ += (size_t)tf.second;
        }
        ++num_documents_;
    }

private:
    size_t num_documents_ = 0;
    size_t num_tokens_ = 0;
};

}  // namespace data_type
}  // namespace heteromm

#endif  // HETEROMM_B200_DEV_TYPES_MEMORY_H_
