// paged_attention.h — the PagedAttention memory manager (B200 build).
//
// Interface of the reference's deploy/paged_attention.h: a MemoryManager over
// KV cache -> paged key index -> page scores -> top-k pages -> block-sparse
// attention, built from PagedKVIndexBuilder, InnerProductCompute,
// TopKRetrieval and BlockSparseAttention, with a fluent builder and a seeded
// projection-weight generator.  Its size hooks now override the base's (the
// reference's are non-virtual overloads, :127-137, which leave the class
// abstract).  When the schedule puts compute_score, memory_retrieval and
// apply_memory on the GPU and the stock steps are in place, the three run as
// one device-resident pass (device_chain.h).
#ifndef HETEROMM_B200_DEPLOY_PAGED_ATTENTION_H_
#define HETEROMM_B200_DEPLOY_PAGED_ATTENTION_H_

#include <cmath>
#include <iostream>
#include <memory>
#include <string>
#include <typeinfo>
#include <vector>

#include "device_chain.h"
#include "memory_manager.h"

namespace heteromm {
namespace deploy {

using PagedAttentionManager =
    MemoryManager<data_type::KVCacheData<float>,              // RetrievedData: the KV cache
                  data_type::FlatIndexMemory<float>,          // Memory: page summaries
                  data_type::VectorQuery<float>,              // Query: scores the summaries
                  data_type::VectorScore<float>,              // Score: one per page
                  data_type::TopKIndex,                       // Index: the selected pages
                  data_type::VectorInputOutputData<float>,    // Input: the attention query
                  data_type::VectorInputOutputData<float>>;   // Output: the attention output

class PagedAttention : public PagedAttentionManager {
public:
    PagedAttention(const std::string& schedule_path,
                   const std::vector<std::vector<float>>& projection_weight, size_t page_size,
                   size_t top_k)
        : PagedAttentionManager(schedule_path),
          projection_weight_(projection_weight),
          page_size_(page_size),
          top_k_(top_k) {}

    explicit PagedAttention(const std::string& schedule_path = "")
        : PagedAttentionManager(schedule_path) {}

    ~PagedAttention() override = default;

    void set_projection_weight(const std::vector<std::vector<float>>& weight) {
        projection_weight_ = weight;
        build_memory_step_.reset();
    }
    void set_page_size(size_t page_size) {
        page_size_ = page_size;
        build_memory_step_.reset();
        apply_memory_step_.reset();
    }
    void set_top_k(size_t top_k) {
        top_k_ = top_k;
        memory_retrieval_step_.reset();
    }

    size_t page_size() const { return page_size_; }
    size_t top_k() const { return top_k_; }
    const std::vector<std::vector<float>>& projection_weight() const { return projection_weight_; }

    int ret_data_size(const data_type::KVCacheData<float>& retrieved_data) override {
        return static_cast<int>(retrieved_data.get_context_length());
    }
    int memory_size(const data_type::FlatIndexMemory<float>& memory) override {
        return static_cast<int>(memory.get_num_entries());
    }

protected:
    std::shared_ptr<BuildMemoryStepT> create_build_memory_step() override {
        return std::make_shared<step::PagedKVIndexBuilder>(projection_weight_,
                                                           static_cast<int>(page_size_));
    }
    std::shared_ptr<ComputeScoreStepT> create_compute_score_step() override {
        return std::make_shared<step::InnerProductCompute>();
    }
    std::shared_ptr<MemoryRetrievalStepT> create_memory_retrieval_step() override {
        return std::make_shared<step::TopKRetrieval>(top_k_);
    }
    std::shared_ptr<ApplyMemoryStepT> create_apply_memory_step() override {
        return std::make_shared<step::BlockSparseAttention>(page_size_);
    }

    // The stock steps (exactly these classes, so a subclass's own GPU arm is
    // never bypassed) run as one device-resident pass.
    bool run_device_chain(const data_type::KVCacheData<float>& kv,
                          const data_type::FlatIndexMemory<float>& memory,
                          const data_type::VectorQuery<float>& query,
                          const data_type::VectorInputOutputData<float>& input,
                          data_type::VectorInputOutputData<float>& output, ExecutionResult& result,
                          bool verbose) override {
        auto score = get_or_create_compute_score_step();
        auto retrieval = get_or_create_memory_retrieval_step();
        auto apply = get_or_create_apply_memory_step();
        if (!score || !retrieval || !apply) return false;
        if (typeid(*score) != typeid(step::InnerProductCompute) ||
            typeid(*retrieval) != typeid(step::TopKRetrieval) ||
            typeid(*apply) != typeid(step::BlockSparseAttention))
            return false;
        const size_t k = static_cast<const step::TopKRetrieval&>(*retrieval).k();
        const size_t page = static_cast<const step::BlockSparseAttention&>(*apply).page_size();
        if (verbose)
            std::clog << "[PagedAttention] compute_score -> memory_retrieval -> apply_memory as "
                         "one device-resident GPU pass."
                      << std::endl;
        gpu::ChainTimes t;
        output.set_data(gpu::paged_attention_chain(kv, memory, query.data_ref(), k,
                                                   input.data_ref(), page, &t));
        result.compute_score_time_ms = t.score_topk_ms;   // score and top-k are one launch
        result.retrieval_time_ms = 0.0;
        result.apply_memory_time_ms = t.apply_ms;
        return true;
    }

private:
    std::vector<std::vector<float>> projection_weight_;
    size_t page_size_ = 16;
    size_t top_k_ = 8;
};

// Fluent construction (reference paged_attention.h:198-260): the settings
// collect in one struct, each with_* call overwrites one field, and build()
// hands them all to the PagedAttention constructor.
class PagedAttentionBuilder {
public:
    PagedAttentionBuilder() = default;
    PagedAttentionBuilder& with_schedule_path(const std::string& path) {
        return assign(&Settings::schedule_path, path);
    }
    PagedAttentionBuilder& with_projection_weight(const std::vector<std::vector<float>>& weight) {
        return assign(&Settings::projection_weight, weight);
    }
    PagedAttentionBuilder& with_page_size(size_t page_size) {
        return assign(&Settings::page_size, page_size);
    }
    PagedAttentionBuilder& with_top_k(size_t top_k) { return assign(&Settings::top_k, top_k); }
    std::shared_ptr<PagedAttention> build() {
        const Settings& c = settings_;
        return std::make_shared<PagedAttention>(c.schedule_path, c.projection_weight, c.page_size,
                                                c.top_k);
    }

private:
    struct Settings {
        std::string schedule_path;
        std::vector<std::vector<float>> projection_weight;
        size_t page_size = 16;   // the reference's defaults
        size_t top_k = 8;
    };
    template <typename Field, typename Value>
    PagedAttentionBuilder& assign(Field Settings::*field, const Value& value) {
        settings_.*field = value;
        return *this;
    }
    Settings settings_;
};

inline PagedAttentionBuilder create_paged_attention() { return PagedAttentionBuilder(); }

// A [proj_dim][head_dim] weight, uniform in [-0.5, 0.5] x sqrt(2 / (head_dim +
// proj_dim)) (Xavier/Glorot scale).  The values come from the linear
// congruential generator state = state * 1103515245 + 12345 (mod 2^32), taking
// bits 16..30 of each state as (v / 32767) - 0.5, row-major: the generator the
// reference uses (paged_attention.h:270-294), so a seed gives the same weight
// in both.
inline std::vector<std::vector<float>> create_random_projection_weight(size_t head_dim,
                                                                       size_t proj_dim,
                                                                       unsigned int seed = 42) {
    std::vector<std::vector<float>> weight(proj_dim, std::vector<float>(head_dim));
    unsigned int state = seed;
    const float scale = std::sqrt(2.0f / static_cast<float>(head_dim + proj_dim));
    for (auto& row : weight)
        for (auto& w : row) {
            state = state * 1103515245u + 12345u;
            w = (static_cast<float>((state >> 16) & 0x7FFFu) / 32767.0f - 0.5f) * scale;
        }
    return weight;
}

}  // namespace deploy
}  // namespace heteromm

#endif  // HETEROMM_B200_DEPLOY_PAGED_ATTENTION_H_
