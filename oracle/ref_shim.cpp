// ref_shim.cpp — C entry points into the reference's own CPU code, compiled by
// oracle/build_ref.sh into oracle/_ref/libheteromm_ref.so.
//
// Test infrastructure only.  Each entry point builds the reference's own
// data_type objects from flat arrays, calls the reference step through its
// public execute() API (KernelType::CPU, the shipped code path) or the
// reference's testbench function, and flattens the result.  Used to generate
// golden vectors (tests/golden/make_golden.py), to pin the oracle
// (tests/test_oracle_pins.py) and as the CPU arm of `bench.py --impl reference`.
#include <cstdint>
#include <cstring>
#include <thread>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "ref_ap_int.h"
#include "ref_consts.h"
#include "steps/apply_memory.h"
#include "steps/build_memory.h"
#include "steps/compute_score.h"
#include "steps/memory_retrieval.h"

using namespace heteromm;

namespace dsa_ref {
void indexer_top_ref(const int L, const std::vector<std::vector<ap_int<16>>>& query_vecs,
                     const std::vector<std::vector<ap_int<16>>>& key_vecs,
                     const std::vector<float>& weights, std::vector<int>& topk_ids);
}
namespace lserve_ref {
void indexer_top_ref(const int L, const int NUM_QUERY,
                     const std::vector<std::vector<ap_int<16>>>& past_keys,
                     const std::vector<std::vector<ap_int<16>>>& queries,
                     const std::vector<std::vector<ap_int<16>>>& new_keys,
                     std::vector<std::vector<int>>& topk_block_indices);
}
namespace seer_budget_ref {
void indexer_top_ref(const int L, const int NUM_QUERY,
                     const std::vector<std::vector<ap_int<16>>>& past_keys,
                     const std::vector<std::vector<ap_int<16>>>& queries,
                     const std::vector<std::vector<ap_int<16>>>& new_keys,
                     std::vector<std::vector<int>>& topk_indices);
}
namespace seer_threshold_ref {
void indexer_top_ref(const int L, const int NUM_QUERY, const int THRESHOLD,
                     const std::vector<std::vector<ap_int<16>>>& past_keys,
                     const std::vector<std::vector<ap_int<16>>>& queries,
                     const std::vector<std::vector<ap_int<16>>>& new_keys,
                     std::vector<std::vector<bool>>& sparse_bitmap);
}
namespace heteromm { namespace step {
void bm25_ref_cpu_kernel(const data_type::BM25IndexMemory& memory,
                         const data_type::BM25Query& query, data_type::TopKIndex& index);
}}

namespace {

std::vector<std::vector<float>> rows_f32(const float* p, int64_t n, int64_t d) {
    std::vector<std::vector<float>> r((size_t)n, std::vector<float>((size_t)d));
    for (int64_t i = 0; i < n; ++i) std::memcpy(r[i].data(), p + i * d, sizeof(float) * d);
    return r;
}

float bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

std::vector<std::vector<ap_int<16>>> rows_i16(const int16_t* p, int64_t n, int64_t d) {
    std::vector<std::vector<ap_int<16>>> r((size_t)n, std::vector<ap_int<16>>((size_t)d));
    for (int64_t i = 0; i < n; ++i)
        for (int64_t j = 0; j < d; ++j) r[i][j] = ap_int<16>(p[i * d + j]);
    return r;
}

// The score -> top-k -> threshold pipeline of one query through the
// reference's public step API (InnerProductCompute, TopKRetrieval,
// ThresholdRetrieval; KernelType::CPU).
void flat_pipeline_one(const data_type::FlatIndexMemory<float>& mem, const float* q, int64_t d,
                       int64_t k, float thr, int32_t* out_idx, uint64_t* out_words,
                       float* out_scores) {
    data_type::VectorQuery<float> query(std::vector<float>(q, q + d));
    data_type::VectorScore<float> score;
    step::InnerProductCompute ip;
    ip.execute(mem, query, score);
    step::TopKRetrieval topk((size_t)k);
    data_type::TopKIndex idx;
    topk.execute(score, idx);
    const auto sel = idx.export_data();
    for (int64_t i = 0; i < k; ++i) out_idx[i] = i < (int64_t)sel.size() ? sel[i] : -1;
    if (out_words) {
        step::ThresholdRetrieval th(thr);
        data_type::ThresholdBitmapIndex bm;
        th.execute(score, bm);
        const auto w = bm.export_data();
        std::memcpy(out_words, w.data(), sizeof(uint64_t) * w.size());
    }
    if (out_scores) {
        const auto s = score.export_data();
        std::memcpy(out_scores, s.data(), sizeof(float) * s.size());
    }
}

}  // namespace

extern "C" {

// ---------------------------------------------------------------- a-1..a-3

void ref_ip_score_f32(const float* mem, int64_t n, int64_t d, const float* q, float* out) {
    data_type::FlatIndexMemory<float> memory(rows_f32(mem, n, d));
    data_type::VectorQuery<float> query(std::vector<float>(q, q + d));
    data_type::VectorScore<float> score;
    step::InnerProductCompute ip;
    ip.execute(memory, query, score);
    const auto s = score.export_data();
    std::memcpy(out, s.data(), sizeof(float) * s.size());
}

int64_t ref_topk_f32(const float* scores, int64_t n, int64_t k, int32_t* out) {
    data_type::VectorScore<float> score(std::vector<float>(scores, scores + n));
    step::TopKRetrieval topk((size_t)k);
    data_type::TopKIndex idx;
    topk.execute(score, idx);
    const auto sel = idx.export_data();
    for (size_t i = 0; i < sel.size(); ++i) out[i] = sel[i];
    return (int64_t)sel.size();
}

int64_t ref_threshold_f32(const float* scores, int64_t n, float thr, uint64_t* out) {
    data_type::VectorScore<float> score(std::vector<float>(scores, scores + n));
    step::ThresholdRetrieval th(thr);
    data_type::ThresholdBitmapIndex bm;
    th.execute(score, bm);
    const auto w = bm.export_data();
    std::memcpy(out, w.data(), sizeof(uint64_t) * w.size());
    return (int64_t)w.size();
}

// A FlatIndexMemory held across calls, so timing excludes its construction.
void* ref_flat_create_f32(const float* mem, int64_t n, int64_t d) {
    return new data_type::FlatIndexMemory<float>(rows_f32(mem, n, d));
}

void* ref_flat_create_bf16(const uint16_t* mem, int64_t n, int64_t d) {
    std::vector<std::vector<float>> r((size_t)n, std::vector<float>((size_t)d));
    for (int64_t i = 0; i < n; ++i)
        for (int64_t j = 0; j < d; ++j) r[i][j] = bf16_to_f32(mem[i * d + j]);
    return new data_type::FlatIndexMemory<float>(r);
}

void ref_flat_destroy(void* h) { delete static_cast<data_type::FlatIndexMemory<float>*>(h); }

// nq queries [nq][d] through the reference pipeline, queries spread over
// n_threads host threads (each query is run by one thread, unchanged).
void ref_flat_pipeline(void* h, const float* queries, int64_t nq, int64_t d, int64_t k,
                       float thr, int with_threshold, int32_t* out_idx, uint64_t* out_words,
                       int64_t words_per_query, int n_threads) {
    const auto& mem = *static_cast<const data_type::FlatIndexMemory<float>*>(h);
    if (n_threads < 1) n_threads = 1;
    std::vector<std::thread> pool;
    for (int t = 0; t < n_threads; ++t) {
        pool.emplace_back([&, t]() {
            for (int64_t q = t; q < nq; q += n_threads)
                flat_pipeline_one(mem, queries + q * d, d, k, thr, out_idx + q * k,
                                  with_threshold ? out_words + q * words_per_query : nullptr,
                                  nullptr);
        });
    }
    for (auto& th : pool) th.join();
}

// -------------------------------------------------------------- a-5, a-6

int64_t ref_paged_kv_summary_f32(const float* keys, int64_t L, int64_t D, const float* w,
                                 int64_t out_dim, int64_t page_size, float* out) {
    data_type::KVCache<float> kv;
    kv.keys = rows_f32(keys, L, D);
    kv.values = kv.keys;
    data_type::KVCacheData<float> raw(kv);
    step::PagedKVIndexBuilder b(rows_f32(w, out_dim, D), (int)page_size);
    data_type::FlatIndexMemory<float> mem;
    b.execute(raw, mem);
    const auto r = mem.export_data();
    for (size_t i = 0; i < r.size(); ++i)
        std::memcpy(out + i * out_dim, r[i].data(), sizeof(float) * r[i].size());
    return (int64_t)r.size();
}

void ref_block_sparse_attention_f32(const float* keys, const float* values, int64_t L, int64_t D,
                                    const int32_t* blocks, int64_t nb, const float* q,
                                    int64_t page_size, float* out) {
    data_type::KVCache<float> kv;
    kv.keys = rows_f32(keys, L, D);
    kv.values = rows_f32(values, L, D);
    data_type::KVCacheData<float> raw(kv);
    data_type::TopKIndex idx(std::vector<int>(blocks, blocks + nb));
    data_type::VectorInputOutputData<float> in(std::vector<float>(q, q + D));
    data_type::VectorInputOutputData<float> o;
    step::BlockSparseAttention att((size_t)page_size);
    att.execute(raw, idx, in, o);
    const auto r = o.export_data();
    std::memcpy(out, r.data(), sizeof(float) * r.size());
}

// Paged-KV decode for one (sequence, head) through the reference steps:
// PagedKVIndexBuilder (identity projection) -> InnerProductCompute ->
// TopKRetrieval -> BlockSparseAttention.  keys/values [L][D] fp32.
void ref_paged_decode_f32(const float* keys, const float* values, int64_t L, int64_t D,
                          const float* q, int64_t block, int64_t topk, int32_t* out_blocks,
                          float* out) {
    data_type::KVCache<float> kv;
    kv.keys = rows_f32(keys, L, D);
    kv.values = rows_f32(values, L, D);
    data_type::KVCacheData<float> raw(kv);
    std::vector<std::vector<float>> eye((size_t)D, std::vector<float>((size_t)D, 0.0f));
    for (int64_t i = 0; i < D; ++i) eye[i][i] = 1.0f;
    step::PagedKVIndexBuilder b(eye, (int)block);
    data_type::FlatIndexMemory<float> summaries;
    b.execute(raw, summaries);
    data_type::FlatIndexMemory<float> mem(summaries.export_data());
    data_type::VectorQuery<float> query(std::vector<float>(q, q + D));
    data_type::VectorScore<float> score;
    step::InnerProductCompute ip;
    ip.execute(mem, query, score);
    step::TopKRetrieval tk((size_t)topk);
    data_type::TopKIndex idx;
    tk.execute(score, idx);
    const auto sel = idx.export_data();
    for (int64_t i = 0; i < topk; ++i) out_blocks[i] = i < (int64_t)sel.size() ? sel[i] : -1;
    data_type::VectorInputOutputData<float> in(std::vector<float>(q, q + D));
    data_type::VectorInputOutputData<float> o;
    step::BlockSparseAttention att((size_t)block);
    att.execute(raw, idx, in, o);
    const auto r = o.export_data();
    std::memcpy(out, r.data(), sizeof(float) * r.size());
}

// -------------------------------------------------------------- indexers

// kernels/dsa_indexer/indexer_tb.cpp:17-57 (16 heads, d=128, top-2048).
void ref_dsa_i16(const int16_t* q, const int16_t* keys, int64_t L, const float* w,
                 int32_t* out) {
    std::vector<int> ids;
    dsa_ref::indexer_top_ref((int)L, rows_i16(q, dsa_ref::NUM_INDEX_HEAD, dsa_ref::HEAD_DIM),
                             rows_i16(keys, L, dsa_ref::HEAD_DIM),
                             std::vector<float>(w, w + dsa_ref::NUM_INDEX_HEAD), ids);
    for (size_t i = 0; i < ids.size(); ++i) out[i] = ids[i];
}
int64_t ref_dsa_topk(void) { return dsa_ref::TOP_K; }
int64_t ref_dsa_heads(void) { return dsa_ref::NUM_INDEX_HEAD; }

static void pad_out(const std::vector<std::vector<int>>& r, int64_t nq, int64_t k, int32_t* out) {
    for (int64_t q = 0; q < nq; ++q)
        for (int64_t i = 0; i < k; ++i)
            out[q * k + i] = i < (int64_t)r[q].size() ? r[q][i] : -1;
}

// kernels/lserve/indexer_lserve_tb.cpp:20-92 (d=128, top-64 blocks of 16).
void ref_lserve_i16(const int16_t* past, int64_t L, const int16_t* queries,
                    const int16_t* new_keys, int64_t nq, int32_t* out) {
    std::vector<std::vector<int>> r;
    lserve_ref::indexer_top_ref((int)L, (int)nq, rows_i16(past, L, lserve_ref::HEAD_DIM),
                                rows_i16(queries, nq, lserve_ref::HEAD_DIM),
                                rows_i16(new_keys, nq, lserve_ref::HEAD_DIM), r);
    pad_out(r, nq, lserve_ref::TOP_K, out);
}

// kernels/seerattention/indexer_seer_token_budget_tb.cpp:19-73 (top-64 tokens).
void ref_seer_budget_i16(const int16_t* past, int64_t L, const int16_t* queries,
                         const int16_t* new_keys, int64_t nq, int32_t* out) {
    std::vector<std::vector<int>> r;
    seer_budget_ref::indexer_top_ref((int)L, (int)nq, rows_i16(past, L, seer_budget_ref::HEAD_DIM),
                                     rows_i16(queries, nq, seer_budget_ref::HEAD_DIM),
                                     rows_i16(new_keys, nq, seer_budget_ref::HEAD_DIM), r);
    pad_out(r, nq, seer_budget_ref::TOP_K, out);
}

// kernels/seerattention/indexer_seer_threshold_tb.cpp:18-77; the bool bitmap
// of each query is packed into words_per_query uint64 words.
void ref_seer_threshold_i16(const int16_t* past, int64_t L, const int16_t* queries,
                            const int16_t* new_keys, int64_t nq, int64_t threshold,
                            int64_t words_per_query, uint64_t* out) {
    std::vector<std::vector<bool>> r;
    seer_threshold_ref::indexer_top_ref(
        (int)L, (int)nq, (int)threshold, rows_i16(past, L, seer_threshold_ref::HEAD_DIM),
        rows_i16(queries, nq, seer_threshold_ref::HEAD_DIM),
        rows_i16(new_keys, nq, seer_threshold_ref::HEAD_DIM), r);
    std::memset(out, 0, sizeof(uint64_t) * nq * words_per_query);
    for (int64_t q = 0; q < nq; ++q)
        for (size_t t = 0; t < r[q].size() && (int64_t)(t / 64) < words_per_query; ++t)
            if (r[q][t]) out[q * words_per_query + t / 64] |= 1ull << (t % 64);
}

// steps/example_kernel/bm25_fpga_retrieval.cpp:138-205 on an index given as a
// CSR inverted index (converted to the reference's per-document maps).
// Returns the number of indices written (the reference fixes k = 64).
void* ref_bm25_create(const int64_t* term_ptr, const int32_t* post_doc, const uint16_t* post_tf,
                      int64_t n_terms, int64_t n_docs) {
    data_type::BM25IndexData data;
    data.doc_freqs.resize((size_t)n_docs);
    for (int64_t t = 0; t < n_terms; ++t) {
        for (int64_t p = term_ptr[t]; p < term_ptr[t + 1]; ++p)
            data.doc_freqs[post_doc[p]][(int)t] = post_tf[p];
        if (term_ptr[t + 1] > term_ptr[t]) data.df_map[(int)t] = (int)(term_ptr[t + 1] - term_ptr[t]);
    }
    return new data_type::BM25IndexMemory(data);
}
void ref_bm25_destroy(void* h) { delete static_cast<data_type::BM25IndexMemory*>(h); }

int64_t ref_bm25_query(void* h, const int32_t* terms, int64_t nterms, int32_t* out) {
    data_type::BM25QueryType m;
    for (int64_t i = 0; i < nterms; ++i)
        if (terms[i] >= 0) m[terms[i]] += 1;
    data_type::BM25Query query(m);
    data_type::TopKIndex idx;
    step::bm25_ref_cpu_kernel(*static_cast<data_type::BM25IndexMemory*>(h), query, idx);
    const auto sel = idx.export_data();
    for (size_t i = 0; i < sel.size(); ++i) out[i] = sel[i];
    return (int64_t)sel.size();
}

}  // extern "C"
