// steps_bm25.cpp — FusedBM25Retrieval: CPU body (the reference's arithmetic,
// steps/example_kernel/bm25_fpga_retrieval.cpp:143-205: fp64 BM25 summed over
// the query's tokens in the query map's iteration order, top-64) and the GPU
// adapter onto the CSR kernels (hmm_bm25_prepare + hmm_bm25_topk_csr), which
// sum the tokens in ascending token-id order.
#include <algorithm>
#include <cmath>
#include <iostream>
#include <numeric>
#include <unordered_map>

#include "device.h"
#include "heteromm/dev/steps/fused_steps/template.h"

namespace heteromm {
namespace step {

namespace {
constexpr size_t kBM25TopK = 64;   // the reference's fixed k (:191)
constexpr double kK1 = 1.2, kB = 0.75;

std::vector<double> doc_lengths(const data_type::BM25IndexData& d, double* avg_dl) {
    std::vector<double> dl(d.doc_freqs.size(), 0.0);
    double sum = 0.0;
    for (size_t i = 0; i < d.doc_freqs.size(); ++i) {
        for (const auto& tf : d.doc_freqs[i]) dl[i] += tf.second;
        sum += dl[i];
    }
    *avg_dl = d.doc_freqs.empty() ? 0.0 : sum / static_cast<double>(d.doc_freqs.size());
    return dl;
}

std::vector<int> best_docs(const std::vector<double>& scores, size_t k) {
    const size_t m = std::min(k, scores.size());
    std::vector<int> idx(scores.size());
    std::iota(idx.begin(), idx.end(), 0);
    std::partial_sort(idx.begin(), idx.begin() + (std::ptrdiff_t)m, idx.end(),
                      [&](int a, int b) { return scores[a] != scores[b] ? scores[a] > scores[b] : a < b; });
    idx.resize(m);
    return idx;
}
}  // namespace

FusedBM25Retrieval::~FusedBM25Retrieval() = default;

void FusedBM25Retrieval::run_test_kernel(const data_type::BM25IndexMemory& memory,
                                         const data_type::BM25Query& query,
                                         data_type::TopKIndex& index) {
    const auto& d = memory.data_ref();
    const size_t n = d.doc_freqs.size();
    if (n == 0) {
        index = data_type::TopKIndex(std::vector<int>{});
        return;
    }
    const double N = static_cast<double>(n);
    double avg_dl = 0.0;
    const std::vector<double> dl = doc_lengths(d, &avg_dl);
    std::vector<double> scores(n, 0.0);
    for (const auto& qt : query.data_ref()) {
        const auto df_it = d.df_map.find(qt.first);
        if (df_it == d.df_map.end()) continue;
        const double df = static_cast<double>(df_it->second);
        const double idf = std::log((N - df + 0.5) / (df + 0.5) + 1.0);
        for (size_t i = 0; i < n; ++i) {
            const auto tf_it = d.doc_freqs[i].find(qt.first);
            if (tf_it == d.doc_freqs[i].end()) continue;
            const double tf = static_cast<double>(tf_it->second);
            scores[i] += idf * (tf * (kK1 + 1.0)) / (tf + kK1 * (1.0 - kB + kB * dl[i] / avg_dl));
        }
    }
    index = data_type::TopKIndex(best_docs(scores, kBM25TopK));
}

void FusedBM25Retrieval::run_cpu_kernel(const data_type::BM25IndexMemory& memory,
                                        const data_type::BM25Query& query,
                                        data_type::TopKIndex& index) {
    run_test_kernel(memory, query, index);
}

void FusedBM25Retrieval::run_gpu_kernel(const data_type::BM25IndexMemory& memory,
                                        const data_type::BM25Query& query,
                                        data_type::TopKIndex& index) {
    const auto& d = memory.data_ref();
    const size_t n_docs = d.doc_freqs.size();
    if (n_docs == 0) {
        index = data_type::TopKIndex(std::vector<int>{});
        return;
    }
    // dense term ids: the tokens of df_map, ascending
    std::vector<int> tokens;
    tokens.reserve(d.df_map.size());
    for (const auto& p : d.df_map) tokens.push_back(p.first);
    std::sort(tokens.begin(), tokens.end());
    std::unordered_map<int, int> term_of;
    for (size_t t = 0; t < tokens.size(); ++t) term_of[tokens[t]] = (int)t;
    const size_t n_terms = tokens.size();

    // CSR postings (docs ascending within each term) and document lengths
    std::vector<int64_t> term_ptr(n_terms + 1, 0);
    std::vector<int32_t> doc_len(n_docs, 0);
    for (size_t i = 0; i < n_docs; ++i)
        for (const auto& tf : d.doc_freqs[i]) {
            doc_len[i] += tf.second;
            const auto it = term_of.find(tf.first);
            if (it != term_of.end()) ++term_ptr[(size_t)it->second + 1];
        }
    for (size_t t = 0; t < n_terms; ++t) term_ptr[t + 1] += term_ptr[t];
    std::vector<int64_t> fill(term_ptr.begin(), term_ptr.end() - 1);
    std::vector<int32_t> post_doc((size_t)term_ptr[n_terms]);
    std::vector<uint16_t> post_tf((size_t)term_ptr[n_terms]);
    for (size_t i = 0; i < n_docs; ++i)
        for (const auto& tf : d.doc_freqs[i]) {
            const auto it = term_of.find(tf.first);
            if (it == term_of.end()) continue;
            if (tf.second < 0 || tf.second > 65535)
                throw std::invalid_argument("FusedBM25Retrieval: term frequency outside uint16");
            const int64_t p = fill[(size_t)it->second]++;
            post_doc[(size_t)p] = (int32_t)i;
            post_tf[(size_t)p] = (uint16_t)tf.second;
        }
    // idf from the memory's own df_map (:176-178) and avg_dl (:158-169), host libm
    const double N = static_cast<double>(n_docs);
    std::vector<double> idf(n_terms);
    for (size_t t = 0; t < n_terms; ++t) {
        const double df = static_cast<double>(d.df_map.at(tokens[t]));
        idf[t] = std::log((N - df + 0.5) / (df + 0.5) + 1.0);
    }
    double avg_dl = 0.0;
    for (size_t i = 0; i < n_docs; ++i) avg_dl += doc_len[i];
    avg_dl /= N;
    // the query's known tokens as dense term ids
    std::vector<int32_t> qterms;
    for (const auto& qt : query.data_ref()) {
        const auto it = term_of.find(qt.first);
        if (it != term_of.end()) qterms.push_back(it->second);
    }
    if (qterms.empty()) qterms.push_back(-1);
    if (qterms.size() > 64)
        throw std::invalid_argument("FusedBM25Retrieval GPU kernel: more than 64 query tokens");

    const int64_t* dtp = gpu::upload(gpu::kMem, term_ptr);
    const int32_t* dpd = gpu::upload(gpu::kAux, post_doc);
    const uint16_t* dpt = gpu::upload(gpu::kAux2, post_tf);
    const int32_t* ddl = gpu::upload(gpu::kAux3, doc_len);
    const double* didf = gpu::upload(gpu::kOut2, idf);
    const int32_t* dq = gpu::upload(gpu::kQuery, qterms);
    const size_t n_skips = hmm_bm25_skips_count((int64_t)n_terms, (int64_t)n_docs);
    const size_t n_post = post_doc.size();
    // one allocation for skips, impacts and the top-k workspace
    const size_t k = std::min(kBM25TopK, n_docs);
    const size_t ws_topk = hmm_bm25_topk_workspace_size((int64_t)n_docs, 1, (int64_t)k);
    const size_t off_imp = ((sizeof(int32_t) * n_skips + 255) & ~size_t(255));
    const size_t off_ws = off_imp + ((sizeof(double) * n_post + 255) & ~size_t(255));
    unsigned char* w =
        static_cast<unsigned char*>(gpu::scratch(gpu::kWork).get(off_ws + ws_topk + 256));
    auto* skips = reinterpret_cast<int32_t*>(w);
    auto* impact = reinterpret_cast<double*>(w + off_imp);
    gpu::check(hmm_bm25_prepare(dtp, dpd, dpt, (int64_t)n_terms, ddl, (int64_t)n_docs, didf,
                                avg_dl, skips, impact, w + off_ws, ws_topk + 256, nullptr),
               "FusedBM25Retrieval GPU index preparation");
    auto* di = static_cast<int32_t*>(gpu::scratch(gpu::kIdx).get(sizeof(int32_t) * k));
    gpu::check(hmm_bm25_topk_csr(dpd, impact, (int64_t)n_post, (int64_t)n_terms, (int64_t)n_docs,
                                 skips, dq, 1, (int64_t)qterms.size(), (int64_t)k, di, nullptr,
                                 w + off_ws, ws_topk, nullptr),
               "FusedBM25Retrieval GPU kernel");
    std::vector<int> out(k);
    gpu::download(out, di);
    index = data_type::TopKIndex(out);
}

void FusedBM25Retrieval::run_fpga_kernel(const data_type::BM25IndexMemory&,
                                         const data_type::BM25Query&, data_type::TopKIndex&) {
    std::clog << "[FusedBM25Retrieval] FPGA kernel not available in this build." << std::endl;
}

}  // namespace step
}  // namespace heteromm
