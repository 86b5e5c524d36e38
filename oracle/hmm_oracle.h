/*
 * hmm_oracle.h — CPU oracle for the HeteroMM score -> select -> apply path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a plain-C restatement of the reference
 * algorithms, used by tests/, by __graft_entry__.smoke() and by the CPU
 * baseline leg of bench.py as the checker.  No product code path may link,
 * load or call it.
 *
 * Every function cites the reference file:line it restates (paths relative to
 * the OswaldHe/HeteroLLM checkout).  Shared conventions:
 *   - fp32 dot products are fl(fl(a*b) + s) in ascending index order, the
 *     arithmetic g++ emits for `dot += m[i][j] * q[j]` on x86-64 without
 *     -march (SSE scalar, no FMA);
 *   - every top-k breaks ties by lowest index (the reference sorts are
 *     unstable; its only tie test, unittest/test_topk_retrieval.cpp:52-64,
 *     expects the lowest indices).  NaN ranks below every number and -0.0
 *     ties with +0.0, exactly as the `>` comparator treats them;
 *   - top-k outputs are ordered best-first; slots beyond min(k, n) hold -1.
 *
 * Pinned by tests/test_oracle_pins.py against (1) the reference's own doctest
 * known-answer cases and (2) golden vectors produced by the reference code
 * compiled from its sources (oracle/build_ref.sh -> oracle/_ref/).
 */
#ifndef HMM_ORACLE_H_
#define HMM_ORACLE_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

void orc_set_threads(int n);

/* Orderable 32-bit key of a float: larger key = better score.  NaN -> 0,
 * -0.0 -> key of +0.0. */
uint32_t orc_f32_key(float f);

/* a-1  steps/example_kernel/inner_product_compute.cpp:11-31
 * out[q*n + i] = sum_{j<d} mem[i*d + j] * qry[q*d + j]   (fp32, j ascending, no FMA) */
void orc_ip_score_f32(const float* mem, int64_t n, int64_t d,
                      const float* qry, int64_t nq, float* out);

/* a-1 on bf16 storage: inputs are widened exactly to fp32 first. */
void orc_ip_score_bf16(const uint16_t* mem, int64_t n, int64_t d,
                       const uint16_t* qry, int64_t nq, float* out);

/* a-2  steps/example_kernel/topk_retrieval.cpp:13-31
 * Top-k of one score vector, best first.  Returns min(k, n). */
int64_t orc_topk_f32(const float* scores, int64_t n, int64_t k, int32_t* out_idx);

/* Same, 64-bit indices with an index offset (for sharded memories). */
int64_t orc_topk_f32_i64(const float* scores, int64_t n, int64_t k,
                         int64_t idx_offset, int64_t* out_idx, float* out_scores);

/* a-3  steps/example_kernel/threshold_retrieval.cpp:11-32
 * bitmap[i/64] bit (i%64) set iff scores[i] >= thr.  ceil(n/64) words. */
void orc_threshold_bitmap_f32(const float* scores, int64_t n, float thr, uint64_t* bitmap);

/* Fused a-1 + a-2 + a-3 for nq queries (config 1).  out_idx [nq][k],
 * out_bitmap [nq][ceil(n/64)] (nullable), out_scores [nq][n] (nullable). */
void orc_ip_topk_f32(const float* mem, int64_t n, int64_t d, const float* qry, int64_t nq,
                     int64_t k, float thr, int32_t* out_idx, uint64_t* out_bitmap,
                     float* out_scores);

/* a-1 + a-2 on bf16 rows (config 5, one shard): top-k with global int64
 * indices (row_offset added), scores returned best first. */
void orc_ip_topk_bf16(const uint16_t* mem, int64_t n, int64_t d, const uint16_t* qry,
                      int64_t nq, int64_t k, int64_t row_offset,
                      int64_t* out_idx, float* out_scores);

/* Multi-GPU merge (config 5): cand_* are [n_shards][nq][k] (idx -1 = empty);
 * outputs [nq][k] by (score desc, global index asc). */
void orc_shard_merge_topk(const float* cand_scores, const int64_t* cand_idx,
                          int64_t n_shards, int64_t nq, int64_t k,
                          float* out_scores, int64_t* out_idx);

/* a-5  steps/example_kernel/paged_kv_index_builder.cpp:18-85
 * keys [L][D], weight [out_dim][D]; out [ceil(L/P)][out_dim].
 * Returns the number of pages written (0 for empty / mismatched input). */
int64_t orc_paged_kv_summary_f32(const float* keys, int64_t L, int64_t D,
                                 const float* weight, int64_t out_dim, int64_t page_size,
                                 float* out);

/* Mean-pool only (weight = identity, which the projection reproduces
 * exactly: 1*x + 0*y summed in order is x). */
int64_t orc_block_mean_f32(const float* keys, int64_t L, int64_t D, int64_t page_size,
                           float* out);
int64_t orc_block_minmax_f32(const float* keys, int64_t L, int64_t D, int64_t page_size,
                             float* out);
void orc_block_select_minmax(const float* q, const float* minmax, int64_t nb, int64_t D,
                             int64_t top, int32_t* out);

/* a-6  steps/example_kernel/block_sparse_attention.cpp:21-126
 * keys/values [L][D], blocks [nb] (block ids, top-k order), q [D]; out [D]. */
void orc_block_sparse_attention_f32(const float* keys, const float* values, int64_t L,
                                    int64_t D, const int32_t* blocks, int64_t nb,
                                    const float* q, int64_t page_size, float* out);

/* a-7  paged layout: logical page p of sequence s lives in physical page
 * page_table[s*pages_per_seq + p].  Expands the selected blocks of a-6
 * into physical page ids, in top-k order (block b covers logical pages
 * [b*ppb, (b+1)*ppb) clipped to the sequence).  Returns pages written. */
int64_t orc_block_pages(const int32_t* page_table, int64_t pages_per_seq, int64_t seq,
                        const int32_t* blocks, int64_t nb, int64_t pages_per_block,
                        int32_t* out_pages);

/* a-8  kernels/dsa_indexer/indexer_tb.cpp:17-57 (int16 values, one query)
 * q [H][D], keys [L][D], w [H].  Returns min(topk, L) indices. */
int64_t orc_dsa_indexer_i16(const int16_t* q, int64_t H, int64_t D, const int16_t* keys,
                            int64_t L, const float* w, int64_t topk, int32_t* out_idx,
                            float* out_scores);

/* a-8  FP8 e4m3 multi-head form (kernels/deepseek_engram/deepseek_v32_dsa_bench.py:77-101
 * scored with the arithmetic of indexer_tb.cpp:27-46).  q [T][H][D], keys [L][D],
 * w [T][H].  Query t sees keys j <= pos0 + t.  out_idx [T][topk]. */
void orc_dsa_indexer_fp8(const uint8_t* q, int64_t T, int64_t H, int64_t D,
                         const uint8_t* keys, int64_t L, const float* w, int64_t pos0,
                         int64_t topk, int32_t* out_idx, float* out_scores);
/* Exact e4m3 value times 2^9 as an integer (NaN encodings return 0). */
int32_t orc_e4m3_scaled(uint8_t v);
/* Exact score of one (query, key) pair, the building block of the above. */
float orc_dsa_score_fp8(const uint8_t* q_t, int64_t H, int64_t D, const uint8_t* key,
                        const float* w_t);

/* Every exact score of the FP8 indexer: out [T][L], -inf where key j is not
 * visible to token t (j > pos0 + t). */
void orc_dsa_scores_fp8(const uint8_t* q, int64_t T, int64_t H, int64_t D, const uint8_t* keys,
                        int64_t L, const float* w, int64_t pos0, float* out);

/* a-9  kernels/lserve/indexer_lserve_tb.cpp:20-90.  Returns per query the
 * top-k 16-token blocks.  out [nq][topk] (-1 padded). */
void orc_lserve_topk_i16(const int16_t* past, int64_t L, const int16_t* queries,
                         const int16_t* new_keys, int64_t nq, int64_t D, int64_t topk,
                         int64_t block, int32_t* out);

/* a-10  kernels/seerattention/indexer_seer_token_budget_tb.cpp:19-74 */
void orc_seer_budget_i16(const int16_t* past, int64_t L, const int16_t* queries,
                         const int16_t* new_keys, int64_t nq, int64_t D, int64_t topk,
                         int32_t* out);

/* a-10  kernels/seerattention/indexer_seer_threshold_tb.cpp:18-80.
 * out [nq][words_per_query] of uint64 (bit t of the query's bit string). */
int64_t orc_seer_words_per_query(int64_t L, int64_t nq);
void orc_seer_threshold_i16(const int16_t* past, int64_t L, const int16_t* queries,
                            const int16_t* new_keys, int64_t nq, int64_t D,
                            int64_t threshold, uint64_t* out);

/* a-11  steps/example_kernel/bm25_fpga_retrieval.cpp:138-205 over a CSR
 * inverted index: postings of term t are [term_ptr[t], term_ptr[t+1]) with
 * ascending doc ids and term frequencies.  doc_len [n_docs] (sum of tf).
 * qterms [nq][qlen] (-1 = unused slot).  Query terms are summed in
 * ascending term-id order.  out [nq][k]. */
void orc_bm25_idf(const int64_t* term_ptr, int64_t n_terms, int64_t n_docs, double* idf);
double orc_bm25_avgdl(const int32_t* doc_len, int64_t n_docs);
void orc_bm25_topk(const int64_t* term_ptr, const int32_t* post_doc, const uint16_t* post_tf,
                   int64_t n_terms, const int32_t* doc_len, int64_t n_docs,
                   const int32_t* qterms, int64_t nq, int64_t qlen, int64_t k,
                   int32_t* out_idx, double* out_scores);

#ifdef __cplusplus
}
#endif

#endif  /* HMM_ORACLE_H_ */
