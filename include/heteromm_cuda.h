/*
 * heteromm_cuda.h — C ABI of the B200 (sm_100a) kernels behind the HeteroMM
 * score -> select -> apply steps.
 *
 * This is the drop-in boundary: the `KernelType::GPU` arm of every step
 * (steps/compute_score.h:104-112, steps/memory_retrieval.h:96-104,
 * steps/build_memory.h:94-102, steps/apply_memory.h:103-111,
 * steps/fused_steps/template.h:75-83 in the reference) calls these entry
 * points, and so can any FFI (ctypes, cgo, JNI) directly.
 *
 * Conventions
 *   - Plain C: pointers, sizes, status codes.  No exceptions cross the ABI.
 *   - Every data pointer is a DEVICE pointer on the current CUDA device;
 *     `stream` is a cudaStream_t passed as void* (NULL = legacy stream).
 *   - Outputs are caller-owned.  Entry points that need scratch memory take a
 *     caller-provided `workspace` of at least `*_workspace_size(...)` bytes
 *     (sized for the current device); they never allocate.
 *   - Calls are asynchronous on `stream`; argument errors are reported
 *     synchronously, device-side errors through the CUDA error state.
 *   - Top-k outputs are ordered best first; ties are broken by the lowest
 *     row index; NaN ranks below every number and -0.0 ties with +0.0.
 *     Slots beyond min(k, n) hold index -1 and score -inf.
 *   - fp32 dot products are computed exactly as the reference CPU code does:
 *     fl(fl(a*b) + s) with j ascending (no FMA contraction), so fp32 scores
 *     are bit-identical to the reference's.
 *   - hmm_last_error() returns the message of the calling thread's last
 *     failed call.
 */
#ifndef HETEROMM_CUDA_H_
#define HETEROMM_CUDA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    HMM_OK = 0,
    HMM_ERR_INVALID = 1,      /* bad argument (null pointer, negative size, k out of range) */
    HMM_ERR_CUDA = 2,         /* a CUDA runtime call or kernel launch failed */
    HMM_ERR_OOM = 3,          /* workspace too small */
    HMM_ERR_BOUNDS = 4,       /* an index / page-table entry outside its extent */
    HMM_ERR_TIMEOUT = 5,      /* a bounded wait (device or collective) gave up */
    HMM_ERR_UNSUPPORTED = 6   /* shape outside what the kernels implement */
} hmm_status_t;

/* Message of the calling thread's last failed call ("" if none). */
const char* hmm_last_error(void);
/* Library version string, e.g. "heteromm-b200 0.1.0 sm_100a". */
const char* hmm_version(void);

/* ---------------------------------------------------------------- score
 * InnerProductCompute (reference steps/compute_score.h:172-205,
 * steps/example_kernel/inner_product_compute.cpp:11-31).
 * scores[q*n_rows + i] = sum_j mem[i*dim + j] * queries[q*dim + j]
 * mem [n_rows][dim] fp32 row-major, queries [n_queries][dim], dim <= 1024. */
hmm_status_t hmm_ip_score_f32(const float* mem, int64_t n_rows, int64_t dim,
                              const float* queries, int64_t n_queries, float* scores,
                              void* stream);

/* --------------------------------------------------------------- select
 * TopKRetrieval (reference steps/memory_retrieval.h:159-193,
 * steps/example_kernel/topk_retrieval.cpp:13-31) on device-resident scores
 * [n_queries][n].  out_idx [n_queries][k] int32; out_scores [n_queries][k]
 * or NULL.  1 <= k <= 4096. */
size_t hmm_topk_f32_workspace_size(int64_t n, int64_t n_queries, int64_t k);
hmm_status_t hmm_topk_f32(const float* scores, int64_t n, int64_t n_queries, int64_t k,
                          int32_t* out_idx, float* out_scores, void* workspace,
                          size_t workspace_bytes, void* stream);

/* ThresholdRetrieval (reference steps/memory_retrieval.h:200-234,
 * steps/example_kernel/threshold_retrieval.cpp:11-32): bit i%64 of word
 * i/64 is set iff scores[i] >= threshold.  bitmap [n_queries][ceil(n/64)]. */
hmm_status_t hmm_threshold_bitmap_f32(const float* scores, int64_t n, int64_t n_queries,
                                      float threshold, uint64_t* bitmap, void* stream);

/* ---------------------------------------------------- fused score + select
 * FusedComputeScoreAndRetrieval<FlatIndexMemory<float>, VectorQuery<float>,
 * TopKIndex> (reference steps/fused_steps/template.h:21-135), batched over
 * queries: InnerProductCompute -> TopKRetrieval (+ ThresholdRetrieval) in one
 * pass; scores never round-trip through HBM.
 *   out_idx     [n_queries][k] int32 (required)
 *   out_scores  [n_queries][k] fp32 scores of the selected rows, or NULL
 *   out_bitmap  [n_queries][ceil(n_rows/64)] threshold bitmap (>=), or NULL
 * dim <= 1024, 1 <= k <= 256, n_rows < 2^31. */
size_t hmm_ip_topk_f32_workspace_size(int64_t n_rows, int64_t dim, int64_t n_queries,
                                      int64_t k);
hmm_status_t hmm_ip_topk_f32(const float* mem, int64_t n_rows, int64_t dim,
                             const float* queries, int64_t n_queries, int64_t k,
                             int32_t* out_idx, float* out_scores, float threshold,
                             uint64_t* out_bitmap, void* workspace, size_t workspace_bytes,
                             void* stream);

/* Same on bf16 rows and queries (bf16 bit patterns as uint16), fp32
 * accumulate: one shard of a row-sharded memory.  Row i of this shard has
 * global index row_offset + i; out_idx [n_queries][k] int64 global indices,
 * out_scores [n_queries][k] fp32 (required: the shard merge needs them).
 * Scores equal the reference's fp32 inner product of the widened values
 * (j ascending, each product rounded before it is added, as its g++ build
 * without FMA contraction does).
 * For dim == 128, k <= 128, n_rows > 8192 and 16-byte aligned pointers the
 * rows are scored on the tensor cores (tcgen05) and the candidates rescored
 * exactly; that path waits for `stream` before returning (it reads back the
 * kernel's status word) and returns HMM_ERR_TIMEOUT if a bounded device wait
 * gave up.  Other shapes run the exact CUDA-core kernel asynchronously. */
size_t hmm_ip_topk_bf16_workspace_size(int64_t n_rows, int64_t dim, int64_t n_queries,
                                       int64_t k);
hmm_status_t hmm_ip_topk_bf16(const uint16_t* mem, int64_t n_rows, int64_t dim,
                              const uint16_t* queries, int64_t n_queries, int64_t k,
                              int64_t row_offset, int64_t* out_idx, float* out_scores,
                              void* workspace, size_t workspace_bytes, void* stream);

/* The same shard step without waiting for `stream` (no host synchronisation,
 * so a caller can queue the all-gather and merge behind it).  On the
 * tensor-core path a bounded wait that gave up sets HMM_STATUS_TIMEOUT, and
 * a candidate pool that filled up (possible only for rows ordered so that
 * the running k-th best keeps rising) sets HMM_STATUS_POOL_OVERFLOW, in
 * *device_status (an int32 in device memory that the caller zeroes); the
 * outputs are then invalid and hmm_status_read reports HMM_ERR_TIMEOUT or
 * HMM_ERR_UNSUPPORTED.  Recompute an overflowed call with hmm_ip_topk_bf16,
 * which falls back to the exact CUDA-core kernel by itself. */
hmm_status_t hmm_ip_topk_bf16_async(const uint16_t* mem, int64_t n_rows, int64_t dim,
                                    const uint16_t* queries, int64_t n_queries, int64_t k,
                                    int64_t row_offset, int64_t* out_idx, float* out_scores,
                                    int32_t* device_status, void* workspace,
                                    size_t workspace_bytes, void* stream);

/* Final merge of per-shard candidates after the all-gather: cand_* are
 * [n_shards][n_queries][k] (index -1 = empty slot); outputs [n_queries][k]
 * by (score desc, global index asc).  No reference counterpart: the
 * reference has no multi-device path; the merge preserves its top-k order. */
size_t hmm_shard_merge_topk_workspace_size(int64_t n_shards, int64_t n_queries, int64_t k);
hmm_status_t hmm_shard_merge_topk(const float* cand_scores, const int64_t* cand_idx,
                                  int64_t n_shards, int64_t n_queries, int64_t k,
                                  float* out_scores, int64_t* out_idx, void* workspace,
                                  size_t workspace_bytes, void* stream);

/* ------------------------------------------------ allocation-free variant
 * No counterpart in the reference: this entry point exists for callers that
 * cannot allocate device memory and so cannot supply the workspace that
 * hmm_ip_topk_f32 needs - for example a host reached through an FFI (cgo,
 * JNI) that only holds device pointers handed to it by another runtime, or a
 * serving process whose memory pool owns the whole device and forbids
 * cudaMalloc once it is running.
 *
 * Same inputs, outputs and results as hmm_ip_topk_f32.  Its scratch lives in
 * a fixed array of HMM_NOALLOC_SCRATCH_BYTES in device memory inside this
 * library (every GPU that loads the library holds it until the process
 * exits); it calls no cudaMalloc, cudaFree or other allocating routine.
 *   - Problems whose scratch need (the value hmm_ip_topk_f32_workspace_size
 *     returns) exceeds HMM_NOALLOC_SCRATCH_BYTES are rejected with
 *     HMM_ERR_UNSUPPORTED; config-1 sized calls (65,536 x 128 rows, 64
 *     queries, k = 64) need about 2 MiB.
 *   - The first call on each device looks up the array's device address
 *     (cudaGetSymbolAddress) with that device current; make that first call
 *     before any stream capture.  The address is cached per device together
 *     with the CUDA context it belongs to; after a device reset (or any other
 *     re-creation of the context) the next call looks it up again, and that
 *     call, too, belongs before any stream capture.
 *   - Every call on a device shares the one array, which keeps the previous
 *     call's contents (nothing in it needs to start at zero: each call writes
 *     every slot it later reads).  Calls that overlap on the same GPU - on
 *     different streams, or from different host threads - race on the array
 *     and must be serialised by the caller. */
#define HMM_NOALLOC_SCRATCH_BYTES (4u << 20)
hmm_status_t hmm_ip_topk_f32_noalloc(const float* mem, int64_t n_rows, int64_t dim,
                                     const float* queries, int64_t n_queries, int64_t k,
                                     int32_t* out_idx, float* out_scores, float threshold,
                                     uint64_t* out_bitmap, void* stream);

/* ------------------------------------------------------------ paged KV
 * Paged KV cache: physical page `phys` holds `page_tokens` consecutive tokens
 * of one sequence as [page_tokens][D] bf16 (K and V in separate page arrays
 * of n_pages pages); page_table[s*pages_per_seq + p] is the physical page of
 * logical page p of sequence s.  D % 4 == 0, 4 <= D <= 512,
 * seq_len <= pages_per_seq * page_tokens, every sequence has seq_len tokens.
 * A page-table entry outside [0, n_pages) read by a kernel (or a negative
 * block id) makes the call return HMM_ERR_BOUNDS; the kernels never follow
 * such an entry.  Calls that report device-side bounds wait for `stream`.
 *
 * PagedKVIndexBuilder (reference steps/build_memory.h:152-182,
 * steps/example_kernel/paged_kv_index_builder.cpp:18-85) on contiguous fp32
 * keys [n_seq][L][D]: page p pools tokens [p*page_size, min(+page_size, L))
 * (fp32 sum in token order, then / count) and, with a non-NULL weight
 * [out_dim][D], projects it (fp32, d ascending, no FMA).
 * out [n_seq][ceil(L/page_size)][weight ? out_dim : D], bit-identical to the
 * reference.  L == 0 writes nothing (the reference's empty memory). */
hmm_status_t hmm_paged_kv_summary_f32(const float* keys, int64_t n_seq, int64_t L, int64_t D,
                                      const float* weight, int64_t out_dim, int64_t page_size,
                                      float* out, void* stream);

/* Workspace for the three paged calls below (n_sel = selected blocks per
 * sequence, or top_blocks; the summary needs 256 bytes). */
size_t hmm_paged_workspace_size(int64_t n_seq, int64_t n_sel, int64_t block_tokens, int64_t D);

/* Block summaries of a paged bf16 key cache: summary b of sequence s is the
 * fp32 mean of tokens [b*block_tokens, min(+block_tokens, seq_len)), summed
 * in token order as paged_kv_index_builder.cpp:57-67 does (the projection is
 * left out).  out [n_seq][ceil(seq_len/block_tokens)][D] fp32, 16-byte
 * aligned.  Bit-identical to the reference arithmetic. */
hmm_status_t hmm_paged_kv_summary_bf16(const uint16_t* k_pages, int64_t n_pages,
                                       const int32_t* page_table, int64_t n_seq,
                                       int64_t pages_per_seq, int64_t seq_len,
                                       int64_t page_tokens, int64_t block_tokens, int64_t D,
                                       float* out, void* workspace, size_t workspace_bytes,
                                       void* stream);

/* Min/max page summaries of the paged key cache, the reference's
 * MinMaxIndexMemory (types/memory.h:127-230; no reference step computes them):
 * out [n_seq][ceil(seq_len/block_tokens)][2][D] fp32, per block and column the
 * smallest then the largest key (fminf / fmaxf).  Arguments and checks as
 * hmm_paged_kv_summary_bf16. */
hmm_status_t hmm_paged_kv_minmax_bf16(const uint16_t* k_pages, int64_t n_pages,
                                      const int32_t* page_table, int64_t n_seq,
                                      int64_t pages_per_seq, int64_t seq_len,
                                      int64_t page_tokens, int64_t block_tokens, int64_t D,
                                      float* out, void* workspace, size_t workspace_bytes,
                                      void* stream);

/* The min/max-bound block selector over those summaries: per sequence, the
 * top_blocks blocks with the largest u_b = sum_j max(q_j * min_bj, q_j * max_bj)
 * (j ascending, each product rounded before the add), an upper bound of q.k for
 * every key of block b; best first, ties to the lower block, -1 past n_blocks.
 * q [n_seq][D] bf16; the selection feeds hmm_block_sparse_attention_bf16. */
hmm_status_t hmm_block_select_minmax(const uint16_t* q, const float* minmax, int64_t n_seq,
                                     int64_t n_blocks, int64_t D, int64_t top_blocks,
                                     int32_t* out_blocks, void* stream);

/* Physical pages of the selected blocks (the reference has no page table; this
 * is the paged form of the token list of block_sparse_attention.cpp:53-63):
 * for each sequence, logical pages [b*pages_per_block, (b+1)*pages_per_block)
 * of each selected block b in selection order, clipped to [0, pages_per_seq),
 * mapped through the page table.  out_pages [n_seq][n_sel*pages_per_block]
 * (-1 after the last), out_counts [n_seq] (nullable).  Integer, bit-exact. */
hmm_status_t hmm_block_pages(const int32_t* page_table, int64_t n_seq, int64_t pages_per_seq,
                             const int32_t* blocks, int64_t n_sel, int64_t pages_per_block,
                             int32_t* out_pages, int32_t* out_counts, void* stream);

/* BlockSparseAttention (reference steps/apply_memory.h:169-213,
 * steps/example_kernel/block_sparse_attention.cpp:21-126), one query per
 * sequence (decode), over the paged bf16 cache: tokens = concatenation of
 * [b*block_tokens, min(+block_tokens, seq_len)) over the selected blocks in
 * order; s_i = (q.k_i) * (1/sqrtf(D)); softmax with the maximum subtracted;
 * out = sum_i w_i v_i.  An empty token list gives zeros.  fp32 results agree
 * with the reference's to ~1e-6 relative (the device expf and the summation
 * order differ from glibc's and from sequential order); the token / page
 * lists are exact.  blocks [n_seq][n_sel] (n_sel <= 4096), q [n_seq][D] bf16,
 * out [n_seq][D] fp32. */
hmm_status_t hmm_block_sparse_attention_bf16(const uint16_t* q, const uint16_t* k_pages,
                                             const uint16_t* v_pages, int64_t n_pages,
                                             const int32_t* page_table, int64_t n_seq,
                                             int64_t pages_per_seq, int64_t seq_len,
                                             int64_t page_tokens, int64_t block_tokens,
                                             int64_t D, const int32_t* blocks, int64_t n_sel,
                                             float* out, void* workspace,
                                             size_t workspace_bytes, void* stream);

/* The same attention on contiguous fp32 K/V (the reference's own
 * KVCacheData<float> layout): keys, values [n_seq][L][D] fp32, q [n_seq][D]
 * fp32, all 16-byte aligned.  Same token rule, same tolerance. */
hmm_status_t hmm_block_sparse_attention_f32(const float* q, const float* keys,
                                            const float* values, int64_t n_seq, int64_t L,
                                            int64_t D, int64_t block_tokens,
                                            const int32_t* blocks, int64_t n_sel, float* out,
                                            void* workspace, size_t workspace_bytes,
                                            void* stream);

/* One decode step of the paged-KV path: per sequence, score the block
 * summaries [n_seq][ceil(seq_len/block_tokens)][D] fp32 (16-byte aligned)
 * against q widened from bf16 (InnerProductCompute arithmetic: fp32, d
 * ascending, no FMA), keep the top_blocks best (TopKRetrieval: best first,
 * ties to the lowest block id; bit-exact), then block-sparse attention over
 * them as above.  out_blocks [n_seq][top_blocks] (nullable; -1 past the
 * number of blocks) receives the selection. */
hmm_status_t hmm_block_sparse_decode_bf16(const uint16_t* q, const float* summaries,
                                          const uint16_t* k_pages, const uint16_t* v_pages,
                                          int64_t n_pages, const int32_t* page_table,
                                          int64_t n_seq, int64_t pages_per_seq,
                                          int64_t seq_len, int64_t page_tokens,
                                          int64_t block_tokens, int64_t D, int64_t top_blocks,
                                          int32_t* out_blocks, float* out, void* workspace,
                                          size_t workspace_bytes, void* stream);

/* The same step without waiting for `stream`: page-table entries outside
 * [0, n_pages) and negative block ids set bits in *device_status (an int32
 * in device memory the caller zeroes; HMM_STATUS_PAGE_BOUNDS,
 * HMM_STATUS_BLOCK_BOUNDS) instead of making the call return
 * HMM_ERR_BOUNDS; the kernels never follow them.  hmm_status_read waits for
 * `stream` and turns the bits of a device status word into a status:
 * HMM_ERR_BOUNDS for the two above, HMM_ERR_TIMEOUT for HMM_STATUS_TIMEOUT,
 * HMM_ERR_UNSUPPORTED for HMM_STATUS_POOL_OVERFLOW.  For loops that check
 * once per many steps. */
#define HMM_STATUS_PAGE_BOUNDS 1
#define HMM_STATUS_BLOCK_BOUNDS 2
#define HMM_STATUS_TIMEOUT 4
#define HMM_STATUS_POOL_OVERFLOW 8
hmm_status_t hmm_block_sparse_decode_bf16_async(
    const uint16_t* q, const float* summaries, const uint16_t* k_pages, const uint16_t* v_pages,
    int64_t n_pages, const int32_t* page_table, int64_t n_seq, int64_t pages_per_seq,
    int64_t seq_len, int64_t page_tokens, int64_t block_tokens, int64_t D, int64_t top_blocks,
    int32_t* out_blocks, float* out, int32_t* device_status, void* workspace,
    size_t workspace_bytes, void* stream);
hmm_status_t hmm_status_read(const int32_t* device_status, void* stream);

/* ----------------------------------------------------------------- BM25
 * FusedBM25Retrieval (reference steps/example_kernel/bm25_fpga_retrieval.cpp:
 * 143-205) over a CSR inverted index: postings of term t are
 * [term_ptr[t], term_ptr[t+1]) with ascending doc ids post_doc (int32) and
 * term frequencies post_tf (uint16); doc_len[d] = sum of doc d's term
 * frequencies.  Scores are fp64 BM25 (k1 = 1.2, b = 0.75) summed over the
 * query's distinct in-vocabulary terms in ascending term-id order (the
 * reference sums in unordered_map order), bit-identical to the reference's
 * doubles for that order.  Top-k best first, ties to the lowest doc id; docs
 * without a query term score 0.0 and rank like any other doc.
 *
 * hmm_bm25_stats_host (host arrays, no device work): idf[t] =
 * log((N - df + 0.5) / (df + 0.5) + 1.0) (0 for df = 0) and avg_dl exactly
 * as the reference computes them (:158-178), with the host's libm. */
hmm_status_t hmm_bm25_stats_host(const int64_t* term_ptr, int64_t n_terms,
                                 const int32_t* doc_len, int64_t n_docs, double* idf,
                                 double* avg_dl);

/* Index preparation, once per index (device arrays): skips
 * [n_terms][ceil(n_docs/HMM_BM25_RANGE_DOCS)+1] int32 (hmm_bm25_skips_count
 * entries): the first posting of each term at each doc-range boundary; impact
 * [n_postings] fp64: the amount posting p adds to its doc's score,
 * idf * (tf * (k1 + 1)) / (tf + k1 * (1 - b + b * dl / avg_dl)) with the
 * reference's operation order (it depends on the term, the doc and corpus
 * statistics only; the reference ignores the query's own term frequency).
 * idf [n_terms] fp64 is the device copy of hmm_bm25_stats_host's.  A posting
 * whose doc id is outside [0, n_docs) returns HMM_ERR_BOUNDS (the call waits
 * for `stream`); workspace >= 256 bytes. */
#define HMM_BM25_RANGE_DOCS 4096
size_t hmm_bm25_skips_count(int64_t n_terms, int64_t n_docs);
hmm_status_t hmm_bm25_prepare(const int64_t* term_ptr, const int32_t* post_doc,
                              const uint16_t* post_tf, int64_t n_terms, const int32_t* doc_len,
                              int64_t n_docs, const double* idf, double avg_dl, int32_t* skips,
                              double* impact, void* workspace, size_t workspace_bytes,
                              void* stream);

/* Top-k per query over the prepared index.  qterms [n_queries][qlen] int32
 * (ids outside [0, n_terms) and repeats are ignored; qlen <= 64),
 * 1 <= k <= 128 with ceil(n_docs/HMM_BM25_RANGE_DOCS) * k <= 16384.
 * out_idx [n_queries][k] int32 (-1 past min(k, n_docs)), out_scores
 * [n_queries][k] fp64 or NULL.  Asynchronous. */
size_t hmm_bm25_topk_workspace_size(int64_t n_docs, int64_t n_queries, int64_t k);
hmm_status_t hmm_bm25_topk_csr(const int32_t* post_doc, const double* impact,
                               int64_t n_postings, int64_t n_terms, int64_t n_docs,
                               const int32_t* skips, const int32_t* qterms, int64_t n_queries,
                               int64_t qlen, int64_t k, int32_t* out_idx, double* out_scores,
                               void* workspace, size_t workspace_bytes, void* stream);

/* The inverted index built on the device from per-document term counts
 * (replaces the CPU index build behind BuildMemory<TextDBData, BM25IndexMemory>,
 * steps/build_memory.h:183-247, over the reference's term_freq.bin layout,
 * rag_test/export_bm25_data.py:13-27): document d's entries are
 * [doc_ptr[d], doc_ptr[d+1]) of terms (vocabulary index in [0, n_terms)) and
 * counts (in [1, 65535]), each term at most once per document.  Writes
 * term_ptr [n_terms+1] int64, post_doc / post_tf [doc_ptr[n_docs]] with the
 * documents of every term ascending, and doc_len [n_docs] = the sum of each
 * document's counts.  Waits for `stream` to check the inputs: bad doc_ptr or
 * counts give HMM_ERR_INVALID, a term outside the vocabulary HMM_ERR_BOUNDS.
 * Workspace: hmm_bm25_csr_workspace_size bytes (4 B per term per 1,024
 * documents). */
size_t hmm_bm25_csr_workspace_size(int64_t n_docs, int64_t n_terms);
hmm_status_t hmm_bm25_csr_from_docs(const int64_t* doc_ptr, const int32_t* terms,
                                    const uint32_t* counts, int64_t n_docs, int64_t n_terms,
                                    int64_t* term_ptr, int32_t* post_doc, uint16_t* post_tf,
                                    int32_t* doc_len, void* workspace, size_t workspace_bytes,
                                    void* stream);

/* ------------------------------------------------------------ indexers
 * int16 sparse-attention indexers of one index head (the CPU references in
 * kernels/lserve/indexer_lserve_tb.cpp:20-92,
 * kernels/seerattention/indexer_seer_token_budget_tb.cpp:19-73,
 * kernels/seerattention/indexer_seer_threshold_tb.cpp:18-77).
 * past [L][D], queries [n_queries][D], new_keys [n_queries][D] int16 (4-byte
 * aligned), D even <= 256.  Query q sits at position L + q/8 and sees
 * positions 0 .. L + q/8: position p < L is past[p], position L + g is
 * new_keys[min(8g + 7, q)].  Scores are exact int64 dot products (float
 * where the reference converts them).  Top-k outputs are best first, ties to
 * the lowest position / block, -1 padded; bit-exact. */
size_t hmm_indexer_workspace_size(int64_t L, int64_t n_queries);

/* LServe: per query, the top-k blocks of `block` positions (a power of two
 * <= 32; the reference uses 16) by the maximum float score in the block.
 * out [n_queries][topk] int32. */
hmm_status_t hmm_lserve_topk_i16(const int16_t* past, int64_t L, const int16_t* queries,
                                 const int16_t* new_keys, int64_t n_queries, int64_t D,
                                 int64_t topk, int64_t block, int32_t* out, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* SeerAttention token budget: per query, the top-k positions by float
 * score.  out [n_queries][topk] int32. */
hmm_status_t hmm_seer_budget_i16(const int16_t* past, int64_t L, const int16_t* queries,
                                 const int16_t* new_keys, int64_t n_queries, int64_t D,
                                 int64_t topk, int32_t* out, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* SeerAttention threshold: bit p % 64 of word p / 64 of query q's row is set
 * iff position p is visible and dot > threshold (strict).  out_bitmap
 * [n_queries][hmm_seer_words_per_query(L, n_queries)] uint64 (rows cover the
 * last query's window rounded up to 128 positions). */
int64_t hmm_seer_words_per_query(int64_t L, int64_t n_queries);
hmm_status_t hmm_seer_threshold_i16(const int16_t* past, int64_t L, const int16_t* queries,
                                    const int16_t* new_keys, int64_t n_queries, int64_t D,
                                    int64_t threshold, uint64_t* out_bitmap, void* stream);

/* -------------------------------------------------------- DSA indexer
 * DSA lightning indexer (reference kernels/dsa_indexer/indexer_tb.cpp:17-57,
 * multi-head FP8 form of kernels/deepseek_engram/deepseek_v32_dsa_bench.py:
 * 77-101) on FP8 tensor cores: for query token t (position pos0 + t) and
 * key j <= pos0 + t, score = sum_h w[t][h] * ReLU(q[t][h] . k[j]), then the
 * topk best keys per token (best first, ties to the lowest key, -1 past the
 * number of visible keys).
 *   q [T][H][128] e4m3, keys [L][128] e4m3, w [T][H] fp32 (16-byte aligned),
 *   H in {16, 32, 64}, topk <= 4096, pos0 >= -1.
 *   out_idx [T][topk] int32; out_scores [T][topk] fp32 or NULL;
 *   all_scores [T][L] fp32 or NULL: the tensor-core pass's approximate score
 *   of every key (-inf where not visible), for inspection.
 * The selection and out_scores are the reference's exactly: exact integer
 * dots, (float) ReLU, fp32 head sum in head order.  Tensor cores score every
 * key approximately, and the keys whose approximate score could reach a
 * token's k-th are rescored exactly; a token whose candidates do not settle
 * its top-k is recomputed from its exact row.  The workspace holds no
 * [T][L] score matrix.  Waits for `stream`; HMM_ERR_TIMEOUT if a bounded
 * device wait gave up; HMM_ERR_INVALID for e4m3 NaN encodings in q or keys. */
size_t hmm_dsa_indexer_fp8_workspace_size(int64_t T, int64_t H, int64_t L, int64_t topk);
hmm_status_t hmm_dsa_indexer_fp8(const uint8_t* q, const uint8_t* keys, const float* w,
                                 int64_t T, int64_t H, int64_t L, int64_t D, int64_t pos0,
                                 int64_t topk, int32_t* out_idx, float* out_scores,
                                 float* all_scores, void* workspace, size_t workspace_bytes,
                                 void* stream);

/* ------------------------------------------------------ instrumentation
 * No reference counterpart (the reference steps are timed by their callers).
 * hmm_kernel_launches: kernels this library has launched since it was loaded.
 * hmm_profile_enable(1): from then on, record a CUDA event pair on the
 * launching stream around each launch of the dominant kernel of an entry
 * point (tc_score_select_kernel, bsa_split_kernel); hmm_profile_read waits
 * for the recorded pairs and
 * returns their summed duration and count, then forgets them. */
int64_t hmm_kernel_launches(void);
hmm_status_t hmm_profile_enable(int enable);
hmm_status_t hmm_profile_read(double* total_ms, int64_t* launches);

/* Test hook, no reference counterpart.  Sets the limit of every bounded
 * pipeline wait inside the tensor-core kernels (tc_score_select_kernel,
 * dsa_scores_kernel) for the calls that follow, in nanoseconds; a negative
 * value restores the default of 2 s.  A wait that runs out makes its CTA let
 * the copies and MMAs already in flight complete, then exit, and the entry
 * point returns HMM_ERR_TIMEOUT with its outputs invalid.  With 0, the first
 * wait that finds its pipeline stage not yet ready gives up: tests use it to
 * exercise that path without a fault or a hang. */
hmm_status_t hmm_debug_set_wait_limit_ns(int64_t ns);

#ifdef __cplusplus
}
#endif

#endif /* HETEROMM_CUDA_H_ */
