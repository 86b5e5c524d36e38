/*
 * hmm_oracle.c — CPU oracle (test infrastructure only; see hmm_oracle.h).
 *
 * Built with -O2 -ffp-contract=off and no -march so that every fp32/fp64
 * expression rounds exactly as the reference's g++ -O2 x86-64 build does.
 * Loops over independent queries may run on OpenMP threads; each output is
 * computed by one thread in the reference's order, so results do not depend
 * on the thread count.
 */
#include "hmm_oracle.h"

#include <math.h>
#include <omp.h>
#include <stdlib.h>
#include <string.h>

/* Threads of the oracle's OpenMP loops (a launcher may have pinned the
 * process to one thread through OMP_NUM_THREADS). */
void orc_set_threads(int n) {
    if (n > 0) omp_set_num_threads(n);
}

/* ------------------------------------------------------------------ keys */

uint32_t orc_f32_key(float f) {
    uint32_t u;
    if (f != f) return 0u;         /* NaN ranks below every number */
    if (f == 0.0f) f = 0.0f;       /* -0.0 ties with +0.0 */
    memcpy(&u, &f, 4);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

static uint64_t f64_key(double f) {
    uint64_t u;
    if (f != f) return 0ull;
    if (f == 0.0) f = 0.0;
    memcpy(&u, &f, 8);
    return (u & 0x8000000000000000ull) ? ~u : (u | 0x8000000000000000ull);
}

static float bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* -------------------------------------------------- bounded top-k heap */
/* Entries compare by (key desc, idx asc).  The heap is a min-heap on that
 * order: the root is the worst entry kept. */
typedef struct { uint64_t key; int64_t idx; } kent_t;

static int kent_better(kent_t a, kent_t b) {
    return a.key > b.key || (a.key == b.key && a.idx < b.idx);
}

static void heap_sift_down(kent_t* h, int64_t n, int64_t i) {
    for (;;) {
        int64_t l = 2 * i + 1, r = l + 1, w = i;
        if (l < n && kent_better(h[w], h[l])) w = l;
        if (r < n && kent_better(h[w], h[r])) w = r;
        if (w == i) return;
        kent_t t = h[i]; h[i] = h[w]; h[w] = t;
        i = w;
    }
}

static void heap_sift_up(kent_t* h, int64_t i) {
    while (i > 0) {
        int64_t p = (i - 1) / 2;
        if (!kent_better(h[p], h[i])) return;
        kent_t t = h[i]; h[i] = h[p]; h[p] = t;
        i = p;
    }
}

typedef struct { kent_t* h; int64_t n, cap; } topk_t;

static void topk_init(topk_t* t, int64_t k) {
    t->h = (kent_t*)malloc(sizeof(kent_t) * (size_t)(k > 0 ? k : 1));
    t->n = 0;
    t->cap = k;
}

static void topk_push(topk_t* t, uint64_t key, int64_t idx) {
    kent_t e = {key, idx};
    if (t->cap <= 0) return;
    if (t->n < t->cap) {
        t->h[t->n] = e;
        heap_sift_up(t->h, t->n);
        t->n++;
    } else if (kent_better(e, t->h[0])) {
        t->h[0] = e;
        heap_sift_down(t->h, t->n, 0);
    }
}

static int kent_cmp_desc(const void* a, const void* b) {
    kent_t x = *(const kent_t*)a, y = *(const kent_t*)b;
    if (kent_better(x, y)) return -1;
    if (kent_better(y, x)) return 1;
    return 0;
}

/* Sorts best first; returns the count. */
static int64_t topk_finish(topk_t* t) {
    qsort(t->h, (size_t)t->n, sizeof(kent_t), kent_cmp_desc);
    return t->n;
}

static void topk_free(topk_t* t) { free(t->h); }

/* ------------------------------------------------------------------ a-1 */

/* inner_product_compute.cpp:23-29: dot = 0; dot += m[i][j] * q[j]; */
static float dot_f32(const float* a, const float* b, int64_t d) {
    float dot = 0.0f;
    for (int64_t j = 0; j < d; ++j) {
        float p = a[j] * b[j];
        dot = dot + p;
    }
    return dot;
}

void orc_ip_score_f32(const float* mem, int64_t n, int64_t d, const float* qry,
                      int64_t nq, float* out) {
    int64_t q;
#pragma omp parallel for schedule(static)
    for (q = 0; q < nq; ++q)
        for (int64_t i = 0; i < n; ++i)
            out[q * n + i] = dot_f32(mem + i * d, qry + q * d, d);
}

static float dot_bf16(const uint16_t* a, const float* bq, int64_t d) {
    float dot = 0.0f;
    for (int64_t j = 0; j < d; ++j) {
        float p = bf16_to_f32(a[j]) * bq[j];
        dot = dot + p;
    }
    return dot;
}

void orc_ip_score_bf16(const uint16_t* mem, int64_t n, int64_t d, const uint16_t* qry,
                       int64_t nq, float* out) {
    int64_t q;
#pragma omp parallel for schedule(static)
    for (q = 0; q < nq; ++q) {
        float* qf = (float*)malloc(sizeof(float) * (size_t)d);
        for (int64_t j = 0; j < d; ++j) qf[j] = bf16_to_f32(qry[q * d + j]);
        for (int64_t i = 0; i < n; ++i) out[q * n + i] = dot_bf16(mem + i * d, qf, d);
        free(qf);
    }
}

/* ------------------------------------------------------------------ a-2 */

/* topk_retrieval.cpp:82-93: k = min(k_, n); partial_sort by scores[a] > scores[b]. */
int64_t orc_topk_f32(const float* scores, int64_t n, int64_t k, int32_t* out_idx) {
    topk_t t;
    int64_t kk = k < n ? k : n, m;
    topk_init(&t, kk);
    for (int64_t i = 0; i < n; ++i) topk_push(&t, orc_f32_key(scores[i]), i);
    m = topk_finish(&t);
    for (int64_t i = 0; i < k; ++i) out_idx[i] = i < m ? (int32_t)t.h[i].idx : -1;
    topk_free(&t);
    return m;
}

int64_t orc_topk_f32_i64(const float* scores, int64_t n, int64_t k, int64_t idx_offset,
                         int64_t* out_idx, float* out_scores) {
    topk_t t;
    int64_t kk = k < n ? k : n, m;
    topk_init(&t, kk);
    for (int64_t i = 0; i < n; ++i) topk_push(&t, orc_f32_key(scores[i]), i);
    m = topk_finish(&t);
    for (int64_t i = 0; i < k; ++i) {
        out_idx[i] = i < m ? t.h[i].idx + idx_offset : -1;
        if (out_scores) out_scores[i] = i < m ? scores[t.h[i].idx] : -INFINITY;
    }
    topk_free(&t);
    return m;
}

/* ------------------------------------------------------------------ a-3 */

/* threshold_retrieval.cpp:144-154: bit set iff scores[i] >= threshold_. */
void orc_threshold_bitmap_f32(const float* scores, int64_t n, float thr, uint64_t* bitmap) {
    int64_t words = (n + 63) / 64;
    memset(bitmap, 0, sizeof(uint64_t) * (size_t)words);
    for (int64_t i = 0; i < n; ++i)
        if (scores[i] >= thr) bitmap[i / 64] |= 1ull << (i % 64);
}

/* -------------------------------------------------------- fused (cfg 1) */

void orc_ip_topk_f32(const float* mem, int64_t n, int64_t d, const float* qry, int64_t nq,
                     int64_t k, float thr, int32_t* out_idx, uint64_t* out_bitmap,
                     float* out_scores) {
    int64_t q;
#pragma omp parallel for schedule(dynamic)
    for (q = 0; q < nq; ++q) {
        float* s = out_scores ? out_scores + q * n : (float*)malloc(sizeof(float) * (size_t)(n ? n : 1));
        for (int64_t i = 0; i < n; ++i) s[i] = dot_f32(mem + i * d, qry + q * d, d);
        orc_topk_f32(s, n, k, out_idx + q * k);
        if (out_bitmap) orc_threshold_bitmap_f32(s, n, thr, out_bitmap + q * ((n + 63) / 64));
        if (!out_scores) free(s);
    }
}

/* -------------------------------------------------------- bf16 (cfg 5) */

/* dot_bf16 of four rows at once: four independent chains, each in the
 * reference's order (multiply, then add, j ascending), so each result equals
 * dot_bf16's bit for bit; only the CPU's latency is hidden. */
static void dot_bf16_x4(const uint16_t* a, int64_t d, const float* bq, float out[4]) {
    float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
    for (int64_t j = 0; j < d; ++j) {
        float p0 = bf16_to_f32(a[j]) * bq[j];
        float p1 = bf16_to_f32(a[d + j]) * bq[j];
        float p2 = bf16_to_f32(a[2 * d + j]) * bq[j];
        float p3 = bf16_to_f32(a[3 * d + j]) * bq[j];
        s0 = s0 + p0;
        s1 = s1 + p1;
        s2 = s2 + p2;
        s3 = s3 + p3;
    }
    out[0] = s0; out[1] = s1; out[2] = s2; out[3] = s3;
}

/* Exact top-k (score desc, row asc) of every query over bf16 rows.  The work
 * is split into (query, row chunk) pieces, each an exact top-k of its chunk,
 * merged per query: the top-k of a union is the top-k of the parts' top-ks,
 * so the result does not depend on the split. */
void orc_ip_topk_bf16(const uint16_t* mem, int64_t n, int64_t d, const uint16_t* qry,
                      int64_t nq, int64_t k, int64_t row_offset, int64_t* out_idx,
                      float* out_scores) {
    const int64_t CH = (int64_t)1 << 20;
    const int64_t nch = n > 0 ? (n + CH - 1) / CH : 1;
    const int64_t kk = k < n ? k : n;
    kent_t* part = (kent_t*)malloc(sizeof(kent_t) * (size_t)(nq * nch * (kk > 0 ? kk : 1)));
    int64_t* part_n = (int64_t*)calloc((size_t)(nq * nch), sizeof(int64_t));
    float* qf_all = (float*)malloc(sizeof(float) * (size_t)(nq * d + 1));
    int64_t w, q;
    for (int64_t i = 0; i < nq * d; ++i) qf_all[i] = bf16_to_f32(qry[i]);
#pragma omp parallel for schedule(dynamic)
    for (w = 0; w < nq * nch; ++w) {
        const int64_t qq = w / nch, c = w % nch;
        const int64_t r0 = c * CH, r1 = r0 + CH < n ? r0 + CH : n;
        const float* qf = qf_all + qq * d;
        topk_t t;
        int64_t i = r0;
        topk_init(&t, kk);
        for (; i + 4 <= r1; i += 4) {
            float s4[4];
            dot_bf16_x4(mem + i * d, d, qf, s4);
            for (int u = 0; u < 4; ++u) topk_push(&t, orc_f32_key(s4[u]), i + u);
        }
        for (; i < r1; ++i) topk_push(&t, orc_f32_key(dot_bf16(mem + i * d, qf, d)), i);
        part_n[w] = topk_finish(&t);
        memcpy(part + w * kk, t.h, sizeof(kent_t) * (size_t)part_n[w]);
        topk_free(&t);
    }
#pragma omp parallel for schedule(dynamic)
    for (q = 0; q < nq; ++q) {
        const float* qf = qf_all + q * d;
        topk_t t;
        int64_t m;
        topk_init(&t, kk);
        for (int64_t c = 0; c < nch; ++c)
            for (int64_t i = 0; i < part_n[q * nch + c]; ++i)
                topk_push(&t, part[(q * nch + c) * kk + i].key, part[(q * nch + c) * kk + i].idx);
        m = topk_finish(&t);
        for (int64_t i = 0; i < k; ++i) {
            int64_t r = i < m ? t.h[i].idx : -1;
            out_idx[q * k + i] = r >= 0 ? r + row_offset : -1;
            out_scores[q * k + i] = r >= 0 ? dot_bf16(mem + r * d, qf, d) : -INFINITY;
        }
        topk_free(&t);
    }
    free(part);
    free(part_n);
    free(qf_all);
}

void orc_shard_merge_topk(const float* cand_scores, const int64_t* cand_idx,
                          int64_t n_shards, int64_t nq, int64_t k, float* out_scores,
                          int64_t* out_idx) {
    for (int64_t q = 0; q < nq; ++q) {
        topk_t t;
        int64_t m;
        topk_init(&t, k);
        for (int64_t s = 0; s < n_shards; ++s)
            for (int64_t i = 0; i < k; ++i) {
                int64_t o = (s * nq + q) * k + i;
                if (cand_idx[o] < 0) continue;
                topk_push(&t, orc_f32_key(cand_scores[o]), cand_idx[o]);
            }
        m = topk_finish(&t);
        for (int64_t i = 0; i < k; ++i) {
            out_idx[q * k + i] = i < m ? t.h[i].idx : -1;
            if (i < m) {
                /* recover the score from its key */
                uint32_t key = (uint32_t)t.h[i].key, u;
                float f;
                u = (key & 0x80000000u) ? (key & 0x7fffffffu) : ~key;
                memcpy(&f, &u, 4);
                out_scores[q * k + i] = f;
            } else {
                out_scores[q * k + i] = -INFINITY;
            }
        }
        topk_free(&t);
    }
}

/* ------------------------------------------------------------------ a-5 */

/* paged_kv_index_builder.cpp:47-80: num_pages = ceil(L/P); pooled[d] summed
 * over the page's tokens in order, divided by the token count as float, then
 * projected: proj[o] = sum_d w[o][d] * pooled[d]. */
int64_t orc_paged_kv_summary_f32(const float* keys, int64_t L, int64_t D, const float* weight,
                                 int64_t out_dim, int64_t page_size, float* out) {
    int64_t pages, p;
    if (L == 0 || D == 0 || out_dim == 0 || page_size <= 0) return 0;
    pages = (L + page_size - 1) / page_size;
#pragma omp parallel for schedule(static)
    for (p = 0; p < pages; ++p) {
        int64_t start = p * page_size;
        int64_t end = start + page_size < L ? start + page_size : L;
        float* pooled = (float*)calloc((size_t)D, sizeof(float));
        for (int64_t t = start; t < end; ++t)
            for (int64_t d = 0; d < D; ++d) pooled[d] = pooled[d] + keys[t * D + d];
        for (int64_t d = 0; d < D; ++d) pooled[d] = pooled[d] / (float)(end - start);
        for (int64_t o = 0; o < out_dim; ++o) {
            float acc = 0.0f;
            for (int64_t d = 0; d < D; ++d) {
                float pr = weight[o * D + d] * pooled[d];
                acc = acc + pr;
            }
            out[p * out_dim + o] = acc;
        }
        free(pooled);
    }
    return pages;
}

int64_t orc_block_mean_f32(const float* keys, int64_t L, int64_t D, int64_t page_size,
                           float* out) {
    int64_t pages, p;
    if (L == 0 || D == 0 || page_size <= 0) return 0;
    pages = (L + page_size - 1) / page_size;
#pragma omp parallel for schedule(static)
    for (p = 0; p < pages; ++p) {
        int64_t start = p * page_size;
        int64_t end = start + page_size < L ? start + page_size : L;
        for (int64_t d = 0; d < D; ++d) {
            float acc = 0.0f;
            for (int64_t t = start; t < end; ++t) acc = acc + keys[t * D + d];
            out[p * D + d] = acc / (float)(end - start);
        }
    }
    return pages;
}

/* Min/max page summaries of the reference's MinMaxIndexMemory
 * (types/memory.h:127-230: for every block a min vector and a max vector,
 * stored min then max): per block of `page_size` tokens and column, the
 * smallest and the largest key (fminf / fmaxf: NaN ignored unless all are). */
int64_t orc_block_minmax_f32(const float* keys, int64_t L, int64_t D, int64_t page_size,
                             float* out) {
    int64_t pages, p;
    if (L == 0 || D == 0 || page_size <= 0) return 0;
    pages = (L + page_size - 1) / page_size;
    for (p = 0; p < pages; ++p) {
        int64_t start = p * page_size;
        int64_t end = start + page_size < L ? start + page_size : L;
        for (int64_t d = 0; d < D; ++d) {
            float mn = keys[start * D + d], mx = mn;
            for (int64_t t = start + 1; t < end; ++t) {
                mn = fminf(mn, keys[t * D + d]);
                mx = fmaxf(mx, keys[t * D + d]);
            }
            out[(2 * p) * D + d] = mn;
            out[(2 * p + 1) * D + d] = mx;
        }
    }
    return pages;
}

/* Top-`top` blocks by the upper bound of q.k over each block's keys,
 * u_b = sum_j max(q_j * min_bj, q_j * max_bj), j ascending, each product
 * rounded before the add; best first, ties to the lower block, -1 past nb. */
void orc_block_select_minmax(const float* q, const float* minmax, int64_t nb, int64_t D,
                             int64_t top, int32_t* out) {
    float* u = (float*)malloc(sizeof(float) * (size_t)(nb ? nb : 1));
    for (int64_t b = 0; b < nb; ++b) {
        float acc = 0.0f;
        for (int64_t j = 0; j < D; ++j) {
            const float lo = q[j] * minmax[(2 * b) * D + j];
            const float hi = q[j] * minmax[(2 * b + 1) * D + j];
            acc = acc + (lo > hi ? lo : hi);
        }
        u[b] = acc;
    }
    for (int64_t i = 0; i < top; ++i) {
        int64_t best = -1;
        for (int64_t b = 0; b < nb; ++b) {
            int taken = 0;
            for (int64_t j = 0; j < i; ++j) taken |= out[j] == (int32_t)b;
            if (taken) continue;
            if (best < 0 || orc_f32_key(u[b]) > orc_f32_key(u[best])) best = b;
        }
        out[i] = (int32_t)best;
    }
    free(u);
}

/* ------------------------------------------------------------------ a-6 */

/* block_sparse_attention.cpp:50-123 */
void orc_block_sparse_attention_f32(const float* keys, const float* values, int64_t L,
                                    int64_t D, const int32_t* blocks, int64_t nb,
                                    const float* q, int64_t page_size, float* out) {
    int64_t ntok = 0, cap = 0;
    int32_t* tok = NULL;
    float *s, *e, mx, sum, scale;
    for (int64_t d = 0; d < D; ++d) out[d] = 0.0f;
    if (L == 0 || D == 0 || nb == 0) return;
    scale = 1.0f / sqrtf((float)D);
    /* :53-63 token list = concatenation of [b*P, min(b*P+P, L)) in top-k order */
    for (int64_t i = 0; i < nb; ++i) {
        int32_t st = blocks[i] * (int32_t)page_size;
        int32_t en = st + (int32_t)page_size < (int32_t)L ? st + (int32_t)page_size : (int32_t)L;
        for (int32_t t = st; t < en; ++t) {
            if (ntok == cap) {
                cap = cap ? cap * 2 : 256;
                tok = (int32_t*)realloc(tok, sizeof(int32_t) * (size_t)cap);
            }
            tok[ntok++] = t;
        }
    }
    if (ntok == 0) { free(tok); return; }
    s = (float*)malloc(sizeof(float) * (size_t)ntok);
    e = (float*)malloc(sizeof(float) * (size_t)ntok);
    /* :77-87 */
    for (int64_t i = 0; i < ntok; ++i) {
        float dot = 0.0f;
        for (int64_t d = 0; d < D; ++d) {
            float p = q[d] * keys[(int64_t)tok[i] * D + d];
            dot = dot + p;
        }
        s[i] = dot * scale;
    }
    /* :93-108 max_element keeps the first maximum */
    mx = s[0];
    for (int64_t i = 1; i < ntok; ++i) if (mx < s[i]) mx = s[i];
    sum = 0.0f;
    for (int64_t i = 0; i < ntok; ++i) {
        e[i] = expf(s[i] - mx);
        sum = sum + e[i];
    }
    /* :112-123 */
    for (int64_t i = 0; i < ntok; ++i) {
        float w = e[i] / sum;
        for (int64_t d = 0; d < D; ++d) {
            float p = w * values[(int64_t)tok[i] * D + d];
            out[d] = out[d] + p;
        }
    }
    free(s); free(e); free(tok);
}

/* ------------------------------------------------------------------ a-7 */

int64_t orc_block_pages(const int32_t* page_table, int64_t pages_per_seq, int64_t seq,
                        const int32_t* blocks, int64_t nb, int64_t pages_per_block,
                        int32_t* out_pages) {
    int64_t n = 0;
    for (int64_t i = 0; i < nb; ++i) {
        int64_t p0 = (int64_t)blocks[i] * pages_per_block;
        for (int64_t p = p0; p < p0 + pages_per_block; ++p) {
            if (p < 0 || p >= pages_per_seq) continue;
            out_pages[n++] = page_table[seq * pages_per_seq + p];
        }
    }
    return n;
}

/* ------------------------------------------------------------------ a-8 */

/* indexer_tb.cpp:27-46: qk exact in int64, ReLU, total += w[h] * (float)qk. */
int64_t orc_dsa_indexer_i16(const int16_t* q, int64_t H, int64_t D, const int16_t* keys,
                            int64_t L, const float* w, int64_t topk, int32_t* out_idx,
                            float* out_scores) {
    topk_t t;
    int64_t m;
    topk_init(&t, topk < L ? topk : L);
    for (int64_t k = 0; k < L; ++k) {
        float total = 0.0f;
        for (int64_t h = 0; h < H; ++h) {
            int64_t qk = 0;
            for (int64_t d = 0; d < D; ++d)
                qk += (int64_t)q[h * D + d] * (int64_t)keys[k * D + d];
            if (qk < 0) qk = 0;
            {
                float p = w[h] * (float)qk;
                total = total + p;
            }
        }
        topk_push(&t, orc_f32_key(total), k);
    }
    m = topk_finish(&t);
    for (int64_t i = 0; i < topk; ++i) {
        out_idx[i] = i < m ? (int32_t)t.h[i].idx : -1;
        if (out_scores) {
            uint32_t key = (uint32_t)t.h[i < m ? i : 0].key, u;
            float f;
            u = (key & 0x80000000u) ? (key & 0x7fffffffu) : ~key;
            memcpy(&f, &u, 4);
            out_scores[i] = i < m ? f : -INFINITY;
        }
    }
    topk_free(&t);
    return m;
}

/* e4m3 (OCP FP8, bias 7, no infinities, S.1111.111 = NaN): value * 2^9. */
int32_t orc_e4m3_scaled(uint8_t v) {
    int32_t e = (v >> 3) & 0xf, m = v & 7, mag;
    if (e == 15 && m == 7) return 0;
    mag = e == 0 ? m : (8 + m) << (e - 1);
    return (v & 0x80) ? -mag : mag;
}

float orc_dsa_score_fp8(const uint8_t* q_t, int64_t H, int64_t D, const uint8_t* key,
                        const float* w_t) {
    float total = 0.0f;
    for (int64_t h = 0; h < H; ++h) {
        int64_t acc = 0;
        float x;
        for (int64_t d = 0; d < D; ++d)
            acc += (int64_t)orc_e4m3_scaled(q_t[h * D + d]) * (int64_t)orc_e4m3_scaled(key[d]);
        if (acc < 0) acc = 0;
        /* exact dot = acc * 2^-18; (float) rounds once */
        x = (float)ldexp((double)acc, -18);
        {
            float p = w_t[h] * x;
            total = total + p;
        }
    }
    return total;
}

void orc_dsa_indexer_fp8(const uint8_t* q, int64_t T, int64_t H, int64_t D,
                         const uint8_t* keys, int64_t L, const float* w, int64_t pos0,
                         int64_t topk, int32_t* out_idx, float* out_scores) {
    int64_t t;
#pragma omp parallel for schedule(dynamic)
    for (t = 0; t < T; ++t) {
        int64_t visible = pos0 + t + 1 < L ? pos0 + t + 1 : L, m;
        topk_t tk;
        if (visible < 0) visible = 0;
        topk_init(&tk, topk < visible ? topk : visible);
        for (int64_t j = 0; j < visible; ++j)
            topk_push(&tk, orc_f32_key(orc_dsa_score_fp8(q + t * H * D, H, D, keys + j * D,
                                                         w + t * H)), j);
        m = topk_finish(&tk);
        for (int64_t i = 0; i < topk; ++i) {
            out_idx[t * topk + i] = i < m ? (int32_t)tk.h[i].idx : -1;
            if (out_scores)
                out_scores[t * topk + i] =
                    i < m ? orc_dsa_score_fp8(q + t * H * D, H, D, keys + tk.h[i].idx * D,
                                              w + t * H)
                          : -INFINITY;
        }
        topk_free(&tk);
    }
}

void orc_dsa_scores_fp8(const uint8_t* q, int64_t T, int64_t H, int64_t D, const uint8_t* keys,
                        int64_t L, const float* w, int64_t pos0, float* out) {
    int64_t t;
#pragma omp parallel for schedule(dynamic)
    for (t = 0; t < T; ++t)
        for (int64_t j = 0; j < L; ++j)
            out[t * L + j] = j <= pos0 + t
                                 ? orc_dsa_score_fp8(q + t * H * D, H, D, keys + j * D, w + t * H)
                                 : -INFINITY;
}

/* --------------------------------------------------------- a-9 / a-10 */

/* Key visible at position pos to query q (indexer_lserve_tb.cpp:36-45,
 * indexer_seer_threshold_tb.cpp:33-44): past keys below L; position L+g
 * holds the last new key i <= q with i/8 == g. */
static const int16_t* key_at(const int16_t* past, int64_t L, const int16_t* new_keys,
                             int64_t D, int64_t q, int64_t pos) {
    int64_t g, i;
    if (pos < L) return past + pos * D;
    g = pos - L;
    i = 8 * g + 7 < q ? 8 * g + 7 : q;
    return new_keys + i * D;
}

static int64_t dot_i16(const int16_t* a, const int16_t* b, int64_t D) {
    int64_t acc = 0;
    for (int64_t d = 0; d < D; ++d) acc += (int64_t)a[d] * (int64_t)b[d];
    return acc;
}

void orc_lserve_topk_i16(const int16_t* past, int64_t L, const int16_t* queries,
                         const int16_t* new_keys, int64_t nq, int64_t D, int64_t topk,
                         int64_t block, int32_t* out) {
    int64_t q;
#pragma omp parallel for schedule(dynamic)
    for (q = 0; q < nq; ++q) {
        int64_t cur = L + q / 8, ns = cur + 1, nblk = (ns + block - 1) / block, m;
        topk_t t;
        topk_init(&t, topk < nblk ? topk : nblk);
        /* :62-79 block score = max over its scores, init -1e30f, strict > */
        for (int64_t b = 0; b < nblk; ++b) {
            float mx = -1e30f;
            int64_t e = (b + 1) * block < ns ? (b + 1) * block : ns;
            for (int64_t k = b * block; k < e; ++k) {
                float s = (float)dot_i16(queries + q * D, key_at(past, L, new_keys, D, q, k), D);
                if (s > mx) mx = s;
            }
            topk_push(&t, orc_f32_key(mx), b);
        }
        m = topk_finish(&t);
        for (int64_t i = 0; i < topk; ++i) out[q * topk + i] = i < m ? (int32_t)t.h[i].idx : -1;
        topk_free(&t);
    }
}

void orc_seer_budget_i16(const int16_t* past, int64_t L, const int16_t* queries,
                         const int16_t* new_keys, int64_t nq, int64_t D, int64_t topk,
                         int32_t* out) {
    int64_t q;
#pragma omp parallel for schedule(dynamic)
    for (q = 0; q < nq; ++q) {
        int64_t cur = L + q / 8, m;
        topk_t t;
        topk_init(&t, topk < cur + 1 ? topk : cur + 1);
        for (int64_t k = 0; k <= cur; ++k) {
            float s = (float)dot_i16(queries + q * D, key_at(past, L, new_keys, D, q, k), D);
            topk_push(&t, orc_f32_key(s), k);
        }
        m = topk_finish(&t);
        for (int64_t i = 0; i < topk; ++i) out[q * topk + i] = i < m ? (int32_t)t.h[i].idx : -1;
        topk_free(&t);
    }
}

int64_t orc_seer_words_per_query(int64_t L, int64_t nq) {
    int64_t cur = L + (nq > 0 ? (nq - 1) / 8 : 0);
    return ((cur + 128) / 128) * 2;
}

/* indexer_seer_threshold_tb.cpp:47-74: blocks of 128 keys; bit set iff the
 * key is visible (<= current_pos) and dot > THRESHOLD (strict). */
void orc_seer_threshold_i16(const int16_t* past, int64_t L, const int16_t* queries,
                            const int16_t* new_keys, int64_t nq, int64_t D,
                            int64_t threshold, uint64_t* out) {
    int64_t wpq = orc_seer_words_per_query(L, nq), q;
    memset(out, 0, sizeof(uint64_t) * (size_t)(wpq * nq));
#pragma omp parallel for schedule(dynamic)
    for (q = 0; q < nq; ++q) {
        int64_t cur = L + q / 8;
        for (int64_t k = 0; k <= cur; ++k)
            if (dot_i16(queries + q * D, key_at(past, L, new_keys, D, q, k), D) > threshold)
                out[q * wpq + k / 64] |= 1ull << (k % 64);
    }
}

/* ----------------------------------------------------------------- a-11 */

/* bm25_fpga_retrieval.cpp:176-178: idf = log((N - df + 0.5) / (df + 0.5) + 1.0).
 * Terms with df == 0 are absent from df_map and are skipped (:174-175). */
void orc_bm25_idf(const int64_t* term_ptr, int64_t n_terms, int64_t n_docs, double* idf) {
    const double N = (double)n_docs;
    for (int64_t t = 0; t < n_terms; ++t) {
        double df = (double)(term_ptr[t + 1] - term_ptr[t]);
        idf[t] = df > 0 ? log((N - df + 0.5) / (df + 0.5) + 1.0) : 0.0;
    }
}

/* :158-169: avg_dl accumulated in doc order, divided by N. */
double orc_bm25_avgdl(const int32_t* doc_len, int64_t n_docs) {
    double avg = 0.0;
    for (int64_t i = 0; i < n_docs; ++i) avg += (double)doc_len[i];
    return avg / (double)n_docs;
}

static int cmp_i32(const void* a, const void* b) {
    int32_t x = *(const int32_t*)a, y = *(const int32_t*)b;
    return (x > y) - (x < y);
}

void orc_bm25_topk(const int64_t* term_ptr, const int32_t* post_doc, const uint16_t* post_tf,
                   int64_t n_terms, const int32_t* doc_len, int64_t n_docs,
                   const int32_t* qterms, int64_t nq, int64_t qlen, int64_t k,
                   int32_t* out_idx, double* out_scores) {
    const double k1 = 1.2, b = 0.75;
    double* idf = (double*)malloc(sizeof(double) * (size_t)(n_terms ? n_terms : 1));
    double avg_dl;
    int64_t q;
    if (n_docs == 0) {
        for (int64_t i = 0; i < nq * k; ++i) { out_idx[i] = -1; if (out_scores) out_scores[i] = 0.0; }
        free(idf);
        return;
    }
    orc_bm25_idf(term_ptr, n_terms, n_docs, idf);
    avg_dl = orc_bm25_avgdl(doc_len, n_docs);
#pragma omp parallel for schedule(dynamic)
    for (q = 0; q < nq; ++q) {
        double* sc = (double*)calloc((size_t)n_docs, sizeof(double));
        int32_t* terms = (int32_t*)malloc(sizeof(int32_t) * (size_t)(qlen ? qlen : 1));
        int64_t nt = 0, m;
        topk_t t;
        for (int64_t i = 0; i < qlen; ++i) {
            int32_t tid = qterms[q * qlen + i];
            if (tid >= 0 && tid < n_terms) terms[nt++] = tid;
        }
        qsort(terms, (size_t)nt, sizeof(int32_t), cmp_i32);
        for (int64_t i = 0; i < nt; ++i) {
            int32_t tid = terms[i];
            if (i > 0 && terms[i - 1] == tid) continue;          /* map keys are distinct */
            if (term_ptr[tid + 1] == term_ptr[tid]) continue;    /* not in df_map */
            for (int64_t p = term_ptr[tid]; p < term_ptr[tid + 1]; ++p) {
                int32_t d = post_doc[p];
                double tf = (double)post_tf[p];
                double dl = (double)doc_len[d];
                /* :186 idf * (tf * (k1 + 1.0)) / (tf + k1 * (1.0 - b + b * dl / avg_dl)) */
                double num = idf[tid] * (tf * (k1 + 1.0));
                double den = tf + k1 * ((1.0 - b) + (b * dl) / avg_dl);
                sc[d] = sc[d] + num / den;
            }
        }
        topk_init(&t, k < n_docs ? k : n_docs);
        for (int64_t d = 0; d < n_docs; ++d) topk_push(&t, f64_key(sc[d]), d);
        m = topk_finish(&t);
        for (int64_t i = 0; i < k; ++i) {
            out_idx[q * k + i] = i < m ? (int32_t)t.h[i].idx : -1;
            if (out_scores) out_scores[q * k + i] = i < m ? sc[t.h[i].idx] : 0.0;
        }
        topk_free(&t);
        free(terms);
        free(sc);
    }
    free(idf);
}
