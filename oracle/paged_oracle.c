/*
 * CPU oracle for the paged-attention hot path (test infrastructure only; see paged_oracle.h).
 *
 * Numerics follow the reference kernel csrc/src/paged_kernels.cpp:7-105 operation by operation:
 * fp32 dot products accumulated sequentially over head_dim, score = dot * scaling, masked scores
 * = -inf, a row whose scores are all masked uses max = 0, exponentials only for scores > -1e30,
 * normalisation by one reciprocal only when the sum is positive, and the PV product accumulated
 * sequentially over the context.  Built without -ffast-math and with -ffp-contract=off so the
 * compiler keeps that order.
 */
#include "paged_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* Softmax-weighted sum for one (query row, q-head), scores already in `scores[0..n)` with
 * masked entries at -inf.  Restates paged_kernels.cpp:75-103 (the part after the QK loop). */
static void softmax_pv_row(float* scores, int32_t n, float max_score,
                           const float* const* v_rows, int32_t head_dim, float* out_row) {
    if (max_score == -INFINITY) max_score = 0.0f;                 /* :75 */
    float total = 0.0f;
    for (int32_t c = 0; c < n; ++c) {                             /* :77-85 */
        if (scores[c] > -1e30f) {
            scores[c] = expf(scores[c] - max_score);
            total += scores[c];
        } else {
            scores[c] = 0.0f;
        }
    }
    if (total > 0.0f) {                                           /* :86-91 */
        const float inv = 1.0f / total;
        for (int32_t c = 0; c < n; ++c) scores[c] *= inv;
    }
    for (int32_t d = 0; d < head_dim; ++d) {                      /* :93-103 */
        float acc = 0.0f;
        for (int32_t c = 0; c < n; ++c) acc += scores[c] * v_rows[c][d];
        out_row[d] = acc;
    }
}

static float dot_row(const float* a, const float* b, int32_t n) {
    float acc = 0.0f;                                             /* :66-69 */
    for (int32_t d = 0; d < n; ++d) acc += a[d] * b[d];
    return acc;
}

/* The same arithmetic as dot_row for 8 keys at once: kt holds the keys transposed ([d][8]), so
 * lane j accumulates q[d] * k_j[d] over d in the same sequential order dot_row uses, and the
 * compiler may put the 8 independent sums in one SIMD register (no reassociation). */
static void dot_rows8(const float* q, const float* kt, int32_t n, float* out8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int32_t d = 0; d < n; ++d) {
        const float qd = q[d];
#pragma omp simd
        for (int32_t j = 0; j < 8; ++j) acc[j] += qd * kt[d * 8 + j];
    }
    for (int32_t j = 0; j < 8; ++j) out8[j] = acc[j];
}

/* softmax_pv_row with the PV product taken key by key: out[d] still receives
 * scores[0]*v_0[d] + scores[1]*v_1[d] + ... in that order, one rounding per step, so the result
 * is bit-identical; the loop over d is what vectorises.  `acc` holds head_dim floats. */
static void softmax_pv_row_by_key(float* scores, int32_t n, float max_score,
                                  const float* const* v_rows, int32_t head_dim, float* acc,
                                  float* out_row) {
    if (max_score == -INFINITY) max_score = 0.0f;
    float total = 0.0f;
    for (int32_t c = 0; c < n; ++c) {
        if (scores[c] > -1e30f) {
            scores[c] = expf(scores[c] - max_score);
            total += scores[c];
        } else {
            scores[c] = 0.0f;
        }
    }
    if (total > 0.0f) {
        const float inv = 1.0f / total;
        for (int32_t c = 0; c < n; ++c) scores[c] *= inv;
    }
    for (int32_t d = 0; d < head_dim; ++d) acc[d] = 0.0f;
    for (int32_t c = 0; c < n; ++c) {
        const float pc = scores[c];
        const float* v = v_rows[c];
#pragma omp simd
        for (int32_t d = 0; d < head_dim; ++d) acc[d] += pc * v[d];
    }
    for (int32_t d = 0; d < head_dim; ++d) out_row[d] = acc[d];
}

void oracle_paged_attention(const float* query, const float* key_cache, const float* value_cache,
                            int32_t layer_idx, OraclePagedDims dims, const int32_t* gather_slots,
                            const uint8_t* attention_mask, float scaling, float* output,
                            float* scratch) {
    const int32_t hq = dims.num_query_heads, nq = dims.num_query_tokens, hd = dims.head_dim;
    const int32_t hkv = dims.num_kv_heads, nctx = dims.num_context_tokens;
    if (nctx == 0) {                                              /* :30-34 */
        memset(output, 0, (size_t)nq * hq * hd * sizeof(float));
        return;
    }
    const int64_t row = (int64_t)hkv * hd;                        /* floats per cache slot */
    const int64_t per_layer = (int64_t)dims.total_blocks * dims.block_size * row;
    const float* lk = key_cache + (int64_t)layer_idx * per_layer;
    const float* lv = value_cache + (int64_t)layer_idx * per_layer;
    const int32_t group = hq / hkv;                               /* :41, GQA h_kv = h_q / group */

#pragma omp parallel for collapse(2) schedule(static)
    for (int32_t t = 0; t < nq; ++t) {
        for (int32_t h = 0; h < hq; ++h) {
            const int32_t g = h / group;
            const float* qrow = query + ((int64_t)h * nq + t) * hd;           /* [Hq][Nq][D] */
            float* sc = scratch + ((int64_t)t * hq + h) * nctx;
            const float** vrows = (const float**)malloc(sizeof(float*) * (size_t)nctx);
            float mx = -INFINITY;
            for (int32_t c = 0; c < nctx; ++c) {
                const int64_t slot = gather_slots[c];
                vrows[c] = lv + slot * row + (int64_t)g * hd;
                if (!attention_mask[(int64_t)t * nctx + c]) { sc[c] = -INFINITY; continue; }
                const float s = dot_row(qrow, lk + slot * row + (int64_t)g * hd, hd) * scaling;
                sc[c] = s;
                if (s > mx) mx = s;
            }
            softmax_pv_row(sc, nctx, mx, vrows, hd, output + ((int64_t)t * hq + h) * hd);
            free(vrows);
        }
    }
}

void oracle_paged_ragged(const float* q, const float* key_cache, const float* value_cache,
                         int32_t layer_idx, int32_t total_blocks, int32_t block_size,
                         int32_t num_kv_heads, int32_t num_query_heads, int32_t head_dim,
                         int32_t num_seqs, const int32_t* block_tables, int32_t block_table_stride,
                         const int32_t* start_positions, const int32_t* new_token_counts,
                         float scaling, float* out) {
    const int64_t row = (int64_t)num_kv_heads * head_dim;
    const int64_t per_layer = (int64_t)total_blocks * block_size * row;
    const float* lk = key_cache + (int64_t)layer_idx * per_layer;
    const float* lv = value_cache + (int64_t)layer_idx * per_layer;
    const int32_t group = num_query_heads / num_kv_heads;

    int64_t* first_token = (int64_t*)malloc(sizeof(int64_t) * (size_t)(num_seqs + 1));
    first_token[0] = 0;                       /* cu_seqlens, app/model/paged_attention.py:121-125 */
    for (int32_t s = 0; s < num_seqs; ++s) first_token[s + 1] = first_token[s] + new_token_counts[s];

    int32_t max_ctx = 1;
    for (int32_t s = 0; s < num_seqs; ++s)
        if (start_positions[s] + new_token_counts[s] > max_ctx)
            max_ctx = start_positions[s] + new_token_counts[s];
    const int64_t num_tokens = first_token[num_seqs];

    /* One task per new token (not per sequence), so a batch of a few long chunks still spreads
     * over every core; each row's arithmetic and its order are unchanged. */
#pragma omp parallel
    {
        float* sc = (float*)malloc(sizeof(float) * (size_t)max_ctx * (size_t)group);
        const float** vr = (const float**)malloc(sizeof(float*) * (size_t)max_ctx);
        float* kt = (float*)malloc(sizeof(float) * 8 * (size_t)head_dim);
        float* acc = (float*)malloc(sizeof(float) * (size_t)head_dim);
#pragma omp for schedule(dynamic, 4)
        for (int64_t tok = 0; tok < num_tokens; ++tok) {
            int32_t lo = 0, hi = num_seqs; /* sequence of this token: first_token[s] <= tok */
            while (hi - lo > 1) {
                const int32_t mid = (lo + hi) / 2;
                if (first_token[mid] <= tok) lo = mid; else hi = mid;
            }
            const int32_t s = lo;
            const int32_t* bt = block_tables + (int64_t)s * block_table_stride;
            /* causal window [0, pos], paged_attention.py:108-115 */
            const int32_t pos = start_positions[s] + (int32_t)(tok - first_token[s]);
            const int32_t n = pos + 1;
            for (int32_t g = 0; g < num_kv_heads; ++g) {
                const int64_t koff = (int64_t)g * head_dim;
                /* scores of the group's query heads: sc[hh * max_ctx + p] */
                int32_t p = 0;
                for (; p + 8 <= n; p += 8) {
                    for (int32_t j = 0; j < 8; ++j) {
                        /* slot = block*BS + offset, manager.py:320-333 */
                        const int32_t pj = p + j;
                        const int64_t slot = (int64_t)bt[pj / block_size] * block_size + pj % block_size;
                        const float* kr = lk + slot * row + koff;
                        for (int32_t d = 0; d < head_dim; ++d) kt[d * 8 + j] = kr[d];
                    }
                    for (int32_t hh = 0; hh < group; ++hh) {
                        const float* qrow = q + (tok * num_query_heads + g * group + hh) * head_dim;
                        float d8[8];
                        dot_rows8(qrow, kt, head_dim, d8);
                        for (int32_t j = 0; j < 8; ++j) sc[(int64_t)hh * max_ctx + p + j] = d8[j] * scaling;
                    }
                }
                for (; p < n; ++p) {
                    const int64_t slot = (int64_t)bt[p / block_size] * block_size + p % block_size;
                    for (int32_t hh = 0; hh < group; ++hh) {
                        const float* qrow = q + (tok * num_query_heads + g * group + hh) * head_dim;
                        sc[(int64_t)hh * max_ctx + p] = dot_row(qrow, lk + slot * row + koff, head_dim) * scaling;
                    }
                }
                for (int32_t c = 0; c < n; ++c) {
                    const int64_t slot = (int64_t)bt[c / block_size] * block_size + c % block_size;
                    vr[c] = lv + slot * row + koff;
                }
                for (int32_t hh = 0; hh < group; ++hh) {
                    float* srow = sc + (int64_t)hh * max_ctx;
                    float mx = -INFINITY;
                    for (int32_t c = 0; c < n; ++c)
                        if (srow[c] > mx) mx = srow[c];
                    /* Masked columns (c > pos) contribute exact zeros in the reference's PV loop,
                     * so the window [0, pos] gives bit-identical rows. */
                    softmax_pv_row_by_key(srow, n, mx, vr, head_dim, acc,
                                          out + (tok * num_query_heads + g * group + hh) * head_dim);
                }
            }
        }
        free(sc);
        free(vr);
        free(kt);
        free(acc);
    }
    free(first_token);
}

int64_t oracle_reshape_and_cache(const void* key, const void* value, void* key_cache,
                                 void* value_cache, int32_t layer_idx, int64_t slots_per_layer,
                                 int64_t row_bytes, const int64_t* slot_mapping,
                                 int64_t num_tokens) {
    int64_t bad = 0;
    char* kc = (char*)key_cache + (int64_t)layer_idx * slots_per_layer * row_bytes;
    char* vc = (char*)value_cache + (int64_t)layer_idx * slots_per_layer * row_bytes;
    for (int64_t t = 0; t < num_tokens; ++t) {
        const int64_t slot = slot_mapping[t];
        if (slot < 0 || slot >= slots_per_layer) { ++bad; continue; }
        memcpy(kc + slot * row_bytes, (const char*)key + t * row_bytes, (size_t)row_bytes);
        memcpy(vc + slot * row_bytes, (const char*)value + t * row_bytes, (size_t)row_bytes);
    }
    return bad;
}

struct OracleFifo {
    int32_t total;
    int32_t* queue;      /* ring of capacity `total` */
    int64_t front;       /* index of the next block to hand out */
    int64_t size;        /* number of queued (free) blocks */
    int32_t* refcount;
};

OracleFifo* oracle_fifo_create(int32_t total_blocks) {
    OracleFifo* f = (OracleFifo*)calloc(1, sizeof(OracleFifo));
    f->total = total_blocks;
    f->queue = (int32_t*)malloc(sizeof(int32_t) * (size_t)(total_blocks > 0 ? total_blocks : 1));
    f->refcount = (int32_t*)calloc((size_t)(total_blocks > 0 ? total_blocks : 1), sizeof(int32_t));
    for (int32_t i = 0; i < total_blocks; ++i) f->queue[i] = i;   /* page_allocator.hpp:78-81 */
    f->front = 0;
    f->size = total_blocks;
    return f;
}

void oracle_fifo_destroy(OracleFifo* f) {
    if (!f) return;
    free(f->queue);
    free(f->refcount);
    free(f);
}

int32_t oracle_fifo_allocate(OracleFifo* f, int32_t count, int32_t* out_ids) {
    if (count < 0 || f->size < count) return -1;                  /* :114-116 */
    for (int32_t i = 0; i < count; ++i) {                         /* :119-125 */
        const int32_t id = f->queue[f->front % f->total];
        f->front = (f->front + 1) % f->total;
        f->size -= 1;
        f->refcount[id] = 1;
        out_ids[i] = id;
    }
    return 0;
}

int32_t oracle_fifo_free(OracleFifo* f, int32_t block_id) {
    if (block_id < 0 || block_id >= f->total) return -3;          /* validate_block_id :353-357 */
    if (f->refcount[block_id] <= 0) return -2;                    /* :169-171 */
    f->refcount[block_id] -= 1;                                   /* :173-176 */
    if (f->refcount[block_id] == 0) {
        f->queue[(f->front + f->size) % f->total] = block_id;
        f->size += 1;
    }
    return 0;
}

int32_t oracle_fifo_share(OracleFifo* f, int32_t block_id) {
    if (block_id < 0 || block_id >= f->total) return -3;
    if (f->refcount[block_id] <= 0) return -2;                    /* :145-147 */
    f->refcount[block_id] += 1;
    return 0;
}

int32_t oracle_fifo_num_free(const OracleFifo* f) { return (int32_t)f->size; }

int32_t oracle_fifo_snapshot(const OracleFifo* f, int32_t* out) {
    for (int64_t i = 0; i < f->size; ++i) out[i] = f->queue[(f->front + i) % f->total];
    return (int32_t)f->size;
}
