/*
 * CPU oracle for the paged-attention hot path.  TEST INFRASTRUCTURE ONLY: the test suite, the
 * smoke check and the CPU-baseline leg of bench.py use it as the checker.  The product path
 * never links, loads or calls anything in this directory.
 *
 * Every function restates the arithmetic of the reference (Pakanor/Low-Latency-Distributed-
 * LLM-Serving-Infrastructure-Custom-K8s-Control-Plane) in plain C; the reference file:line each
 * one follows is cited beside it.  Parity of this restatement is pinned two ways:
 *   - bit-exact against the reference's own C++ kernel compiled from its sources (oracle/_ref);
 *   - against the literal values of the reference's unit tests (cu_seqlens, masks, slots,
 *     FIFO block order) and the golden fixtures in tests/golden/.
 */
#ifndef PAGED_ORACLE_H
#define PAGED_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same field order as PagedAttentionDims, csrc/include/paged_kernels.h:11-20. */
typedef struct {
    int32_t num_query_heads;
    int32_t num_query_tokens;
    int32_t head_dim;
    int32_t num_layers;
    int32_t total_blocks;
    int32_t block_size;
    int32_t num_kv_heads;
    int32_t num_context_tokens;
} OraclePagedDims;

/* Masked attention over a flat gather-slot list, restating csrc/src/paged_kernels.cpp:7-105.
 * query [Hq][Nq][D], caches [L][NB][BS][Hkv][D], gather_slots [Nctx], mask [Nq][Nctx] (u8),
 * output [Nq][Hq][D], scratch [Nq][Hq][Nctx].  fp32, sequential accumulation per (q, h_q). */
void oracle_paged_attention(const float* query, const float* key_cache, const float* value_cache,
                            int32_t layer_idx, OraclePagedDims dims, const int32_t* gather_slots,
                            const uint8_t* attention_mask, float scaling, float* output,
                            float* scratch);

/* Ragged causal attention read through block tables.  For sequence s the query tokens are rows
 * [cu_q[s], cu_q[s]+count[s]) of q, at positions start[s]+i, and the context is positions
 * [0, start[s]+count[s]) whose slots are block_tables[s][p/BS]*BS + p%BS.  This is what the
 * reference computes when PagedStepContext (app/model/paged_attention.py:40-118) feeds its gather
 * slots and block-diagonal causal mask to the kernel above; each (token, head) row is
 * bit-identical to that call.  Decode is the case count[s] == 1.
 * q [Ntok][Hq][D], out [Ntok][Hq][D]. */
void oracle_paged_ragged(const float* q, const float* key_cache, const float* value_cache,
                         int32_t layer_idx, int32_t total_blocks, int32_t block_size,
                         int32_t num_kv_heads, int32_t num_query_heads, int32_t head_dim,
                         int32_t num_seqs, const int32_t* block_tables, int32_t block_table_stride,
                         const int32_t* start_positions, const int32_t* new_token_counts,
                         float scaling, float* out);

/* reshape_and_cache: cache[layer].view(-1, Hkv, D)[slot] = src, restating
 * app/memory/manager.py:150-168 (index_put).  Rows are copied as raw bytes of
 * row_bytes = Hkv*D*elem_size; src rows are contiguous.  Returns the number of slots that were
 * out of range [0, NB*BS) (those rows are not written). */
int64_t oracle_reshape_and_cache(const void* key, const void* value, void* key_cache,
                                 void* value_cache, int32_t layer_idx, int64_t slots_per_layer,
                                 int64_t row_bytes, const int64_t* slot_mapping,
                                 int64_t num_tokens);

/* FIFO block pool with reference counts, restating PageAllocator's GPU-block bookkeeping in
 * csrc/include/page_allocator.hpp:78-81 (initial queue 0..N-1), :100-110 (allocate_block pops
 * the front, ref_count = 1), :112-127 (allocate_blocks: all-or-nothing), :142-149 (share_block),
 * :151-177 (free_block: decrement, push to the back at zero). */
typedef struct OracleFifo OracleFifo;
OracleFifo* oracle_fifo_create(int32_t total_blocks);
void        oracle_fifo_destroy(OracleFifo* f);
/* 0 = ok; -1 = out of memory (nothing allocated). */
int32_t     oracle_fifo_allocate(OracleFifo* f, int32_t count, int32_t* out_ids);
/* 0 = ok; -2 = double free / unallocated; -3 = block id out of range. */
int32_t     oracle_fifo_free(OracleFifo* f, int32_t block_id);
/* 0 = ok; -2 = share of an unallocated block; -3 = block id out of range. */
int32_t     oracle_fifo_share(OracleFifo* f, int32_t block_id);
int32_t     oracle_fifo_num_free(const OracleFifo* f);
/* Copies the free queue front-to-back into out (capacity >= total); returns its length. */
int32_t     oracle_fifo_snapshot(const OracleFifo* f, int32_t* out);

#ifdef __cplusplus
}
#endif

#endif /* PAGED_ORACLE_H */
