/*
 * b200_paged.h -- C ABI of libb200paged.so, the B200 (sm_100a) paged-attention hot path.
 *
 * Plain pointers and sizes only; no torch or C++ types cross this boundary.  Unless a comment
 * says "host", every pointer is a device pointer of the CUDA device that is current on the
 * calling thread, and `stream` is a cudaStream_t (NULL = legacy default stream).  All work is
 * enqueued on `stream`; no entry point synchronises the device unless it says so.
 *
 * Functions returning int return a B200_* status code; b200_status_string() names it.  Kernels
 * never trap: a bad block id, slot or an expired bounded wait is recorded as a bit in the
 * caller's device status word (B200_DEVICE_*) and the offending access is skipped.
 *
 * Each entry point names the reference (Pakanor/Low-Latency-Distributed-LLM-Serving-
 * Infrastructure-Custom-K8s-Control-Plane) interface it replaces, as file:line.
 */
#ifndef B200_PAGED_H
#define B200_PAGED_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (map onto the reference's C++ exceptions, csrc/src/bindings.cpp) -------- */
#define B200_OK 0
#define B200_ERR_INVALID_ARGUMENT 1 /* std::invalid_argument -> ValueError                   */
#define B200_ERR_OUT_OF_MEMORY 2    /* runtime_error("Out of Memory ...") -> RuntimeError    */
#define B200_ERR_OUT_OF_RANGE 3     /* std::out_of_range -> IndexError                       */
#define B200_ERR_RUNTIME 4          /* other runtime_error (double free, ...) -> RuntimeError */
#define B200_ERR_UNSUPPORTED 5      /* shape / dtype outside what the kernels cover          */
#define B200_ERR_CUDA 6             /* CUDA runtime or launch error                          */

/* ---- device status word bits ---------------------------------------------------------------- */
#define B200_DEVICE_BAD_BLOCK 1   /* block id outside [0, total_blocks)                     */
#define B200_DEVICE_BAD_SLOT 2    /* slot outside [0, total_blocks * block_size)            */
#define B200_DEVICE_TIMEOUT 4     /* a bounded mbarrier wait expired                        */
#define B200_DEVICE_BAD_OP 8      /* block-pool op inconsistent with the pool state         */
#define B200_DEVICE_BAD_STEP 16   /* step metadata: bad sequence slot, negative start/count,
                                     or more tokens than the outputs hold                   */

/* ---- element types --------------------------------------------------------------------------- */
#define B200_DTYPE_F32 0
#define B200_DTYPE_BF16 1
#define B200_DTYPE_F16 2

const char* b200_status_string(int status);
/* Last CUDA error text seen by the library on this thread (for B200_ERR_CUDA). */
const char* b200_last_error(void);

/* ============================================================================================
 * 1. Drop-in for the reference C ABI of the paged-attention kernel
 * ==========================================================================================*/

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
} PagedAttentionDims;

/* Replaces paged_attention, csrc/include/paged_kernels.h:22-34 (CPU body
 * csrc/src/paged_kernels.cpp:7-105), same signature and meaning: query [Hq][Nq][D], caches
 * [L][NB][BS][Hkv][D], gather_slots [Nctx], attention_mask [Nq][Nctx] (u8, nonzero = attend),
 * output [Nq][Hq][D], all fp32 -- but device pointers, and `stream` is the cudaStream_t the
 * work is enqueued on.  `scratch` is accepted for signature compatibility and not used.
 * Like the reference it returns nothing; b200_last_error() reports a failed launch. */
void paged_attention(const float* query, const float* key_cache, const float* value_cache,
                     const int32_t layer_idx, const PagedAttentionDims dims,
                     const int32_t* gather_slots, const uint8_t* attention_mask,
                     const float scaling, float* output, float* scratch, void* stream);

/* The same operation with a status code and a device status word (may be NULL). */
int b200_paged_attention(const float* query, const float* key_cache, const float* value_cache,
                         int32_t layer_idx, PagedAttentionDims dims, const int32_t* gather_slots,
                         const uint8_t* attention_mask, float scaling, float* output,
                         int32_t* status_word, void* stream);

/* ============================================================================================
 * 2. Attention read through block tables (decode: one new token per sequence)
 * ==========================================================================================*/

/* KV cache geometry: key and value caches are each (L, NB, BS, Hkv, D), contiguous, of
 * `dtype` -- the layout of app/memory/strategies.py:82-86 and :110-115. */
typedef struct {
  int32_t num_layers;
  int32_t total_blocks;
  int32_t block_size;
  int32_t num_kv_heads;
  int32_t head_dim;
  int32_t dtype; /* B200_DTYPE_* */
} B200CacheGeometry;

typedef struct {
  const void* query;      /* one row per sequence: [row][Hq][D] with the strides below     */
  int64_t q_stride_row;   /* elements between query rows                                   */
  int64_t q_stride_head;  /* elements between heads of a row (D contiguous)                */
  const int32_t* query_rows; /* (S,) row of each sequence's query/output; NULL = row s;   */
                             /* each entry must be a row of both query and out          */
  const void* key_cache;
  const void* value_cache;
  B200CacheGeometry geom;
  int32_t layer_idx;
  int32_t num_query_heads;
  const int32_t* block_tables; /* (S, block_table_stride) int32, -1 padded (manager.py:236-271) */
  int32_t block_table_stride;
  const int32_t* context_lens; /* (S,) int32: tokens to attend, including the new one      */
  int32_t num_seqs;
  int32_t max_context_len;     /* host upper bound of context_lens (sizes the split plan)   */
  float scale;
  void* out;                   /* [row][Hq][D] of geom.dtype, strides below                 */
  int64_t o_stride_row;
  int64_t o_stride_head;
  int32_t* status_word;        /* device int32 or NULL                                     */
} B200DecodeParams;

/* Bytes of device workspace b200_paged_decode needs for these parameters. */
size_t b200_paged_decode_workspace_bytes(const B200DecodeParams* p);

/* Replaces the decode leg of the reference: NativePagedBackend.attend
 * (app/model/attention_backends.py:88-117) and the inline SDPA over gathered slots
 * (app/model/paged_attention.py:165-180) for steps where every sequence adds one token.
 * Split-K over the context with a last-CTA merge; bf16/f16 caches on tensor cores, fp32 on
 * CUDA cores.  `workspace` must hold b200_paged_decode_workspace_bytes(p) bytes. */
int b200_paged_decode(const B200DecodeParams* p, void* workspace, size_t workspace_bytes,
                      void* stream);

/* No counterpart in the reference.  The same decode as b200_paged_decode, for callers that cannot
 * allocate device memory at decode time (a server that gave nearly all free HBM to its KV block
 * pool, a plain C caller with no device allocator, a loop that must not pay for cudaMalloc and its
 * synchronisation): the scratch comes from a static device array of
 * B200_DECODE_STATIC_SCRATCH_BYTES that every GPU loading this library holds until exit.  Batches
 * needing more scratch than that (b200_paged_decode_workspace_bytes) are rejected with
 * B200_ERR_INVALID_ARGUMENT.  The first call in a device's CUDA context looks up the array's
 * device address (make it before any stream capture); after a cudaDeviceReset the next call looks
 * it up again in the new context.  Calls share the array: each call resets what must start at
 * zero, and calls that overlap on the GPU race.  Allocates nothing. */
#define B200_DECODE_STATIC_SCRATCH_BYTES ((size_t)64 << 20)
int b200_paged_decode_static(const B200DecodeParams* p, void* stream);

/* Split size of the decode plan, in tokens (rounded up to a multiple of 16); 0 restores the
 * built-in rule: 2048 tokens, halved (down to 512) while the batch would give fewer
 * (sequence, split, KV head) work items than half the SMs. */
void b200_set_decode_split_tokens(int32_t tokens);

/* ============================================================================================
 * 2b. Ragged causal attention through block tables (prefill chunks, mixed steps)
 * ==========================================================================================*/

typedef struct {
  const void* query;      /* [token][Hq][D] with the strides below                           */
  int64_t q_stride_token;
  int64_t q_stride_head;
  const void* key_cache;
  const void* value_cache;
  B200CacheGeometry geom;
  int32_t layer_idx;
  int32_t num_query_heads;
  const int32_t* block_tables; /* (S, block_table_stride) int32                             */
  int32_t block_table_stride;
  const int64_t* cu_seqlens;   /* (S+1): tokens of sequence s are rows [cu[s], cu[s+1])     */
  const int32_t* context_lens; /* (S,): context incl. this step's tokens; token i of s sits at
                                  position context_lens[s] - count_s + i and attends [0, pos] */
  int32_t num_seqs;
  int32_t num_tokens;
  int32_t max_query_len;       /* host upper bounds                                         */
  int32_t max_context_len;
  float scale;
  void* out;                   /* [token][Hq][D] of geom.dtype                              */
  int64_t o_stride_token;
  int64_t o_stride_head;
  int32_t* status_word;
} B200PrefillParams;

size_t b200_paged_prefill_workspace_bytes(const B200PrefillParams* p);

/* Replaces the prefill / mixed-step leg of the reference: the SDPA over the gathered context with
 * the block-diagonal causal mask, app/model/paged_attention.py:92-118 and :165-180 (and
 * TorchSdpBackend.attend, app/model/attention_backends.py:55-78).  Every new token of every
 * sequence attends causally to its sequence's cached prefix and to the earlier new tokens, read
 * through the block table after b200_reshape_and_cache has written them. */
int b200_paged_prefill(const B200PrefillParams* p, void* workspace, size_t workspace_bytes,
                       void* stream);

/* Nonzero: run b200_paged_prefill on the CUDA-core kernel even where the tcgen05 kernel applies
 * (for A/B comparison); 0 restores the default. */
void b200_set_prefill_cuda_cores(int32_t enable);

/* Which tensor-core prefill kernel b200_paged_prefill runs (results agree within the bf16
 * tolerance; a tuning and comparison knob):
 *   0 = one query tile per work item, the K/V tiles alternating between the two softmax
 *       warpgroups;
 *   1 = two query tiles per work item, one per softmax warpgroup, each K/V tile staged once for
 *       both (the default);
 *   2 = two independent work streams per CTA, each with its own query tile, K/V rings, MMA warp
 *       and softmax warpgroup, so one stream's item transitions overlap the other's work. */
void b200_set_prefill_kernel(int32_t kernel);

/* Share of the two-tile prefill's softmax exponentials computed by a cubic on the FMA pipe
 * instead of the SFU's ex2 (relative error below 7.5e-5 either way, far under bf16's): 0 = none,
 * 1 = one pair of keys in four (the default), 2 = one pair in two.  A tuning knob. */
void b200_set_prefill_poly_exp(int32_t mode);

/* ============================================================================================
 * 3. KV-cache slot write (reshape_and_cache)
 * ==========================================================================================*/

/* Replaces PagedKVCacheManager.scatter_layer_kv, app/memory/manager.py:150-168:
 *   key_cache[layer].view(-1, Hkv, D)[slot_mapping[t]] = key[t]   (same for value).
 * key/value rows may be strided views ([t][h][d] with the given element strides, d contiguous),
 * e.g. the (1,Hkv,Ntok,D) -> (Ntok,Hkv,D) transpose of paged_attention.py:152-153.
 * Slots < 0 are padding and skipped; slots >= NB*BS set B200_DEVICE_BAD_SLOT and are skipped. */
int b200_reshape_and_cache(const void* key, int64_t k_stride_token, int64_t k_stride_head,
                           const void* value, int64_t v_stride_token, int64_t v_stride_head,
                           void* key_cache, void* value_cache, const B200CacheGeometry* geom,
                           int32_t layer_idx, const int64_t* slot_mapping, int32_t num_tokens,
                           int32_t* status_word, void* stream);

/* Rotary embedding fused into the slot write.  Replaces the rotary step the model runs before
 * the attention hook (transformers' apply_rotary_pos_emb, rotate-half form) together with
 * scatter_layer_kv (app/model/paged_attention.py:150-152, app/memory/manager.py:150-168).
 * qkv: (num_tokens, qkv_stride_token) rows laid out [q heads | k heads | v heads], each head
 * head_dim contiguous elements of the cache dtype (the fused QKV projection output).
 * positions: int64 per token; inv_freq: fp32 (head_dim/2,) rotary frequencies.
 * Writes rotated q to q_out (num_tokens, num_query_heads, head_dim) with the given token stride,
 * rotated k and unchanged v to the cache slots (slots < 0 skipped, >= NB*BS flag
 * B200_DEVICE_BAD_SLOT).  Angles, cos/sin and the rotation are computed in fp32 with every
 * product and sum rounded separately, bit-identical to the unfused elementwise path. */
int b200_rope_reshape_and_cache(const void* qkv, int64_t qkv_stride_token, int32_t num_tokens,
                                int32_t num_query_heads, const int64_t* positions,
                                const float* inv_freq, void* q_out, int64_t q_out_stride_token,
                                void* key_cache, void* value_cache, const B200CacheGeometry* geom,
                                int32_t layer_idx, const int64_t* slot_mapping,
                                int32_t* status_word, void* stream);

/* Whole-block copy between two KV caches with the same layers, block size, heads, head_dim and
 * dtype (their block counts may differ).  Replaces CudaKVCacheStrategy.copy_blocks
 * (app/memory/strategies.py:117-122): pair i copies block src_blocks[i] of every layer of the
 * source K and V caches into block dst_blocks[i] of the destination.  Either cache may be
 * device memory or page-locked host memory (cudaHostAlloc / torch pin_memory, which the device
 * addresses directly), so the same call moves blocks out to a host swap space, back in, or
 * between device blocks (a copy before writing a shared block).  The two value caches may both
 * be NULL to copy the key caches only (a single-cache copy).  The id arrays must be readable by
 * the device; pageable host memory anywhere is rejected with B200_ERR_INVALID_ARGUMENT.  Pairs
 * run in parallel: within one call no block may be both a destination and a source.  Ids
 * outside a side's pool flag B200_DEVICE_BAD_BLOCK and that pair is skipped.  The bookkeeping of
 * which block went where stays with the allocator (PageAllocator::swap_out / swap_in /
 * share_block, page_allocator.hpp:142-241). */
int b200_copy_blocks(const void* src_key_cache, const void* src_value_cache,
                     const B200CacheGeometry* src_geom, void* dst_key_cache,
                     void* dst_value_cache, const B200CacheGeometry* dst_geom,
                     const int32_t* src_blocks, const int32_t* dst_blocks, int32_t num_blocks,
                     int32_t* status_word, void* stream);

/* ============================================================================================
 * 4. Device block pool (FIFO free list + per-sequence block tables resident on the GPU)
 * ==========================================================================================*/

/* Replaces the GPU-block bookkeeping of PageAllocator / SequenceBlockTable
 * (csrc/include/page_allocator.hpp:78-177, :426-469) for the engine's batched path: the free
 * list is a device ring in the reference's FIFO order, tables are device rows indexed by a
 * sequence slot.  The host side of the handle keeps only counts, so scheduling decisions
 * (free-block checks, scheduler.py:104,130) need no device round trip.  Ops are queued on the
 * host and applied in order by one kernel per b200_pool_flush. */
typedef struct B200BlockPool B200BlockPool;

/* Allocates the pool's device arrays on the current device (cudaMalloc). */
int b200_pool_create(int32_t total_blocks, int32_t block_size, int32_t max_seqs,
                     int32_t max_blocks_per_seq, B200BlockPool** out);
int b200_pool_destroy(B200BlockPool* pool);
/* Queue: append n tokens to sequence slot `slot`, allocating a block whenever its token count
 * crosses a multiple of block_size (SequenceBlockTable::append_token, :426-434).  If the pool
 * runs dry the tokens that fit are appended and B200_ERR_OUT_OF_MEMORY is returned, as the
 * reference's token-by-token loop leaves them (manager.py:86-93). */
int b200_pool_append_tokens(B200BlockPool* pool, int32_t slot, int32_t n);
/* Queue: free the slot's blocks in table order and reset it (release_internal, :461-469). */
int b200_pool_release(B200BlockPool* pool, int32_t slot);
/* Prefix sharing.  The empty slot dst_slot takes the first num_blocks blocks of src_slot, each
 * gaining an owner (PageAllocator::share_block + SequenceBlockTable::append_block,
 * page_allocator.hpp:142-149, :409-413); dst_slot then counts num_blocks * block_size tokens.
 * A shared block returns to the free list only when its last owner releases it.  Flushes of
 * batches that involve shared blocks apply their ops in order on one thread and read the exact
 * free count back (one stream synchronisation). */
int b200_pool_share(B200BlockPool* pool, int32_t dst_slot, int32_t src_slot, int32_t num_blocks);
/* Copy-on-write: table entry block_index of the slot gets a fresh block from the front of the free
 * list and the old block loses an owner (allocate_block + SequenceBlockTable::replace_block +
 * free_block, page_allocator.hpp:100-127, :416-424, :151-177).  After the flush,
 * b200_pool_cow_pairs gives the (old, new) block ids of every replacement of that flush as two
 * device arrays, ready for b200_copy_blocks (so the copy needs no host round trip); they hold
 * that flush's pairs until the next b200_pool_flush, which may also reallocate them, so enqueue
 * the copy before flushing again.  Replace only blocks that have another owner: a sole owner's
 * old block would be freed in the same flush. */
int b200_pool_copy_on_write(B200BlockPool* pool, int32_t slot, int32_t block_index);
int32_t b200_pool_cow_pairs(const B200BlockPool* pool, const int32_t** old_blocks,
                            const int32_t** new_blocks);

/* Apply the queued ops on `stream` (one small H2D copy + one kernel).  No host sync, except for
 * batches that involve shared blocks (see b200_pool_share). */
int b200_pool_flush(B200BlockPool* pool, void* stream);
/* Host-side counts (exact; no device access). */
int32_t b200_pool_num_free_blocks(const B200BlockPool* pool);
int32_t b200_pool_tokens(const B200BlockPool* pool, int32_t slot);
int32_t b200_pool_num_blocks(const B200BlockPool* pool, int32_t slot);
/* Device views: tables (max_seqs, max_blocks_per_seq) int32 (-1 = empty), ring (NB) int32,
 * device status word. */
const int32_t* b200_pool_tables(const B200BlockPool* pool);
int32_t b200_pool_table_stride(const B200BlockPool* pool);
const int32_t* b200_pool_ring(const B200BlockPool* pool);
int32_t* b200_pool_status(const B200BlockPool* pool);
/* Host copy of the free queue front-to-back (synchronises `stream`); returns its length. */
int32_t b200_pool_snapshot_free(B200BlockPool* pool, int32_t* host_out, int32_t capacity,
                                void* stream);

/* ============================================================================================
 * 5. Per-step ragged metadata built on the device
 * ==========================================================================================*/

/* Replaces PagedStepContext (app/model/paged_attention.py:40-90, :121-135) with
 * build_slot_mapping (app/memory/manager.py:104-128, :301-333) and build_block_tables
 * (:236-271).  Inputs are device arrays of S entries: the pool slot of each sequence, the
 * position of its first new token and its new-token count; the sequence's tokens must already
 * be appended in the pool.  Outputs (device, caller-allocated):
 *   cu_seqlens (S+1) int64, cu_context (S+1) int64, context_lens (S) int32,
 *   position_ids (num_tokens) int64, slot_mapping (num_tokens) int64,
 *   block_tables (S, bt_stride) int32 padded with -1,
 *   gather_slots (num_context_tokens) int64 or NULL (only the masked-form kernel needs it).
 * Every write stays inside these sizes: a sequence slot outside the pool, a negative start or
 * count (the sequence then counts as empty), or counts whose sum overruns num_tokens /
 * num_context_tokens set B200_DEVICE_BAD_STEP and the entries that do not fit are skipped.
 * Warp/block prefix sums; two launches. */
int b200_build_step_metadata(const B200BlockPool* pool, const int32_t* seq_slots,
                             const int32_t* start_positions, const int32_t* new_token_counts,
                             int32_t num_seqs, int32_t num_tokens, int64_t* cu_seqlens,
                             int64_t* cu_context, int32_t* context_lens, int64_t* position_ids,
                             int64_t* slot_mapping, int32_t* block_tables, int32_t bt_stride,
                             int64_t* gather_slots, int64_t num_context_tokens, void* stream);

/* ============================================================================================
 * 6. Host mirror of the reference allocator API (PageAllocator / SequenceBlockTable)
 * ==========================================================================================*/

/* Host C++ re-implementation of llm_allocator_cpp.PageAllocator (page_allocator.hpp:45-374)
 * with identical FIFO / refcount / swap-bookkeeping semantics and error mapping; used by the
 * drop-in Python module of the same name.  Errors return B200_ERR_* and leave a message for
 * b200_host_last_message(). */
typedef struct B200HostAllocator B200HostAllocator;
int b200_host_allocator_create(int64_t total_blocks, int64_t tokens_per_block,
                               int64_t bytes_per_token, int64_t total_cpu_blocks,
                               B200HostAllocator** out);
void b200_host_allocator_destroy(B200HostAllocator* a);
int b200_host_allocate_block(B200HostAllocator* a, int32_t* out_id);
int b200_host_allocate_blocks(B200HostAllocator* a, int64_t count, int32_t* out_ids);
int b200_host_share_block(B200HostAllocator* a, int32_t block_id);
int b200_host_free_block(B200HostAllocator* a, int32_t block_id);
int b200_host_swap_out(B200HostAllocator* a, int32_t gpu_block_id, int32_t* out_cpu_block);
int b200_host_swap_in(B200HostAllocator* a, int32_t cpu_block_id, int32_t* out_gpu_block);
int b200_host_get_cpu_block_id(B200HostAllocator* a, int32_t gpu_block_id, int32_t* out);
int b200_host_release_swapped_block(B200HostAllocator* a, int32_t cpu_block_id);
int b200_host_get_host_ptr(B200HostAllocator* a, int32_t cpu_block_id, uint64_t* out);
/* Deprecated in the reference (page_allocator.hpp:291-302): the host pool base, 0 without one. */
int b200_host_get_device_ptr(B200HostAllocator* a, int32_t gpu_block_id, uint64_t* out);
int64_t b200_host_num_free_blocks(const B200HostAllocator* a);
int64_t b200_host_num_free_cpu_blocks(const B200HostAllocator* a);
int64_t b200_host_total_blocks(const B200HostAllocator* a);
int64_t b200_host_block_size(const B200HostAllocator* a);
int64_t b200_host_bytes_per_token(const B200HostAllocator* a);
int64_t b200_host_pool_bytes(const B200HostAllocator* a);
double b200_host_utilization(const B200HostAllocator* a);
const char* b200_host_last_message(void);

#ifdef __cplusplus
}
#endif

#endif /* B200_PAGED_H */
