// Internal interface of the cache-write (K2), block-pool (K5) and step-metadata (K4) kernels.
#pragma once

#include "common.cuh"

namespace b200 {

struct CacheWriteArgs {
  const void* key;
  const void* value;
  int64_t k_stok, k_shead, v_stok, v_shead;  // bytes
  void* kc;
  void* vc;
  int32_t layer, nb, bs, hkv;
  int64_t head_bytes;  // D * element size
  const int64_t* slots;
  int32_t num_tokens;
  int32_t* status;
};

cudaError_t launch_reshape_and_cache(const CacheWriteArgs& a, int vec_bytes, int num_sms,
                                     cudaStream_t stream);

struct RopeCacheArgs {
  const void* qkv;           // (tokens, (hq + 2*hkv) * D): q heads, then k heads, then v heads
  int64_t qkv_stok;          // elements
  int32_t hq, hkv, head_dim;
  const int64_t* positions;  // (tokens,)
  const float* inv_freq;     // (D/2,)
  void* q_out;               // (tokens, hq, D), heads contiguous
  int64_t q_stok;            // elements
  void* kc;
  void* vc;
  int32_t layer, nb, bs;
  const int64_t* slots;
  int32_t num_tokens;
  int32_t* status;
};

cudaError_t launch_rope_cache(const RopeCacheArgs& a, int dtype, int num_sms, cudaStream_t stream);

struct BlockCopyArgs {
  const void* src_k;
  const void* src_v;
  void* dst_k;
  void* dst_v;
  int32_t layers;
  int32_t kv_count;             // 2: K and V; 1: K only (single-cache copy)
  int32_t src_nb, dst_nb;       // blocks per layer of each side
  int64_t block_bytes;          // BS * Hkv * D * element size
  const int32_t* src_blocks;
  const int32_t* dst_blocks;
  int32_t num_blocks;
  int32_t* status;
};

cudaError_t launch_copy_blocks(const BlockCopyArgs& a, int vec_bytes, int num_sms,
                               cudaStream_t stream);

// One queued block-pool op, uploaded as 4 int32.
//   kind 0 = ALLOC:   append `count` blocks to slot's table starting at table index `first`
//   kind 1 = RELEASE: free the slot's first `count` blocks in table order, clear the row
//   kind 2 = SHARE:   the (empty) slot takes the first `count` blocks of slot `first`, each
//                     block's owner count + 1
//   kind 3 = REPLACE: table entry `first` of the slot gets a fresh block (copy-on-write); the old
//                     block loses an owner and is freed if that was the last one
struct PoolOp {
  int32_t kind, slot, first, count;
};

struct PoolApplyArgs {
  const PoolOp* ops;
  int32_t num_ops;
  int32_t nb;
  int32_t table_stride;
  int32_t* ring;
  int32_t* tables;
  int32_t* nblocks;
  int32_t* refcount;
  int64_t* head_tail;  // [0] = head (next block to hand out), [1] = tail (next free position)
  int32_t* status;
};

cudaError_t launch_pool_apply(const PoolApplyArgs& a, cudaStream_t stream);
// All four kinds, strictly in queue order (one thread); REPLACE k records its (old, new) block
// pair in cow_src[k] / cow_dst[k].
cudaError_t launch_pool_apply_ordered(const PoolApplyArgs& a, int32_t* cow_src, int32_t* cow_dst,
                                      cudaStream_t stream);
cudaError_t launch_pool_init(int32_t* ring, int32_t* refcount, int32_t* tables, int32_t* nblocks,
                             int64_t* head_tail, int32_t nb, int64_t table_elems, int32_t max_seqs,
                             cudaStream_t stream);

struct MetaArgs {
  const int32_t* seq_slots;
  const int32_t* starts;
  const int32_t* counts;
  int32_t S;
  int32_t bs;
  const int32_t* pool_tables;
  const int32_t* pool_nblocks;
  int32_t pool_stride;
  int32_t nb;
  int64_t* cu_seqlens;
  int64_t* cu_context;
  int32_t* context_lens;
  int64_t* position_ids;
  int64_t* slot_mapping;
  int32_t* block_tables;
  int32_t bt_stride;
  int64_t* gather_slots;
  int32_t* status;
  int32_t max_seqs;      // pool slots: seq_slots entries must lie in [0, max_seqs)
  int64_t max_tokens;    // entries of position_ids / slot_mapping
  int64_t max_ctx;       // entries of gather_slots
};

cudaError_t launch_step_metadata(const MetaArgs& a, cudaStream_t stream);

// Block-wide exclusive scan over 1024 threads; returns the exclusive prefix of v and writes the
// block total to *total (visible to all threads after the call).
__device__ __forceinline__ int64_t block_exclusive_scan_1024(int64_t v, int64_t* warp_buf,
                                                             int64_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int64_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t t = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += t;
  }
  if (lane == 31) warp_buf[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int64_t w = warp_buf[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t t = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += t;
    }
    warp_buf[lane] = w;
    if (lane == 31) *total = w;
  }
  __syncthreads();
  const int64_t incl = x + (warp > 0 ? warp_buf[warp - 1] : 0);
  __syncthreads();
  return incl - v;
}

}  // namespace b200
