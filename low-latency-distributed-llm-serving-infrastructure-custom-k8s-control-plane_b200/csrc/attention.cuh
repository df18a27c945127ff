// Internal interface between the attention kernels (attention.cu) and the C ABI (api.cu).
#pragma once

#include "common.cuh"

namespace b200 {

constexpr int kDecodeWarps = 4;
constexpr int kDecodeThreads = 32 * kDecodeWarps;
constexpr int kDecodeStages = 3;  // TMA ring depth per warp (2 CTAs per SM fit)

// Shared-memory tile of one 16-token unit: K then V, each D/64 sub-buffers of 16 rows x 128 B
// (128B-swizzled, as TMA writes them).
template <int D>
struct TcTile {
  static constexpr int kSub = D / 64;
  static constexpr int kHalf = 16 * D * 2;  // bytes of the K (or V) tile
  static constexpr int kStage = 2 * kHalf;
};

struct DecodeHeader {
  int32_t total_items;
  int32_t next_item;
  int32_t total_splits;
  int32_t pad;
};

struct PlanArgs {
  const int32_t* ctx_lens;
  const int32_t* query_rows;
  const int64_t* cu_q;  // mixed batch: only sequences with exactly one new token are decoded
  int32_t S;
  int32_t max_ctx;
  int32_t split_tokens;
  int32_t items_per_split;
  int32_t hq;
  int32_t head_dim;
  int32_t esize;
  int64_t o_srow, o_shead;
  void* out;
  int32_t* status;
  DecodeHeader* hdr;
  int32_t* cu_splits;
  int2* work_sp;
  int32_t* counters;
};

struct DecodeArgs {
  const void* q;
  int64_t q_srow, q_shead;
  const int32_t* query_rows;
  const int64_t* cu_q;  // mixed batch: the query row of sequence s is cu_q[s]
  int32_t layer, nb, bs, hkv, hq, group, nchunks, hpc;
  const int32_t* bt;
  int32_t bt_stride;
  const int32_t* ctx_lens;
  int32_t S;
  int32_t max_ctx;
  int32_t split_tokens;
  float scale_log2;
  void* out;
  int64_t o_srow, o_shead;
  int32_t* status;
  DecodeHeader* hdr;
  const int32_t* cu_splits;
  const int2* work_sp;
  int32_t* counters;
  float* part_lse;
  float* part_o;
};

enum RowMode : int32_t { kRowBlockTable = 0, kRowMask = 1 };

struct RowArgs {
  int32_t mode;
  const void* q;
  int64_t q_srow, q_shead;
  const int32_t* query_rows;
  const void* kc;
  const void* vc;
  int32_t layer, nb, bs, hkv, head_dim, group, nchunks;
  // block-table mode
  const int32_t* bt;
  int32_t bt_stride;
  const int32_t* ctx_lens;
  const int64_t* cu_q;  // NULL: one row per sequence (decode)
  int32_t S;
  // mask mode
  const int32_t* gather;
  const uint8_t* mask;
  int32_t num_ctx;
  float scale;
  void* out;
  int64_t o_srow, o_shead;
  int32_t* status;
};

constexpr int kPrefillThreads = 384;

struct PrefillHeader {
  int32_t total_items;
  int32_t pad[3];
};

struct PrefillPlanArgs {
  const int64_t* cu_q;
  // context lengths: when given, the work list is ordered by decreasing cost (KV tiles per
  // item), so that the kernels' snake traversal hands every CTA a near-equal share
  const int32_t* ctx_lens;
  int32_t skip_single;  // sequences with one new token go to the decode kernel instead
  int32_t S;
  int32_t tq;
  int32_t hkv;
  int32_t max_work;
  int32_t* status;
  PrefillHeader* hdr;
  int2* work;
};

struct PrefillArgs {
  int32_t layer, nb, bs, hkv, hq, group, tq;
  const int32_t* bt;
  int32_t bt_stride;
  const int64_t* cu_q;
  const int32_t* ctx_lens;
  int32_t S;
  float scale_log2;
  void* out;
  int64_t o_stok, o_shead;
  int32_t vec_out;
  int32_t* status;
  const PrefillHeader* hdr;
  const int2* work;
};

cudaError_t launch_prefill_plan(const PrefillPlanArgs& a, cudaStream_t stream);

// Work item of CTA blockIdx.x in traversal round `round` of a persistent prefill kernel: rounds
// alternate direction over the CTAs (snake order), so with the work list sorted by decreasing
// cost the CTA that got the largest item of one round gets the smallest of the next.
__device__ __forceinline__ int snake_item(int round) {
  const int g = static_cast<int>(gridDim.x);
  return round * g + ((round & 1) ? (g - 1 - static_cast<int>(blockIdx.x))
                                  : static_cast<int>(blockIdx.x));
}
cudaError_t launch_prefill_tc(int dtype, int head_dim, const CUtensorMap& qm,
                              const CUtensorMap& km, const CUtensorMap& vm, const PrefillArgs& a,
                              int max_items, int num_sms, cudaStream_t stream);

// Two query tiles per work item, one per softmax warpgroup (prefill_q2.cu); the plan counts
// items in pairs of tiles.
// poly_mode: share of the softmax exponentials computed on the FMA pipe instead of the SFU
// (0 = none, 1 = one pair in four, 2 = one pair in two).
cudaError_t launch_prefill_q2(int dtype, int head_dim, const CUtensorMap& qm,
                              const CUtensorMap& km, const CUtensorMap& vm, const PrefillArgs& a,
                              int max_items, int num_sms, int poly_mode, cudaStream_t stream);

// Two independent work streams per CTA (prefill_ds.cu), items of one query tile each.
cudaError_t launch_prefill_ds(int dtype, int head_dim, const CUtensorMap& qm,
                              const CUtensorMap& km, const CUtensorMap& vm, const PrefillArgs& a,
                              int max_items, int num_sms, int poly_mode, cudaStream_t stream);

cudaError_t launch_plan(const PlanArgs& a, cudaStream_t stream);
cudaError_t launch_decode_tc(int dtype, int head_dim, const CUtensorMap& km, const CUtensorMap& vm,
                             const DecodeArgs& a, int max_items, cudaStream_t stream);
cudaError_t launch_row(int dtype, const RowArgs& a, int rows, cudaStream_t stream);

}  // namespace b200
