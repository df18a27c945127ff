// K2: reshape_and_cache -- scatter the step's new K/V rows into their cache slots.
//
// cache[layer].view(-1, Hkv, D)[slot_mapping[t]] = src[t] for key and value
// (app/memory/manager.py:150-168).  One thread per 16-byte (or narrower, when alignment demands)
// chunk of a (token, kv head) row; consecutive threads take consecutive chunks of the same row,
// so both the strided source rows and the destination slot rows are read and written in full
// coalesced lines.  The op is pure data movement: HBM bound at 2 x bytes moved.
#include "cache_ops.cuh"

namespace b200 {

template <typename V>
__global__ void __launch_bounds__(256) reshape_and_cache_kernel(CacheWriteArgs a) {
  const int64_t chunks_per_head = a.head_bytes / static_cast<int64_t>(sizeof(V));
  const int64_t chunks_per_tok = chunks_per_head * a.hkv;
  const int64_t total = chunks_per_tok * a.num_tokens;
  const int64_t slots = static_cast<int64_t>(a.nb) * a.bs;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / chunks_per_tok;
    const int64_t rem = i - t * chunks_per_tok;
    const int64_t h = rem / chunks_per_head;
    const int64_t cidx = rem - h * chunks_per_head;
    const int64_t slot = a.slots[t];
    if (slot < 0) continue;  // padding
    if (slot >= slots) {
      if (cidx == 0 && h == 0) flag_status(a.status, B200_DEVICE_BAD_SLOT);
      continue;
    }
    const int64_t dst = ((static_cast<int64_t>(a.layer) * slots + slot) * a.hkv + h) * a.head_bytes +
                        cidx * static_cast<int64_t>(sizeof(V));
    const V kv = *reinterpret_cast<const V*>(static_cast<const char*>(a.key) +
                                             t * a.k_stok + h * a.k_shead + cidx * sizeof(V));
    const V vv = *reinterpret_cast<const V*>(static_cast<const char*>(a.value) +
                                             t * a.v_stok + h * a.v_shead + cidx * sizeof(V));
    *reinterpret_cast<V*>(static_cast<char*>(a.kc) + dst) = kv;
    *reinterpret_cast<V*>(static_cast<char*>(a.vc) + dst) = vv;
  }
}

cudaError_t launch_reshape_and_cache(const CacheWriteArgs& a, int vec_bytes, int num_sms,
                                     cudaStream_t stream) {
  if (a.num_tokens <= 0) return cudaSuccess;
  const int64_t total = a.head_bytes / vec_bytes * a.hkv * a.num_tokens;
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = static_cast<int64_t>(num_sms > 0 ? num_sms : 148) * 8;
  if (blocks > cap) blocks = cap;
  const int grid = static_cast<int>(blocks);
  switch (vec_bytes) {
    case 16: reshape_and_cache_kernel<uint4><<<grid, 256, 0, stream>>>(a); break;
    case 8: reshape_and_cache_kernel<uint2><<<grid, 256, 0, stream>>>(a); break;
    case 4: reshape_and_cache_kernel<uint32_t><<<grid, 256, 0, stream>>>(a); break;
    case 2: reshape_and_cache_kernel<uint16_t><<<grid, 256, 0, stream>>>(a); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// K2 with rotary embedding: the QKV projection output of a step goes in, the rotated queries come
// out and the rotated keys and the values land in their cache slots -- in one pass instead of the
// rotary elementwise ops (transformers' apply_rotary_pos_emb, run by the model before the
// attention hook) followed by scatter_layer_kv (app/model/paged_attention.py:150-152,
// app/memory/manager.py:150-168).
//
// Rotate-half rotary on (token, head) rows: with c = cos(pos * inv_freq[i]), s = sin(...) in fp32,
//   y[i] = x[i]*c - x[i+D/2]*s,   y[i+D/2] = x[i+D/2]*c + x[i]*s,
// each product and sum rounded separately, as the unfused elementwise ops round them, so the
// result is bit-identical to that path.  One CTA per token: cos/sin of the token's D/2 angles are
// computed once into shared memory and reused by all its q and k heads.
template <typename T>
__global__ void __launch_bounds__(128) rope_cache_kernel(RopeCacheArgs a) {
  extern __shared__ float cs[];  // cos[0, D/2), sin[D/2, D)
  const int half = a.head_dim / 2;
  const int64_t slots_total = static_cast<int64_t>(a.nb) * a.bs;
  const int rot_rows = a.hq + a.hkv;
  for (int64_t t = blockIdx.x; t < a.num_tokens; t += gridDim.x) {
    __syncthreads();  // the previous token's angles are no longer read
    const float pos = static_cast<float>(a.positions[t]);
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
      const float ang = __fmul_rn(pos, a.inv_freq[i]);
      cs[i] = cosf(ang);
      cs[half + i] = sinf(ang);
    }
    __syncthreads();
    const T* row = static_cast<const T*>(a.qkv) + t * a.qkv_stok;
    const int64_t slot = a.slots[t];
    const bool write_kv = slot >= 0 && slot < slots_total;
    if (slot >= slots_total && threadIdx.x == 0) flag_status(a.status, B200_DEVICE_BAD_SLOT);
    const int64_t cache_row =
        write_kv ? ((static_cast<int64_t>(a.layer) * slots_total + slot) * a.hkv) : 0;
    for (int w = threadIdx.x; w < rot_rows * half; w += blockDim.x) {
      const int r = w / half;
      const int i = w - r * half;
      const T* src = row + static_cast<int64_t>(r) * a.head_dim;
      const float x1 = to_f32<T>(src[i]);
      const float x2 = to_f32<T>(src[i + half]);
      const float c = cs[i], s = cs[half + i];
      const float y1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
      const float y2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
      T* dst;
      if (r < a.hq) {
        dst = static_cast<T*>(a.q_out) + t * a.q_stok + static_cast<int64_t>(r) * a.head_dim;
      } else if (write_kv) {
        dst = static_cast<T*>(a.kc) + (cache_row + (r - a.hq)) * a.head_dim;
      } else {
        continue;
      }
      dst[i] = from_f32<T>(y1);
      dst[i + half] = from_f32<T>(y2);
    }
    if (write_kv) {
      const T* vsrc = row + static_cast<int64_t>(rot_rows) * a.head_dim;
      T* vdst = static_cast<T*>(a.vc) + cache_row * a.head_dim;
      for (int w = threadIdx.x; w < a.hkv * a.head_dim; w += blockDim.x) vdst[w] = vsrc[w];
    }
  }
}

cudaError_t launch_rope_cache(const RopeCacheArgs& a, int dtype, int num_sms, cudaStream_t stream) {
  if (a.num_tokens <= 0) return cudaSuccess;
  int64_t grid = a.num_tokens;
  const int64_t cap = static_cast<int64_t>(num_sms > 0 ? num_sms : 148) * 16;
  if (grid > cap) grid = cap;
  const size_t smem = static_cast<size_t>(a.head_dim) * sizeof(float);
  switch (dtype) {
    case B200_DTYPE_BF16:
      rope_cache_kernel<__nv_bfloat16><<<static_cast<int>(grid), 128, smem, stream>>>(a);
      break;
    case B200_DTYPE_F16:
      rope_cache_kernel<__half><<<static_cast<int>(grid), 128, smem, stream>>>(a);
      break;
    case B200_DTYPE_F32:
      rope_cache_kernel<float><<<static_cast<int>(grid), 128, smem, stream>>>(a);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// K6: whole-block copy between two caches of the same per-block geometry, for swapping blocks out
// to and back from pinned host memory and for copying a shared block before it is written
// (CudaKVCacheStrategy.copy_blocks, app/memory/strategies.py:117-122, which copies block by block
// with one copy_ per block and then synchronises).  Pair i copies block src_blocks[i] of every
// layer of K and V into block dst_blocks[i].  One block of one layer is BS*Hkv*D contiguous
// elements; consecutive threads take consecutive 16-byte (or narrower) chunks of it, so either
// side may be device memory or page-locked host memory mapped into the device address space (the
// copy then streams over the host link).  Ids outside a side's pool set B200_DEVICE_BAD_BLOCK
// and the pair is skipped.
template <typename V>
__global__ void __launch_bounds__(256) copy_blocks_kernel(BlockCopyArgs a) {
  const int64_t chunks = a.block_bytes / static_cast<int64_t>(sizeof(V));
  const int64_t per_pair = chunks * a.layers * a.kv_count;
  const int64_t total = per_pair * a.num_blocks;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t pair = i / per_pair;
    int64_t rem = i - pair * per_pair;
    const int64_t kv = rem / (chunks * a.layers);
    rem -= kv * chunks * a.layers;
    const int64_t layer = rem / chunks;
    const int64_t c = rem - layer * chunks;
    const int32_t sb = a.src_blocks[pair];
    const int32_t db = a.dst_blocks[pair];
    if (sb < 0 || sb >= a.src_nb || db < 0 || db >= a.dst_nb) {
      if (rem == 0 && kv == 0) flag_status(a.status, B200_DEVICE_BAD_BLOCK);
      continue;
    }
    const char* src = static_cast<const char*>(kv ? a.src_v : a.src_k) +
                      (layer * a.src_nb + sb) * a.block_bytes;
    char* dst = static_cast<char*>(kv ? a.dst_v : a.dst_k) + (layer * a.dst_nb + db) * a.block_bytes;
    reinterpret_cast<V*>(dst)[c] = reinterpret_cast<const V*>(src)[c];
  }
}

cudaError_t launch_copy_blocks(const BlockCopyArgs& a, int vec_bytes, int num_sms,
                               cudaStream_t stream) {
  if (a.num_blocks <= 0) return cudaSuccess;
  const int64_t total = a.block_bytes / vec_bytes * a.layers * a.kv_count * a.num_blocks;
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = static_cast<int64_t>(num_sms > 0 ? num_sms : 148) * 8;
  if (blocks > cap) blocks = cap;
  const int grid = static_cast<int>(blocks);
  switch (vec_bytes) {
    case 16: copy_blocks_kernel<uint4><<<grid, 256, 0, stream>>>(a); break;
    case 8: copy_blocks_kernel<uint2><<<grid, 256, 0, stream>>>(a); break;
    case 4: copy_blocks_kernel<uint32_t><<<grid, 256, 0, stream>>>(a); break;
    case 2: copy_blocks_kernel<uint16_t><<<grid, 256, 0, stream>>>(a); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace b200
