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

}  // namespace b200
