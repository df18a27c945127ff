// Host side of the device block pool (K5) and the step-metadata entry point (K4).
//
// The host keeps only integers: the free-block count and, per sequence slot, its token and block
// counts.  That is all the scheduler's decisions need (scheduler.py:100-104, :128-130); the block
// ids themselves live on the device.  Ops are queued here and applied in order by
// pool_apply_kernel at flush time.
#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "cache_ops.cuh"
#include "nvtx.cuh"

namespace {
int pfail(int code, const char* msg) {
  b200::set_last_error(msg);
  return code;
}
}  // namespace

struct B200BlockPool {
  int32_t total_blocks = 0, block_size = 0, max_seqs = 0, max_blocks = 0;
  int32_t* d_ring = nullptr;
  int32_t* d_refcount = nullptr;
  int32_t* d_tables = nullptr;
  int32_t* d_nblocks = nullptr;
  int64_t* d_head_tail = nullptr;
  int32_t* d_status = nullptr;
  b200::PoolOp* d_ops = nullptr;
  int32_t ops_cap = 0;
  bool initialised = false;
  int64_t free_count = 0;
  std::vector<int32_t> tokens, nblocks;
  std::vector<uint8_t> shared;    // slot holds (or held out) blocks with more than one owner
  std::vector<b200::PoolOp> queue;
  bool ordered = false;           // queue holds SHARE / REPLACE or a release of a shared slot
  int32_t pending_replace = 0;    // REPLACE ops in the queue
  int32_t* d_cow = nullptr;       // [cow_cap] old blocks, then [cow_cap] new blocks
  int32_t cow_cap = 0;
  int32_t cow_count = 0;          // pairs recorded by the last flush
};

namespace {

int ensure_ops_capacity(B200BlockPool* p, int32_t n) {
  if (n <= p->ops_cap) return B200_OK;
  int32_t cap = p->ops_cap > 0 ? p->ops_cap : 256;
  while (cap < n) cap *= 2;
  if (p->d_ops) cudaFree(p->d_ops);  // cudaFree waits for kernels still reading the old buffer
  p->d_ops = nullptr;
  if (cudaMalloc(&p->d_ops, cap * sizeof(b200::PoolOp)) != cudaSuccess)
    return pfail(B200_ERR_CUDA, "pool op buffer allocation failed");
  p->ops_cap = cap;
  return B200_OK;
}

int flush_segment(B200BlockPool* p, const b200::PoolOp* ops, int32_t n, cudaStream_t st) {
  if (n <= 0) return B200_OK;
  int rc = ensure_ops_capacity(p, n);
  if (rc != B200_OK) return rc;
  // Pageable source: the runtime stages it before returning, so the host queue can be reused at
  // once; the device buffer is reused in stream order (this copy runs after the previous apply).
  if (cudaMemcpyAsync(p->d_ops, ops, n * sizeof(b200::PoolOp), cudaMemcpyHostToDevice, st) !=
      cudaSuccess)
    return pfail(B200_ERR_CUDA, "pool op upload failed");
  b200::PoolApplyArgs a{};
  a.ops = p->d_ops;
  a.num_ops = n;
  a.nb = p->total_blocks;
  a.table_stride = p->max_blocks;
  a.ring = p->d_ring;
  a.tables = p->d_tables;
  a.nblocks = p->d_nblocks;
  a.refcount = p->d_refcount;
  a.head_tail = p->d_head_tail;
  a.status = p->d_status;
  if (b200::launch_pool_apply(a, st) != cudaSuccess)
    return pfail(B200_ERR_CUDA, "pool apply launch failed");
  return B200_OK;
}

// Ordered path: the whole queue by the one-thread kernel, then the exact free count read back
// (a shared block is freed only with its last owner, which the host cannot see).
int flush_ordered(B200BlockPool* p, cudaStream_t st) {
  const int32_t n = static_cast<int32_t>(p->queue.size());
  int rc = ensure_ops_capacity(p, n);
  if (rc != B200_OK) return rc;
  if (p->pending_replace > p->cow_cap) {
    int32_t cap = p->cow_cap > 0 ? p->cow_cap : 64;
    while (cap < p->pending_replace) cap *= 2;
    if (p->d_cow) cudaFree(p->d_cow);
    p->d_cow = nullptr;
    p->cow_cap = 0;
    if (cudaMalloc(&p->d_cow, 2 * static_cast<size_t>(cap) * sizeof(int32_t)) != cudaSuccess)
      return pfail(B200_ERR_CUDA, "copy-on-write pair buffer allocation failed");
    p->cow_cap = cap;
  }
  if (cudaMemcpyAsync(p->d_ops, p->queue.data(), n * sizeof(b200::PoolOp),
                      cudaMemcpyHostToDevice, st) != cudaSuccess)
    return pfail(B200_ERR_CUDA, "pool op upload failed");
  b200::PoolApplyArgs a{};
  a.ops = p->d_ops;
  a.num_ops = n;
  a.nb = p->total_blocks;
  a.table_stride = p->max_blocks;
  a.ring = p->d_ring;
  a.tables = p->d_tables;
  a.nblocks = p->d_nblocks;
  a.refcount = p->d_refcount;
  a.head_tail = p->d_head_tail;
  a.status = p->d_status;
  if (b200::launch_pool_apply_ordered(a, p->d_cow, p->d_cow + p->cow_cap, st) != cudaSuccess)
    return pfail(B200_ERR_CUDA, "pool apply launch failed");
  int64_t ht[2];
  if (cudaMemcpyAsync(ht, p->d_head_tail, sizeof(ht), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return pfail(B200_ERR_CUDA, "pool free-count read-back failed");
  p->free_count = ht[1] - ht[0];
  p->cow_count = p->pending_replace;
  return B200_OK;
}

}  // namespace

extern "C" {

int b200_pool_create(int32_t total_blocks, int32_t block_size, int32_t max_seqs,
                     int32_t max_blocks_per_seq, B200BlockPool** out) {
  if (out == nullptr) return pfail(B200_ERR_INVALID_ARGUMENT, "null out");
  *out = nullptr;
  if (block_size <= 0) return pfail(B200_ERR_INVALID_ARGUMENT, "tokens_per_block must be greater than 0");
  if (total_blocks <= 0 || max_seqs <= 0 || max_blocks_per_seq <= 0)
    return pfail(B200_ERR_INVALID_ARGUMENT, "pool sizes must be positive");
  auto* p = new B200BlockPool();
  p->total_blocks = total_blocks;
  p->block_size = block_size;
  p->max_seqs = max_seqs;
  p->max_blocks = max_blocks_per_seq;
  p->free_count = total_blocks;
  p->tokens.assign(max_seqs, 0);
  p->nblocks.assign(max_seqs, 0);
  p->shared.assign(max_seqs, 0);
  const int64_t table_elems = static_cast<int64_t>(max_seqs) * max_blocks_per_seq;
  bool ok = cudaMalloc(&p->d_ring, total_blocks * sizeof(int32_t)) == cudaSuccess &&
            cudaMalloc(&p->d_refcount, total_blocks * sizeof(int32_t)) == cudaSuccess &&
            cudaMalloc(&p->d_tables, table_elems * sizeof(int32_t)) == cudaSuccess &&
            cudaMalloc(&p->d_nblocks, max_seqs * sizeof(int32_t)) == cudaSuccess &&
            cudaMalloc(&p->d_head_tail, 2 * sizeof(int64_t)) == cudaSuccess &&
            cudaMalloc(&p->d_status, sizeof(int32_t)) == cudaSuccess;
  if (!ok) {
    b200_pool_destroy(p);
    return pfail(B200_ERR_CUDA, "pool device allocation failed");
  }
  cudaMemset(p->d_status, 0, sizeof(int32_t));
  if (b200::launch_pool_init(p->d_ring, p->d_refcount, p->d_tables, p->d_nblocks, p->d_head_tail,
                             total_blocks, table_elems, max_seqs, nullptr) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess) {
    b200_pool_destroy(p);
    return pfail(B200_ERR_CUDA, "pool init failed");
  }
  *out = p;
  return B200_OK;
}

int b200_pool_destroy(B200BlockPool* p) {
  if (p == nullptr) return B200_OK;
  cudaFree(p->d_ring);
  cudaFree(p->d_refcount);
  cudaFree(p->d_tables);
  cudaFree(p->d_nblocks);
  cudaFree(p->d_head_tail);
  cudaFree(p->d_status);
  if (p->d_ops) cudaFree(p->d_ops);
  if (p->d_cow) cudaFree(p->d_cow);
  delete p;
  return B200_OK;
}

int b200_pool_append_tokens(B200BlockPool* p, int32_t slot, int32_t n) {
  if (p == nullptr) return pfail(B200_ERR_INVALID_ARGUMENT, "null pool");
  if (slot < 0 || slot >= p->max_seqs) return pfail(B200_ERR_OUT_OF_RANGE, "sequence slot out of range");
  if (n < 0) return pfail(B200_ERR_INVALID_ARGUMENT, "negative token count");
  if (n == 0) return B200_OK;
  const int64_t T = p->tokens[slot];
  const int64_t have = p->nblocks[slot];
  const int64_t bs = p->block_size;
  // blocks needed = number of multiples of bs in [T, T+n) (append_token allocates at T % bs == 0)
  int64_t need = (T + n + bs - 1) / bs - (T + bs - 1) / bs;
  int64_t fit = n;
  int rc = B200_OK;
  if (need > p->free_count) {
    // the tokens that fit into owned + free blocks, then the reference's loop throws
    fit = (have + p->free_count) * bs - T;
    if (fit < 0) fit = 0;
    need = (T + fit + bs - 1) / bs - (T + bs - 1) / bs;
    rc = pfail(B200_ERR_OUT_OF_MEMORY, "Out of Memory: No free VRAM pages available in KV-Cache pool!");
  }
  if (have + need > p->max_blocks)
    return pfail(B200_ERR_INVALID_ARGUMENT, "sequence exceeds max_blocks_per_seq");
  if (need > 0)
    p->queue.push_back(b200::PoolOp{0, slot, static_cast<int32_t>(have), static_cast<int32_t>(need)});
  p->tokens[slot] = static_cast<int32_t>(T + fit);
  p->nblocks[slot] = static_cast<int32_t>(have + need);
  p->free_count -= need;
  return rc;
}

int b200_pool_release(B200BlockPool* p, int32_t slot) {
  if (p == nullptr) return pfail(B200_ERR_INVALID_ARGUMENT, "null pool");
  if (slot < 0 || slot >= p->max_seqs) return pfail(B200_ERR_OUT_OF_RANGE, "sequence slot out of range");
  const int32_t nb = p->nblocks[slot];
  if (nb > 0) p->queue.push_back(b200::PoolOp{1, slot, 0, nb});
  if (p->shared[slot]) {
    // some of these blocks have other owners: how many come free is known after the flush
    if (nb > 0) p->ordered = true;
    p->shared[slot] = 0;
  } else {
    p->free_count += nb;
  }
  p->tokens[slot] = 0;
  p->nblocks[slot] = 0;
  return B200_OK;
}

int b200_pool_share(B200BlockPool* p, int32_t dst_slot, int32_t src_slot, int32_t num_blocks) {
  if (p == nullptr) return pfail(B200_ERR_INVALID_ARGUMENT, "null pool");
  if (dst_slot < 0 || dst_slot >= p->max_seqs || src_slot < 0 || src_slot >= p->max_seqs)
    return pfail(B200_ERR_OUT_OF_RANGE, "sequence slot out of range");
  if (dst_slot == src_slot) return pfail(B200_ERR_INVALID_ARGUMENT, "a slot cannot share with itself");
  if (p->nblocks[dst_slot] != 0)
    return pfail(B200_ERR_INVALID_ARGUMENT, "the receiving slot must be empty");
  if (num_blocks <= 0 || num_blocks > p->nblocks[src_slot])
    return pfail(B200_ERR_INVALID_ARGUMENT, "num_blocks must be in [1, blocks of the source slot]");
  p->queue.push_back(b200::PoolOp{2, dst_slot, src_slot, num_blocks});
  p->nblocks[dst_slot] = num_blocks;
  p->tokens[dst_slot] = num_blocks * p->block_size;
  p->shared[dst_slot] = p->shared[src_slot] = 1;
  p->ordered = true;
  return B200_OK;
}

int b200_pool_copy_on_write(B200BlockPool* p, int32_t slot, int32_t block_index) {
  if (p == nullptr) return pfail(B200_ERR_INVALID_ARGUMENT, "null pool");
  if (slot < 0 || slot >= p->max_seqs) return pfail(B200_ERR_OUT_OF_RANGE, "sequence slot out of range");
  if (block_index < 0 || block_index >= p->nblocks[slot])
    return pfail(B200_ERR_OUT_OF_RANGE, "block index out of range");
  if (p->free_count < 1)
    return pfail(B200_ERR_OUT_OF_MEMORY, "Out of Memory: No free VRAM pages available in KV-Cache pool!");
  p->queue.push_back(b200::PoolOp{3, slot, block_index, 1});
  p->free_count -= 1;
  ++p->pending_replace;
  p->ordered = true;
  return B200_OK;
}

int32_t b200_pool_cow_pairs(const B200BlockPool* p, const int32_t** old_blocks,
                            const int32_t** new_blocks) {
  if (p == nullptr) return 0;
  if (old_blocks) *old_blocks = p->d_cow;
  if (new_blocks) *new_blocks = p->d_cow ? p->d_cow + p->cow_cap : nullptr;
  return p->cow_count;
}

int b200_pool_flush(B200BlockPool* p, void* stream) {
  b200::NvtxRange nvtx_range("b200_pool_flush");
  if (p == nullptr) return pfail(B200_ERR_INVALID_ARGUMENT, "null pool");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  p->cow_count = 0;
  if (p->ordered) {
    const int rc = p->queue.empty() ? B200_OK : flush_ordered(p, st);
    p->queue.clear();
    p->ordered = false;
    p->pending_replace = 0;
    return rc;
  }
  // The apply kernel runs all RELEASEs of a launch before its ALLOCs, so a RELEASE of a slot that
  // an earlier ALLOC of the same launch filled starts a new launch.
  std::vector<uint8_t> allocated(p->max_seqs, 0);
  size_t seg = 0;
  int rc = B200_OK;
  for (size_t i = 0; i < p->queue.size() && rc == B200_OK; ++i) {
    const b200::PoolOp& op = p->queue[i];
    if (op.kind == 1 && allocated[op.slot]) {
      rc = flush_segment(p, p->queue.data() + seg, static_cast<int32_t>(i - seg), st);
      std::fill(allocated.begin(), allocated.end(), 0);
      seg = i;
    }
    if (op.kind == 0) allocated[op.slot] = 1;
  }
  if (rc == B200_OK)
    rc = flush_segment(p, p->queue.data() + seg, static_cast<int32_t>(p->queue.size() - seg), st);
  p->queue.clear();
  return rc;
}

int32_t b200_pool_num_free_blocks(const B200BlockPool* p) {
  return p ? static_cast<int32_t>(p->free_count) : 0;
}
int32_t b200_pool_tokens(const B200BlockPool* p, int32_t slot) {
  return (p && slot >= 0 && slot < p->max_seqs) ? p->tokens[slot] : 0;
}
int32_t b200_pool_num_blocks(const B200BlockPool* p, int32_t slot) {
  return (p && slot >= 0 && slot < p->max_seqs) ? p->nblocks[slot] : 0;
}
const int32_t* b200_pool_tables(const B200BlockPool* p) { return p ? p->d_tables : nullptr; }
int32_t b200_pool_table_stride(const B200BlockPool* p) { return p ? p->max_blocks : 0; }
const int32_t* b200_pool_ring(const B200BlockPool* p) { return p ? p->d_ring : nullptr; }
int32_t* b200_pool_status(const B200BlockPool* p) { return p ? p->d_status : nullptr; }

int32_t b200_pool_snapshot_free(B200BlockPool* p, int32_t* host_out, int32_t capacity,
                                void* stream) {
  if (p == nullptr) return -1;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  int64_t ht[2];
  std::vector<int32_t> ring(p->total_blocks);
  if (cudaMemcpyAsync(ht, p->d_head_tail, sizeof(ht), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaMemcpyAsync(ring.data(), p->d_ring, ring.size() * sizeof(int32_t),
                      cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return -1;
  const int64_t n = ht[1] - ht[0];
  int32_t k = 0;
  for (int64_t i = 0; i < n && k < capacity; ++i)
    host_out[k++] = ring[(ht[0] + i) % p->total_blocks];
  return static_cast<int32_t>(n);
}

int b200_build_step_metadata(const B200BlockPool* pool, const int32_t* seq_slots,
                             const int32_t* start_positions, const int32_t* new_token_counts,
                             int32_t num_seqs, int32_t num_tokens, int64_t* cu_seqlens,
                             int64_t* cu_context, int32_t* context_lens, int64_t* position_ids,
                             int64_t* slot_mapping, int32_t* block_tables, int32_t bt_stride,
                             int64_t* gather_slots, int64_t num_context_tokens, void* stream) {
  b200::NvtxRange nvtx_range("b200_build_step_metadata");
  if (pool == nullptr) return pfail(B200_ERR_INVALID_ARGUMENT, "null pool");
  if (num_seqs < 0 || num_tokens < 0 || bt_stride < 0 || num_context_tokens < 0)
    return pfail(B200_ERR_INVALID_ARGUMENT, "negative sizes");
  b200::MetaArgs a{};
  a.seq_slots = seq_slots;
  a.starts = start_positions;
  a.counts = new_token_counts;
  a.S = num_seqs;
  a.bs = pool->block_size;
  a.pool_tables = pool->d_tables;
  a.pool_nblocks = pool->d_nblocks;
  a.pool_stride = pool->max_blocks;
  a.nb = pool->total_blocks;
  a.cu_seqlens = cu_seqlens;
  a.cu_context = cu_context;
  a.context_lens = context_lens;
  a.position_ids = position_ids;
  a.slot_mapping = slot_mapping;
  a.block_tables = block_tables;
  a.bt_stride = bt_stride;
  a.gather_slots = gather_slots;
  a.status = pool->d_status;
  a.max_seqs = pool->max_seqs;
  a.max_tokens = num_tokens;
  a.max_ctx = gather_slots != nullptr ? num_context_tokens : 0;
  if (b200::launch_step_metadata(a, static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return pfail(B200_ERR_CUDA, "step metadata launch failed");
  return B200_OK;
}

}  // extern "C"
