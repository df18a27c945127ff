// K5: device block pool, and K4: per-step ragged metadata.
//
// The pool keeps the reference's FIFO free list (csrc/include/page_allocator.hpp:78-81 initial
// order, :100-127 pop from the front, :173-176 push freed blocks to the back) as a ring in device
// memory, plus one block-table row per sequence slot.  A batch of queued ops is applied by one
// single-CTA kernel: frees first (each RELEASE appends its blocks at tail + exclusive prefix of the
// freed counts), then allocations (each ALLOC takes ring[head + exclusive prefix of the allocated
// counts]).  Because the host only queues an ALLOC when its running free count covers it, every
// ring position an ALLOC reads was written by a RELEASE that precedes it in queue order, so the
// two-phase kernel hands out exactly the blocks the reference's sequential loop would.  Batches
// that involve shared blocks go through an ordered one-thread kernel instead.
//
// The metadata kernels build what PagedStepContext (app/model/paged_attention.py:40-90) and
// build_block_tables (app/memory/manager.py:236-271) build on the host: cu_seqlens, cu_context,
// context_lens, position_ids, slot_mapping, padded block tables and (optionally) gather slots.
#include <mutex>
#include <vector>

#include "cache_ops.cuh"

namespace b200 {

// ============================================================================================
// Kernels
// ============================================================================================

__global__ void pool_init_kernel(int32_t* ring, int32_t* refcount, int32_t* tables,
                                 int32_t* nblocks, int64_t* head_tail, int32_t nb,
                                 int64_t table_elems, int32_t max_seqs) {
  const int64_t i0 = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = i0; i < nb; i += stride) {
    ring[i] = static_cast<int32_t>(i);
    refcount[i] = 0;
  }
  for (int64_t i = i0; i < table_elems; i += stride) tables[i] = -1;
  for (int64_t i = i0; i < max_seqs; i += stride) nblocks[i] = 0;
  if (i0 == 0) {
    head_tail[0] = 0;
    head_tail[1] = nb;  // all blocks queued
  }
}

__global__ void __launch_bounds__(1024) pool_apply_kernel(PoolApplyArgs a) {
  __shared__ int64_t warp_buf[32];
  __shared__ int64_t tot;
  const int tid = threadIdx.x;
  const int64_t head = a.head_tail[0];
  const int64_t tail = a.head_tail[1];

  // Phase 1: releases, in queue order, appended at the tail.
  int64_t carry = 0;
  for (int base = 0; base < a.num_ops; base += 1024) {
    const int i = base + tid;
    const int64_t n = (i < a.num_ops && a.ops[i].kind == 1) ? a.ops[i].count : 0;
    const int64_t excl = block_exclusive_scan_1024(n, warp_buf, &tot) + carry;
    __syncthreads();
    const int64_t chunk_total = tot;
    __syncthreads();
    // Each thread applies its own op; ops of one batch touch disjoint ring positions and rows.
    if (i < a.num_ops && n > 0) {
      const PoolOp op = a.ops[i];
      int32_t* row = a.tables + static_cast<int64_t>(op.slot) * a.table_stride;
      for (int32_t j = 0; j < op.count; ++j) {
        const int32_t b = row[j];
        if (b < 0 || b >= a.nb) {
          flag_status(a.status, B200_DEVICE_BAD_OP);
          continue;
        }
        if (a.refcount[b] != 1) flag_status(a.status, B200_DEVICE_BAD_OP);
        a.refcount[b] = 0;
        a.ring[(tail + excl + j) % a.nb] = b;
        row[j] = -1;
      }
      a.nblocks[op.slot] = 0;
    }
    carry += chunk_total;
    __syncthreads();
  }
  const int64_t freed = carry;
  __syncthreads();

  // Phase 2: allocations, in queue order, taken from the head.
  carry = 0;
  for (int base = 0; base < a.num_ops; base += 1024) {
    const int i = base + tid;
    const int64_t n = (i < a.num_ops && a.ops[i].kind == 0) ? a.ops[i].count : 0;
    const int64_t excl = block_exclusive_scan_1024(n, warp_buf, &tot) + carry;
    __syncthreads();
    const int64_t chunk_total = tot;
    __syncthreads();
    if (i < a.num_ops && n > 0) {
      const PoolOp op = a.ops[i];
      int32_t* row = a.tables + static_cast<int64_t>(op.slot) * a.table_stride;
      for (int32_t j = 0; j < op.count; ++j) {
        const int32_t b = a.ring[(head + excl + j) % a.nb];
        a.refcount[b] = 1;
        if (op.first + j < a.table_stride) row[op.first + j] = b;
        else flag_status(a.status, B200_DEVICE_BAD_OP);
      }
      atomicMax(&a.nblocks[op.slot], op.first + op.count);
    }
    carry += chunk_total;
    __syncthreads();
  }
  if (tid == 0) {
    a.head_tail[0] = head + carry;
    a.head_tail[1] = tail + freed;
  }
}

// Ordered apply, for batches with shared blocks (SHARE / REPLACE ops, or releases of sequences that
// hold shared blocks): a block goes back to the free list only when its last owner lets it go
// (PageAllocator::free_block, page_allocator.hpp:151-177), so where freed blocks land depends on
// every earlier op; one thread applies the batch in queue order, exactly as the reference's
// sequential calls would (share_block :142-149, replace_block :416-424, allocate_block
// :100-127).  Sharing is rare; the parallel kernel above serves everything else.
__global__ void pool_apply_ordered_kernel(PoolApplyArgs a, int32_t* cow_src, int32_t* cow_dst) {
  if (blockIdx.x != 0 || threadIdx.x != 0) return;
  int64_t head = a.head_tail[0];
  int64_t tail = a.head_tail[1];
  int32_t k = 0;
  auto valid = [&](int32_t b) { return b >= 0 && b < a.nb; };
  auto release_one = [&](int32_t b) {
    if (!valid(b) || a.refcount[b] <= 0) {
      flag_status(a.status, B200_DEVICE_BAD_OP);
      return;
    }
    if (--a.refcount[b] == 0) a.ring[(tail++) % a.nb] = b;
  };
  for (int i = 0; i < a.num_ops; ++i) {
    const PoolOp op = a.ops[i];
    int32_t* row = a.tables + static_cast<int64_t>(op.slot) * a.table_stride;
    if (op.kind == 0) {
      for (int32_t j = 0; j < op.count; ++j) {
        if (head >= tail || op.first + j >= a.table_stride) {
          flag_status(a.status, B200_DEVICE_BAD_OP);
          break;
        }
        const int32_t b = a.ring[(head++) % a.nb];
        a.refcount[b] = 1;
        row[op.first + j] = b;
      }
      if (a.nblocks[op.slot] < op.first + op.count) a.nblocks[op.slot] = op.first + op.count;
    } else if (op.kind == 1) {
      for (int32_t j = 0; j < op.count; ++j) {
        release_one(row[j]);
        row[j] = -1;
      }
      a.nblocks[op.slot] = 0;
    } else if (op.kind == 2) {
      const int32_t* src = a.tables + static_cast<int64_t>(op.first) * a.table_stride;
      for (int32_t j = 0; j < op.count; ++j) {
        const int32_t b = src[j];
        if (!valid(b) || a.refcount[b] <= 0) {
          flag_status(a.status, B200_DEVICE_BAD_OP);
          row[j] = -1;
          continue;
        }
        ++a.refcount[b];
        row[j] = b;
      }
      a.nblocks[op.slot] = op.count;
    } else if (op.kind == 3) {
      const int32_t old = row[op.first];
      if (head >= tail || !valid(old)) {
        flag_status(a.status, B200_DEVICE_BAD_OP);
        cow_src[k] = cow_dst[k] = -1;  // the copy kernel skips (and flags) this pair
        ++k;
        continue;
      }
      const int32_t b = a.ring[(head++) % a.nb];
      a.refcount[b] = 1;
      row[op.first] = b;
      release_one(old);
      cow_src[k] = old;
      cow_dst[k] = b;
      ++k;
    } else {
      flag_status(a.status, B200_DEVICE_BAD_OP);
    }
  }
  a.head_tail[0] = head;
  a.head_tail[1] = tail;
}

// K4 part 1: scans (one CTA).
__global__ void __launch_bounds__(1024) meta_scan_kernel(MetaArgs a) {
  __shared__ int64_t warp_buf[32];
  __shared__ int64_t tot;
  int64_t cq = 0, cc = 0;
  for (int base = 0; base < a.S; base += 1024) {
    const int s = base + threadIdx.x;
    int64_t n = 0, ctx = 0;
    if (s < a.S) {
      n = a.counts[s];
      ctx = static_cast<int64_t>(a.starts[s]) + n;
      if (n < 0 || ctx < n) {  // negative count or start: the sequence counts as empty
        flag_status(a.status, B200_DEVICE_BAD_STEP);
        n = ctx = 0;
      }
      a.context_lens[s] = static_cast<int32_t>(ctx);
    }
    const int64_t eq = block_exclusive_scan_1024(n, warp_buf, &tot) + cq;
    __syncthreads();
    const int64_t tq = tot;
    __syncthreads();
    const int64_t ec = block_exclusive_scan_1024(ctx, warp_buf, &tot) + cc;
    __syncthreads();
    const int64_t tc = tot;
    __syncthreads();
    if (s < a.S) {
      a.cu_seqlens[s] = eq;
      a.cu_context[s] = ec;
    }
    cq += tq;
    cc += tc;
  }
  if (threadIdx.x == 0) {
    a.cu_seqlens[a.S] = cq;
    a.cu_context[a.S] = cc;
  }
}

// K4 part 2: per-sequence fill (one CTA per sequence).  Every write is bounded by its output's
// size; what does not fit, or names a slot outside the pool, is flagged and skipped.
__global__ void __launch_bounds__(256) meta_fill_kernel(MetaArgs a) {
  const int s = blockIdx.x;
  const int32_t slot = a.seq_slots[s];
  int32_t start = a.starts[s], count = a.counts[s];
  if (count < 0 || start < 0) start = count = 0;  // flagged by the scan
  const int64_t q0 = a.cu_seqlens[s];
  const bool slot_ok = slot >= 0 && slot < a.max_seqs;
  if (!slot_ok && threadIdx.x == 0) flag_status(a.status, B200_DEVICE_BAD_STEP);
  const int32_t* trow = a.pool_tables + (slot_ok ? static_cast<int64_t>(slot) * a.pool_stride : 0);
  const int32_t owned = slot_ok ? min(a.pool_nblocks[slot], a.pool_stride) : 0;
  for (int i = threadIdx.x; i < a.bt_stride; i += blockDim.x)
    a.block_tables[static_cast<int64_t>(s) * a.bt_stride + i] = i < owned ? trow[i] : -1;
  if (q0 < 0 || q0 + count > a.max_tokens) {
    if (threadIdx.x == 0) flag_status(a.status, B200_DEVICE_BAD_STEP);
  } else {
    for (int i = threadIdx.x; i < count; i += blockDim.x) {
      const int32_t pos = start + i;
      a.position_ids[q0 + i] = pos;
      const int32_t bi = pos / a.bs;
      const int32_t b = bi < owned ? trow[bi] : -1;
      if (b < 0 || b >= a.nb) {
        flag_status(a.status, B200_DEVICE_BAD_BLOCK);
        a.slot_mapping[q0 + i] = -1;
      } else {
        a.slot_mapping[q0 + i] = static_cast<int64_t>(b) * a.bs + pos % a.bs;
      }
    }
  }
  if (a.gather_slots != nullptr) {
    const int64_t c0 = a.cu_context[s];
    const int32_t ctx = start + count;
    if (c0 < 0 || c0 + ctx > a.max_ctx) {
      if (threadIdx.x == 0) flag_status(a.status, B200_DEVICE_BAD_STEP);
      return;
    }
    for (int p = threadIdx.x; p < ctx; p += blockDim.x) {
      const int32_t bi = p / a.bs;
      const int32_t b = bi < owned ? trow[bi] : -1;
      a.gather_slots[c0 + p] = (b < 0 || b >= a.nb) ? -1 : static_cast<int64_t>(b) * a.bs + p % a.bs;
    }
  }
}

cudaError_t launch_pool_init(int32_t* ring, int32_t* refcount, int32_t* tables, int32_t* nblocks,
                             int64_t* head_tail, int32_t nb, int64_t table_elems, int32_t max_seqs,
                             cudaStream_t stream) {
  pool_init_kernel<<<256, 256, 0, stream>>>(ring, refcount, tables, nblocks, head_tail, nb,
                                            table_elems, max_seqs);
  return cudaGetLastError();
}

cudaError_t launch_pool_apply(const PoolApplyArgs& a, cudaStream_t stream) {
  if (a.num_ops <= 0) return cudaSuccess;
  pool_apply_kernel<<<1, 1024, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_pool_apply_ordered(const PoolApplyArgs& a, int32_t* cow_src, int32_t* cow_dst,
                                      cudaStream_t stream) {
  if (a.num_ops <= 0) return cudaSuccess;
  pool_apply_ordered_kernel<<<1, 32, 0, stream>>>(a, cow_src, cow_dst);
  return cudaGetLastError();
}

cudaError_t launch_step_metadata(const MetaArgs& a, cudaStream_t stream) {
  if (a.S <= 0) return cudaSuccess;
  meta_scan_kernel<<<1, 1024, 0, stream>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  meta_fill_kernel<<<a.S, 256, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace b200
