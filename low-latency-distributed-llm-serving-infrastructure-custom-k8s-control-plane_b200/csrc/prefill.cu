// K3: ragged causal attention on the 5th-generation tensor cores (tcgen05, TMEM accumulators).
//
// One work item = (sequence, tile of TQ = 128/G query tokens, KV head).  The 128 query rows of a
// tile are the G query heads sharing the KV head x TQ tokens (row = g*TQ + t), so every K/V tile
// fetched from HBM feeds all G heads.  K/V are read through the block table in 128-key tiles.
//
// Warp roles (384 threads, three warpgroups of one kind each so that registers can be moved
// between them with setmaxnreg: the softmax warpgroups get kRegsSoftmax per thread, the
// producer / MMA warpgroup kRegsOther):
//   warps 0-3,  two softmax warpgroups.  Warpgroup w takes the KV tiles g with g % 2 == w and keeps
//   warps 4-7   its own running max / sum and its own O accumulator, so the two run concurrently
//               without exchanging anything per tile.  One query row per thread (TMEM lane = row):
//               tcgen05.ld of S, causal mask, online softmax in fp32, P packed to bf16/f16 pairs
//               and stored with tcgen05.st over the S columns already consumed, rescale of O in
//               TMEM when the row max moves.  The epilogue merges the two partial (O, max, sum)
//               triples of each row, as a two-way split-KV combine, and writes O / l.
//   warp 8      TMA producer for Q (4-D map over [token][head][dim]) and K tiles (3-D map over the
//               paged cache, one 16-row box per block and 64-column half), kKStages-deep ring.
//   warp 10     TMA producer for V tiles, kVStages-deep ring.  K and V are issued by different
//               threads: a block-paged tile is 8*D/64 small boxes, and one thread issuing both
//               rings could not keep the tensor core fed.
//   warp 9      TMEM owner and MMA issuer (one thread).  S = Q.K^T (M=128, N=128, K=D) into the
//               TMEM S buffer of the warpgroup that owns the tile; O += P.V (M=128, N=D, K=128)
//               with P read straight from TMEM (the A operand of tcgen05.mma in tensor memory)
//               into that warpgroup's O accumulator; tcgen05.commit on mbarriers.
//   warp 11     idle (completes the third warpgroup).
// TMEM (512 columns): S/P of warpgroup w at columns [128w, 128w+128) (P in the upper 64), O of
// warpgroup w at [256 + w*D, 256 + (w+1)*D).  P(g) aliases S(g); S(g+2) is issued right after
// PV(g) (in-order tcgen05.mma execution orders PV(g)'s TMEM reads before S(g+2)'s writes).
// Every mbarrier wait is bounded; an expired wait records B200_DEVICE_TIMEOUT and stops the CTA.
#include <type_traits>

#include "attention.cuh"
#include "tc05.cuh"

namespace b200 {

namespace {

constexpr int kBN = 128;  // keys per KV tile (the N of S = Q.K^T, the K of O += P.V)
// P column group g (32 keys) of a tile holds key chunk kPChunk[g]: the softmax writes the chunks
// still in registers after the row-max pass first (see the softmax warps).
__device__ constexpr uint32_t kPChunk[4] = {2, 3, 0, 1};
// K and V stream through separate rings: a K stage is released as soon as its S = Q.K^T has
// completed, a V stage when its PV has.  K is needed before V, hence the deeper K ring.
constexpr int kKStages = 3;
constexpr int kVStages = 2;
constexpr int kSoftmaxWarps = 8;
// Register split (setmaxnreg): 256 softmax threads x kRegsSoftmax + 128 other threads x
// kRegsOther must not exceed the 384 x (registers per thread at launch) the CTA is given; the
// launcher checks the compiled count before every first launch (a larger request would wait
// forever).
constexpr uint32_t kRegsSoftmax = 176;
constexpr uint32_t kRegsOther = 136;
constexpr int kWarpK = 8, kWarpMma = 9, kWarpV = 10;

struct SmemLayout {
  uint32_t q, k0, v0, bars, xch, total;
};

template <int D>
__host__ __device__ constexpr SmemLayout prefill_layout() {
  constexpr uint32_t SUB = D / 64;
  constexpr uint32_t Q = SUB * 128 * 128;
  constexpr uint32_t KT = SUB * kBN * 128;
  constexpr uint32_t KV = (kKStages + kVStages) * KT;
  // xch: per item parity, softmax warpgroup and row, the (max, sum) pair the epilogue merge
  // exchanges (double-buffered: a warpgroup with no tile in the next item reaches the next
  // exchange while the other may still read this one)
  return SmemLayout{0, Q, Q + kKStages * KT, Q + KV, Q + KV + 512, Q + KV + 512 + 2 * 2 * 128 * 8};
}

enum : int {
  kBarQFull = 0,
  kBarQEmpty,
  kBarKFull,                          // + K stage
  kBarKEmpty = kBarKFull + kKStages,
  kBarVFull = kBarKEmpty + kKStages,  // + V stage
  kBarVEmpty = kBarVFull + kVStages,
  kBarSFull = kBarVEmpty + kVStages,  // + warpgroup
  kBarPFull = kBarSFull + 2,          // + warpgroup
  kBarPvDone = kBarPFull + 2,         // + warpgroup
  kBarOEmpty = kBarPvDone + 2,
  kBarXchg,
  kBarFinal,
  kNumBars
};

// Bounded wait (same time limit as mbar_wait_bounded) that also gives up when another role has
// already aborted the CTA.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t phase, volatile int* abort_flag,
                                              int32_t* status) {
  if (mbar_try_wait(bar, phase)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    for (uint32_t i = 0; i < kWaitTriesPerCheck; ++i) {
      if (mbar_try_wait(bar, phase)) return true;
      if (*abort_flag) return false;
    }
    if (globaltimer_ns() - t0 > kWaitLimitNs) break;
  }
  *abort_flag = 1;
  flag_status(status, B200_DEVICE_TIMEOUT);
  return false;
}

}  // namespace

// Cost bins of the work-list sort: an item's cost is the number of 128-key KV tiles it reads,
// clamped to the last bin (items that long are ordered among themselves arbitrarily).
constexpr int kCostBins = 512;

// (32-bit arithmetic: token counts and positions are below 2^31; kBN is a power of two)
__device__ __forceinline__ int pair_cost(const PrefillPlanArgs& a, int s, int32_t count, int k) {
  const int32_t tb = k * a.tq;
  const int32_t n = count - tb < a.tq ? count - tb : a.tq;
  const int32_t kv_end = a.ctx_lens[s] - count + tb + n;
  const int32_t c = kv_end <= 0 ? 0 : ((kv_end + kBN - 1) >> 7);
  static_assert(kBN == 128, "cost bins assume 128-key tiles");
  return c >= kCostBins ? kCostBins - 1 : c;
}

__global__ void __launch_bounds__(1024) prefill_plan_kernel(PrefillPlanArgs a) {
  __shared__ int32_t warp_sums[32];
  __shared__ int32_t carry_s;
  __shared__ int32_t bins[kCostBins];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool sorted = a.ctx_lens != nullptr;
  if (tid == 0) carry_s = 0;
  for (int b = tid; b < kCostBins; b += 1024) bins[b] = 0;
  __syncthreads();
  const uint32_t tq = static_cast<uint32_t>(a.tq);
  auto count_of = [&](int s) -> int32_t { return static_cast<int32_t>(a.cu_q[s + 1] - a.cu_q[s]); };
  auto items_of = [&](int32_t count) -> int32_t {
    return (count > 0 && !(a.skip_single && count == 1))
               ? static_cast<int32_t>((static_cast<uint32_t>(count) + tq - 1) / tq)
               : 0;
  };
  for (int base = 0; base < a.S; base += 1024) {
    const int s = base + tid;
    const int32_t count = s < a.S ? count_of(s) : 0;
    const int32_t n = items_of(count);
    int32_t v = n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t t = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += t;
    }
    if (lane == 31) warp_sums[warp] = v;
    __syncthreads();
    if (warp == 0) {
      int32_t w = warp_sums[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int32_t t = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += t;
      }
      warp_sums[lane] = w;
    }
    __syncthreads();
    const int32_t incl = v + (warp > 0 ? warp_sums[warp - 1] : 0) + carry_s;
    const int32_t excl = incl - n;
    if (s < a.S) {
      if (sorted) {
        for (int32_t k = 0; k < n; ++k) atomicAdd(&bins[pair_cost(a, s, count, k)], 1);
      } else {
        for (int32_t k = 0; k < n; ++k)
          if (excl + k < a.max_work) a.work[excl + k] = make_int2(s, k);
          else flag_status(a.status, B200_DEVICE_BAD_OP);
      }
    }
    __syncthreads();
    if (tid == 1023) carry_s = incl;
    __syncthreads();
  }
  if (sorted) {
    // start offset of every bin in decreasing-cost order (warp 0: 16 bins per lane, then a scan
    // across the lanes), then each item is placed at its bin's next free position
    if (warp == 0) {
      constexpr int kPer = kCostBins / 32;
      int32_t local[kPer];
      int32_t sum = 0;
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        local[i] = bins[kCostBins - 1 - (lane * kPer + i)];
        sum += local[i];
      }
      int32_t v = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int32_t t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
      }
      int32_t off = v - sum;
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        bins[kCostBins - 1 - (lane * kPer + i)] = off;
        off += local[i];
      }
    }
    __syncthreads();
    for (int s = tid; s < a.S; s += 1024) {
      const int32_t count = count_of(s);
      const int32_t n = items_of(count);
      for (int32_t k = 0; k < n; ++k) {
        const int32_t pos = atomicAdd(&bins[pair_cost(a, s, count, k)], 1);
        if (pos < a.max_work) a.work[pos] = make_int2(s, k);
        else flag_status(a.status, B200_DEVICE_BAD_OP);
      }
    }
  }
  if (tid == 0) {
    const int32_t tiles = carry_s < a.max_work ? carry_s : a.max_work;
    a.hdr->total_items = tiles * a.hkv;
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(kPrefillThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap qmap,
                      const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap, PrefillArgs a) {
  constexpr int SUB = D / 64;
  constexpr int kChunks = kBN / 16;  // 16-row TMA boxes per tile and 64-column half
  constexpr SmemLayout L = prefill_layout<D>();
  constexpr uint32_t KT = SUB * kBN * 128;  // bytes of one K (or V) tile
  constexpr uint32_t QBYTES = SUB * 128 * 128;
  constexpr uint32_t kTmemCols = 512;
  constexpr uint32_t kColO = 256;
  constexpr uint32_t ab_fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  constexpr uint32_t idesc_s = tc05::idesc_f16(ab_fmt, 128, kBN, 0);
  constexpr uint32_t idesc_o = tc05::idesc_f16(ab_fmt, 128, D, 1);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base = (raw_u32 + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_u32);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    mbar_init(&bars[kBarQFull], 1);
    mbar_init(&bars[kBarQEmpty], 1);
    for (int st = 0; st < kKStages; ++st) {
      mbar_init(&bars[kBarKFull + st], 1);
      mbar_init(&bars[kBarKEmpty + st], 1);
    }
    for (int st = 0; st < kVStages; ++st) {
      mbar_init(&bars[kBarVFull + st], 1);
      mbar_init(&bars[kBarVEmpty + st], 1);
    }
    for (int w = 0; w < 2; ++w) {
      mbar_init(&bars[kBarSFull + w], 1);
      mbar_init(&bars[kBarPFull + w], 4);  // one arrival per warp of the warpgroup
      mbar_init(&bars[kBarPvDone + w], 1);
    }
    mbar_init(&bars[kBarOEmpty], kSoftmaxWarps);
    mbar_init(&bars[kBarXchg], kSoftmaxWarps);
    mbar_init(&bars[kBarFinal], 1);
    *abort_flag = 0;
    fence_proxy_async_smem();
  }
  if (warp == kWarpMma) {
    tc05::tmem_alloc(tmem_slot, kTmemCols);
    tc05::tmem_relinquish();
  }
  tc05::fence_before_sync();
  __syncthreads();
  tc05::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const int total = a.hdr->total_items;
  // move registers from the producer / MMA warpgroup to the two softmax warpgroups
  if (warp >= 8)
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsOther));
  else
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));

  auto decode_item = [&](int item, int& s, int& h, int& q_row0, int& n_q, int& pos0, int& kv_end,
                         int& ctx) {
    const int pair = item / a.hkv;
    h = item - pair * a.hkv;
    const int2 w = a.work[pair];
    s = w.x;
    const int64_t q0 = a.cu_q[s];
    const int count = static_cast<int>(a.cu_q[s + 1] - q0);
    ctx = a.ctx_lens[s];
    const int t_begin = w.y * a.tq;
    n_q = min(a.tq, count - t_begin);
    q_row0 = static_cast<int>(q0) + t_begin;
    pos0 = ctx - count + t_begin;
    kv_end = pos0 + n_q;
  };

  if (warp == kWarpK || warp == kWarpV) {
    // ------------------------------------------------------------------ TMA producers
    // The whole warp runs the loop (warp-uniform coordinates); the elected lane issues.
    {
      const bool leader = elect_one_sync();
      const bool is_k = warp == kWarpK;
      const CUtensorMap* map = is_k ? &kmap : &vmap;
      const uint32_t nst = is_k ? kKStages : kVStages;
      uint64_t* full = &bars[is_k ? kBarKFull : kBarVFull];
      uint64_t* empty = &bars[is_k ? kBarKEmpty : kBarVEmpty];
      uint8_t* ring = smem + (is_k ? L.k0 : L.v0);
      if (leader) {
        if (is_k) prefetch_tensormap(&qmap);
        prefetch_tensormap(map);
      }
      const int32_t layer_base = a.layer * a.nb;
      uint32_t n_items = 0, kv_it = 0, q_issued = 0;
      for (int round = 0, item = snake_item(0); item < total; item = snake_item(++round)) {
        int s, h, q_row0, n_q, pos0, kv_end, ctx;
        decode_item(item, s, h, q_row0, n_q, pos0, kv_end, ctx);
        if (is_k) {
          if (!wait_or_abort(&bars[kBarQEmpty], (n_items & 1u) ^ 1u, abort_flag, a.status)) break;
          ++q_issued;
          if (leader) {
            mbar_arrive_expect_tx(&bars[kBarQFull], QBYTES);
            for (int g = 0; g < a.group; ++g)
#pragma unroll
              for (int sub = 0; sub < SUB; ++sub)
                tc05::tma_load_4d(smem + L.q + sub * 16384 + g * a.tq * 128, &qmap,
                                  &bars[kBarQFull], 0, sub, h * a.group + g, q_row0);
          }
        }
        const int32_t* bt_row = a.bt + static_cast<int64_t>(s) * a.bt_stride;
        const int n_kv = (kv_end + kBN - 1) / kBN;
        bool ok = true;
        // Cache rows of the next tile's 16-row chunks, read one tile ahead so the block-table
        // load latency overlaps the current tile's wait and TMA issue.  (fb, fw) = block index
        // and row within the block of the next chunk; chunks past kv_end load (masked) rows of
        // the sequence's first block.
        int fb = 0, fw = 0;
        int32_t nrow[kChunks];
        auto fetch_rows = [&](int jj) {
#pragma unroll
          for (int b = 0; b < kChunks; ++b) {
            const bool real = jj * kBN + 16 * b < kv_end;
            int32_t blk = bt_row[real ? fb : 0];
            if (blk < 0 || blk >= a.nb) {
              if (leader) flag_status(a.status, B200_DEVICE_BAD_BLOCK);
              blk = 0;
            }
            nrow[b] = (layer_base + blk) * a.bs + (real ? fw : 0);
            fw += 16;
            if (fw == a.bs) {
              fw = 0;
              ++fb;
            }
          }
        };
        fetch_rows(0);
        for (int j = 0; j < n_kv; ++j, ++kv_it) {
          const uint32_t st = kv_it % nst;
          const uint32_t ph = ((kv_it / nst) & 1u) ^ 1u;
          int32_t rows[kChunks];
#pragma unroll
          for (int b = 0; b < kChunks; ++b) rows[b] = nrow[b];
          if (j + 1 < n_kv) fetch_rows(j + 1);
          if (!wait_or_abort(&empty[st], ph, abort_flag, a.status)) {
            ok = false;
            break;
          }
          if (leader) {
            mbar_arrive_expect_tx(&full[st], KT);
            uint8_t* dst = ring + st * KT;
#pragma unroll
            for (int b = 0; b < kChunks; ++b)
#pragma unroll
              for (int sub = 0; sub < SUB; ++sub)
                tma_load_3d(dst + sub * (kBN * 128) + b * 2048, map, &full[st], 0,
                            h * SUB + sub, rows[b]);
          }
        }
        if (!ok) break;
        ++n_items;
      }
      // Every fill this thread issued has landed before the CTA retires (each barrier's latest
      // phase belongs to the last fill issued on it; bounded waits).
      for (uint32_t f = kv_it > nst ? kv_it - nst : 0; f < kv_it; ++f)
        mbar_wait_bounded(&full[f % nst], (f / nst) & 1u);
      if (q_issued > 0) mbar_wait_bounded(&bars[kBarQFull], (q_issued - 1) & 1u);
    }
    __syncwarp();
  } else if (warp == kWarpMma) {
    // ------------------------------------------------------------------ MMA issuer
    // The whole warp runs the loop and waits (warp-uniform descriptors); the elected lane issues
    // the MMAs and commits.
    {
      const bool leader = elect_one_sync();
      uint32_t n_items = 0, kv_it = 0, s_it = 0;
      // descriptor words built once; every MMA below adds a compile-time K-step offset and a
      // ring-stage offset to the low word
      constexpr uint32_t kHi = tc05::desc_hi_sw128(1024);
      const uint32_t q_lo = tc05::desc_lo(base + L.q, 16);
      const uint32_t k_lo0 = tc05::desc_lo(base + L.k0, 16);
      const uint32_t v_lo0 = tc05::desc_lo(base + L.v0, kBN * 128);  // LBO: next 64 columns
      auto issue_s = [&](uint32_t wg, uint32_t stage) {
        const uint32_t k_lo = k_lo0 + stage * (KT >> 4);
        const uint32_t d = tmem + wg * kBN;
        if (!leader) return;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t qo = static_cast<uint32_t>(((kk >> 2) * 16384 + (kk & 3) * 32) >> 4);
          const uint32_t ko = static_cast<uint32_t>(((kk >> 2) * (kBN * 128) + (kk & 3) * 32) >> 4);
          tc05::mma_f16(d, tc05::desc_join(q_lo + qo, kHi), tc05::desc_join(k_lo + ko, kHi),
                        idesc_s, kk > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](uint32_t stage, uint32_t wg, bool acc) {
        const uint32_t v_lo = v_lo0 + stage * (KT >> 4);
        // P of this warpgroup: upper half of its S buffer, 2 values per column; column group g
        // (two K=16 steps) holds keys of chunk kPChunk[g] (32 keys = two 16-row V steps)
        const uint32_t p_t = tmem + wg * kBN + 64;
        const uint32_t d = tmem + kColO + wg * D;
        if (!leader) return;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          const uint32_t vrow16 = kPChunk[kk >> 1] * 2 + (kk & 1);  // 16-key V step
          tc05::mma_f16_ts(d, p_t + kk * 8, tc05::desc_join(v_lo + vrow16 * (2048 >> 4), kHi),
                           idesc_o, (acc || kk > 0) ? 1u : 0u);
        }
      };
      // S(g) from K fill f.  S(g) overwrites the S/P buffer of warpgroup g % 2, whose P(g - 2) is
      // the A operand of PV(g - 2).  S(g) is always issued after PV(g - 2) by this thread, and
      // tcgen05.mma operations from one thread execute in issue order, so PV(g - 2) has read P
      // before S(g) writes the buffer; no completion wait is needed.  (The commit after S(g) also
      // covers PV(g - 2), so a warpgroup that sees S(g) may rescale its O.)
      auto issue_s_tile = [&](uint32_t g, uint32_t f) -> bool {
        const uint32_t wg = g & 1u;
        if (!wait_or_abort(&bars[kBarKFull + f % kKStages], (f / kKStages) & 1u, abort_flag,
                           a.status))
          return false;
        tc05::fence_after_sync();
        issue_s(wg, f % kKStages);
        if (leader) {
          tc05::commit(&bars[kBarSFull + wg]);
          tc05::commit(&bars[kBarKEmpty + f % kKStages]);
        }
        return true;
      };
      for (int round = 0, item = snake_item(0); item < total; item = snake_item(++round)) {
        int s, h, q_row0, n_q, pos0, kv_end, ctx;
        decode_item(item, s, h, q_row0, n_q, pos0, kv_end, ctx);
        const int n_kv = (kv_end + kBN - 1) / kBN;
        if (!wait_or_abort(&bars[kBarQFull], n_items & 1u, abort_flag, a.status)) break;
        tc05::fence_after_sync();
        bool ok = true;
        // the first S tiles of this item overlap the previous item's epilogue
        for (int j = 0; j < 2 && j < n_kv && ok; ++j) ok = issue_s_tile(s_it + j, kv_it + j);
        if (!ok) break;
        if (n_kv <= 2 && leader) tc05::commit(&bars[kBarQEmpty]);
        // both O accumulators are free once all softmax warps have read the previous item's O
        if (!wait_or_abort(&bars[kBarOEmpty], (n_items & 1u) ^ 1u, abort_flag, a.status)) break;
        tc05::fence_after_sync();
        for (int j = 0; j < n_kv; ++j) {
          const uint32_t g = s_it + j;
          const uint32_t f = kv_it + j;
          const uint32_t wg = g & 1u;
          if (!wait_or_abort(&bars[kBarPFull + wg], (g >> 1) & 1u, abort_flag, a.status) ||
              !wait_or_abort(&bars[kBarVFull + f % kVStages], (f / kVStages) & 1u, abort_flag,
                             a.status)) {
            ok = false;
            break;
          }
          tc05::fence_after_sync();
          issue_pv(f % kVStages, wg, j >= 2);  // tile j-2 went to the same accumulator
          if (leader) {
            tc05::commit(&bars[kBarPvDone + wg]);
            tc05::commit(&bars[kBarVEmpty + f % kVStages]);
          }
          if (j + 2 < n_kv) {
            if (!issue_s_tile(g + 2, f + 2)) {
              ok = false;
              break;
            }
            if (j + 2 == n_kv - 1 && leader) tc05::commit(&bars[kBarQEmpty]);  // last S of item
          }
        }
        if (!ok) break;
        kv_it += n_kv;
        s_it += n_kv;
        ++n_items;
      }
      // all tcgen05 work the leader issued completes before TMEM is released
      if (leader) tc05::commit(&bars[kBarFinal]);
      mbar_wait_bounded(&bars[kBarFinal], 0);
    }
    __syncwarp();
  } else if (warp < 8) {
    // ------------------------------------------------------------------ softmax / epilogue
    // warps 0-3 = warpgroup 0, warps 4-7 = warpgroup 1; TMEM lane quarter = warp % 4
    const uint32_t wg = static_cast<uint32_t>(warp) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int g = row / a.tq;
    const int t = row - g * a.tq;
    const uint32_t trow = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t s_self = trow + wg * kBN;
    const uint32_t o_self = trow + kColO + wg * D;
    const int sm_tid = (warp & 3) * 32 + lane;  // 0..127 within the warpgroup
    float2* xch = reinterpret_cast<float2*>(smem + L.xch);
    uint32_t s_it = 0, kv_it = 0, n_items = 0;
    for (int round = 0, item = snake_item(0); item < total; item = snake_item(++round)) {
      int s, h, q_row0, n_q, pos0, kv_end, ctx;
      decode_item(item, s, h, q_row0, n_q, pos0, kv_end, ctx);
      const int n_kv = (kv_end + kBN - 1) / kBN;
      const bool valid = t < n_q;
      const int pos = valid ? pos0 + t : -1;
      // tiles of this warpgroup: j = j0, j0 + 2, ... (global tile number g = s_it + j, g % 2 == wg)
      const int j0 = static_cast<int>((s_it ^ wg) & 1u);
      float m = -INFINITY, l = 0.f;
      bool ok = true;
      int j = j0;
      for (; j < n_kv; j += 2) {
        const uint32_t gt = s_it + j;
        ok = wait_or_abort(&bars[kBarSFull + wg], (gt >> 1) & 1u, abort_flag, a.status);
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        tc05::fence_after_sync();
        // causal mask only where some row of this warp ends inside the tile
        const bool need_mask = __any_sync(0xffffffffu, j * kBN + kBN - 1 > pos);
        const int lim = pos - j * kBN;  // columns c > lim are in the future of this row
        // pass 1: row max over the tile, two 64-column halves (one TMEM wait each); the second
        // half stays in registers for pass 2
        float va[32], vb[32];
        auto mask_chunk = [&](float (&v)[32], int chunk) {
          if (need_mask) {
#pragma unroll
            for (int c = 0; c < 32; ++c)
              if (chunk * 32 + c > lim) v[c] = -INFINITY;
          }
        };
        float mx8[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) mx8[k] = -INFINITY;
        auto max_chunk = [&](const float (&v)[32]) {
#pragma unroll
          for (int c = 0; c < 32; ++c) mx8[c & 7] = fmaxf(mx8[c & 7], v[c]);
        };
        tc05::ld_32x32b_x32(s_self, va);
        tc05::ld_32x32b_x32(s_self + 32, vb);
        tc05::wait_ld();
        mask_chunk(va, 0);
        mask_chunk(vb, 1);
        max_chunk(va);
        max_chunk(vb);
        tc05::ld_32x32b_x32(s_self + 64, va);
        tc05::ld_32x32b_x32(s_self + 96, vb);
        tc05::wait_ld();
        mask_chunk(va, 2);
        mask_chunk(vb, 3);
        max_chunk(va);
        max_chunk(vb);
        const float smax = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                                 fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
        // Online softmax with a lazily moved reference max: the row keeps using its current
        // reference m until the tile max exceeds it by more than 8 (log2 units), so p stays below
        // 2^8 and O / l are rescaled only on such jumps.  O and l always share the same m, so the
        // final O / l is exact whichever m was used.
        const float tmax = smax * a.scale_log2;  // scale > 0: max commutes with scaling
        float alpha = 1.f;
        if (m == -INFINITY) {
          m = tmax;                    // first keys of this row in this warpgroup
        } else if (tmax > m + 8.f) {
          alpha = fast_exp2(m - tmax);
          m = tmax;
        }
        const float mu = m == -INFINITY ? 0.f : m;
        // pass 2: p = 2^(s*scale - m), packed in pairs into the upper half of the S buffer
        // (columns 64..127).  Chunks 2 and 3 (still in registers) go first, onto their own
        // consumed columns; then chunks 0 and 1 are re-read.  P column group g (16 columns = 32 keys)
        // holds key chunk kPChunk[g] = 2, 3, 0, 1; the PV MMA reads V in the same order.
        float rs8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        auto exp_chunk = [&](const float (&x)[32], int group) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {  // two 16-key halves, 8 packed columns each
            float pk[8];
#pragma unroll
            for (int c = 0; c < 16; c += 2) {
              const float p0 = fast_exp2(fmaf(x[16 * h + c], a.scale_log2, -mu));
              const float p1 = fast_exp2(fmaf(x[16 * h + c + 1], a.scale_log2, -mu));
              rs8[c & 7] += p0;
              rs8[(c + 1) & 7] += p1;
              pk[c >> 1] = __uint_as_float(MmaOp<T>::pack(p0, p1));
            }
            tc05::st_32x32b_x8(s_self + 64 + group * 16 + h * 8, pk);
          }
        };
        exp_chunk(va, 0);                           // keys 64..95  -> columns 64..79
        exp_chunk(vb, 1);                           // keys 96..127 -> columns 80..95
        tc05::ld_32x32b_x32(s_self, va);            // keys 0..63 again (one wait)
        tc05::ld_32x32b_x32(s_self + 32, vb);
        tc05::wait_ld();
        mask_chunk(va, 0);
        mask_chunk(vb, 1);
        exp_chunk(va, 2);                           // keys 0..31   -> columns 96..111
        exp_chunk(vb, 3);                           // keys 32..63  -> columns 112..127
        const float rs = ((rs8[0] + rs8[1]) + (rs8[2] + rs8[3])) +
                         ((rs8[4] + rs8[5]) + (rs8[6] + rs8[7]));
        l = l * alpha + rs;
        // O rescale: PV(gt - 2), the last MMA into this accumulator, was issued before S(gt) and
        // is covered by the commit that signalled S(gt), so O can be read and written here
        if (j >= 2 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
          for (int ch = 0; ch < D / 16; ++ch) {
            float o[16];
            tc05::ld_32x32b_x16(o_self + ch * 16, o);
            tc05::wait_ld();
#pragma unroll
            for (int c = 0; c < 16; ++c) o[c] *= alpha;
            tc05::st_32x32b_x16(o_self + ch * 16, o);
          }
        }
        tc05::wait_st();
        if (j == n_kv - 1 && kv_end < j * kBN + kBN) {
          // keys past kv_end are masked for every row; their V rows may hold anything -> zero
          // (after the V tile has landed)
          const uint32_t fv = kv_it + j;
          ok = wait_or_abort(&bars[kBarVFull + fv % kVStages], (fv / kVStages) & 1u, abort_flag,
                             a.status);
          if (!__all_sync(0xffffffffu, ok)) {
            ok = false;
            break;
          }
          uint8_t* vst = smem + L.v0 + (fv % kVStages) * KT;
          const int r0 = kv_end - j * kBN;
          const int nz = (kBN - r0) * SUB * 8;  // 16-byte chunks
          for (int idx = sm_tid; idx < nz; idx += 128) {
            const int rr = r0 + idx / (SUB * 8);
            const int rem = idx % (SUB * 8);
            *reinterpret_cast<uint4*>(vst + (rem >> 3) * (kBN * 128) + rr * 128 + (rem & 7) * 16) =
                make_uint4(0u, 0u, 0u, 0u);
          }
          fence_proxy_async_smem();
        }
        tc05::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc05::mbar_arrive(&bars[kBarPFull + wg]);
      }
      if (!ok) break;
      // ---- epilogue: wait for this warpgroup's last PV, exchange (m, l) with the other
      // warpgroup, merge the two partial accumulators (each warpgroup writes half the columns)
      const bool had_tiles = j0 < n_kv;
      if (had_tiles) {
        const uint32_t gl = s_it + static_cast<uint32_t>(j - 2);  // last tile of this warpgroup
        ok = wait_or_abort(&bars[kBarPvDone + wg], (gl >> 1) & 1u, abort_flag, a.status);
        if (!__all_sync(0xffffffffu, ok)) break;
      }
      float2* xb = xch + (n_items & 1u) * 256;
      xb[wg * 128 + row] = make_float2(m, l);
      tc05::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc05::mbar_arrive(&bars[kBarXchg]);
      ok = wait_or_abort(&bars[kBarXchg], n_items & 1u, abort_flag, a.status);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc05::fence_after_sync();
      const float2 other = xb[(wg ^ 1u) * 128 + row];
      // row max / sum of warpgroup 0 and 1
      const float m0 = wg == 0 ? m : other.x, l0 = wg == 0 ? l : other.y;
      const float m1 = wg == 0 ? other.x : m, l1 = wg == 0 ? other.y : l;
      const float mm = fmaxf(m0, m1);
      const float f0 = (l0 > 0.f) ? fast_exp2(m0 - mm) : 0.f;
      const float f1 = (l1 > 0.f) ? fast_exp2(m1 - mm) : 0.f;
      const float lt = l0 * f0 + l1 * f1;
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      const float w0 = f0 * inv, w1 = f1 * inv;
      // an accumulator that received no PV in this item holds stale data: not read at all
      const bool has0 = static_cast<int>((s_it & 1u)) < n_kv;           // warpgroup 0 had tiles
      const bool has1 = static_cast<int>(((s_it ^ 1u) & 1u)) < n_kv;    // warpgroup 1 had tiles
      T* orow = static_cast<T*>(a.out) + static_cast<int64_t>(q_row0 + t) * a.o_stok +
                static_cast<int64_t>(h * a.group + g) * a.o_shead;
#pragma unroll
      for (int hc = 0; hc < D / 32; ++hc) {
        const int c0 = static_cast<int>(wg) * (D / 2) + hc * 16;  // 16-column chunk of O
        float o[16];
        if (has0) {
          tc05::ld_32x32b_x16(trow + kColO + c0, o);
          tc05::wait_ld();
#pragma unroll
          for (int c = 0; c < 16; ++c) o[c] *= w0;
        } else {
#pragma unroll
          for (int c = 0; c < 16; ++c) o[c] = 0.f;
        }
        if (has1) {
          float o1[16];
          tc05::ld_32x32b_x16(trow + kColO + D + c0, o1);
          tc05::wait_ld();
#pragma unroll
          for (int c = 0; c < 16; ++c) o[c] = fmaf(o1[c], w1, o[c]);
        }
        if (valid) {
          if (a.vec_out) {
#pragma unroll
            for (int c8 = 0; c8 < 2; ++c8) {
              uint4 v;
              v.x = MmaOp<T>::pack(o[c8 * 8 + 0], o[c8 * 8 + 1]);
              v.y = MmaOp<T>::pack(o[c8 * 8 + 2], o[c8 * 8 + 3]);
              v.z = MmaOp<T>::pack(o[c8 * 8 + 4], o[c8 * 8 + 5]);
              v.w = MmaOp<T>::pack(o[c8 * 8 + 6], o[c8 * 8 + 7]);
              *reinterpret_cast<uint4*>(orow + c0 + c8 * 8) = v;
            }
          } else {
#pragma unroll
            for (int c = 0; c < 16; ++c) orow[c0 + c] = from_f32<T>(o[c]);
          }
        }
      }
      tc05::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc05::mbar_arrive(&bars[kBarOEmpty]);
      s_it += n_kv;
      kv_it += n_kv;
      ++n_items;
    }
  }

  tc05::fence_before_sync();
  __syncthreads();
  if (warp == kWarpMma) {
    tc05::fence_after_sync();
    tc05::tmem_dealloc(tmem, kTmemCols);
  }
}

template <typename T, int D>
static cudaError_t launch_prefill_tc_t(const CUtensorMap& qm, const CUtensorMap& km,
                                       const CUtensorMap& vm, const PrefillArgs& a,
                                       int max_items, int num_sms, cudaStream_t stream) {
  constexpr SmemLayout L = prefill_layout<D>();
  // at least ~116 KB so that one CTA (and one 256-column TMEM allocation) sits on each SM
  const int smem = static_cast<int>(L.total) + 1024 > 118 * 1024 ? static_cast<int>(L.total) + 1024
                                                                  : 118 * 1024;
  static bool configured = false;
  auto kern = prefill_tc_kernel<T, D>;
  if (!configured) {
    // the register split must fit the registers the CTA is launched with
    cudaFuncAttributes fa{};
    cudaError_t e = cudaFuncGetAttributes(&fa, kern);
    if (e != cudaSuccess) return e;
    if (static_cast<long>(fa.numRegs) * kPrefillThreads <
        256L * kRegsSoftmax + 128L * kRegsOther) {
      set_last_error("prefill kernel compiled with too few registers for its register split");
      return cudaErrorInvalidConfiguration;
    }
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  int grid = num_sms;
  if (max_items < grid) grid = max_items;
  if (grid < 1) grid = 1;
  kern<<<grid, kPrefillThreads, smem, stream>>>(qm, km, vm, a);
  return cudaGetLastError();
}

cudaError_t launch_prefill_plan(const PrefillPlanArgs& a, cudaStream_t stream) {
  prefill_plan_kernel<<<1, 1024, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_prefill_tc(int dtype, int head_dim, const CUtensorMap& qm,
                              const CUtensorMap& km, const CUtensorMap& vm, const PrefillArgs& a,
                              int max_items, int num_sms, cudaStream_t stream) {
  if (dtype == B200_DTYPE_BF16) {
    if (head_dim == 128)
      return launch_prefill_tc_t<__nv_bfloat16, 128>(qm, km, vm, a, max_items, num_sms, stream);
    if (head_dim == 64)
      return launch_prefill_tc_t<__nv_bfloat16, 64>(qm, km, vm, a, max_items, num_sms, stream);
  } else if (dtype == B200_DTYPE_F16) {
    if (head_dim == 128)
      return launch_prefill_tc_t<__half, 128>(qm, km, vm, a, max_items, num_sms, stream);
    if (head_dim == 64)
      return launch_prefill_tc_t<__half, 64>(qm, km, vm, a, max_items, num_sms, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace b200
