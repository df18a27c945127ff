// K3, the default tensor-core prefill (b200_set_prefill_kernel(0) selects the one-tile kernel of
// prefill.cu instead, 2 the two-stream kernel of prefill_ds.cu): two 128-row query tiles per work
// item, one per softmax warpgroup, against one stream of 128-key K/V tiles.
//
// One work item = (sequence, pair of query tiles of TQ = 128/G tokens each, KV head).  Softmax
// warpgroup w owns query tile w (rows g*TQ + t of tokens [t_begin + w*TQ, t_begin + (w+1)*TQ)) for
// the whole KV range it attends, so it keeps one running (max, sum) per row and one O accumulator
// and writes its rows itself: no per-item exchange or merge between the warpgroups.  Each K/V tile
// is staged once and feeds S0 = Q0.K^T, S1 = Q1.K^T, O0 += P0.V, O1 += P1.V.
//
// Roles (384 threads, setmaxnreg split as in prefill.cu):
//   warps 0-3 / 4-7  softmax warpgroup 0 / 1 (query tile 0 / 1)
//   warp 8           TMA: both Q tiles of an item, K tiles (kKStages ring)
//   warp 10          TMA: V tiles (kVStages ring)
//   warp 9           TMEM owner, MMA issuer: per KV tile j, for w = 0, 1: PV_w(j), then S_w(j+1)
//                    (S_w(j+1) overwrites S/P_w after PV_w(j) read P_w: in-order tcgen05.mma)
//   warp 11          idle
// TMEM: S/P of warpgroup w at [128w, 128w + 128) (P in the upper 64 columns), O_w at
// [256 + w*D, 256 + (w+1)*D).
//
// Per-item synchronisation: the MMA warp waits OEmpty_w (warpgroup w has read O_w of the previous
// item) before the first PV_w of an item.  A warpgroup with rows in the item is gated by its first
// SFull wait, and it cannot arrive OEmpty again before the MMA warp consumed the previous arrival
// (that needs PV_w of this item); a warpgroup without rows in the item (the last pair of a sequence
// may hold one tile) waits Begin_w instead, which the MMA warp arrives after that OEmpty_w wait.
// So every parity wait is unambiguous.
// V rows past the item's last key in its last tile are zeroed (masked P is exactly 0, but 0 * NaN
// from an unwritten slot is not) by warpgroup 0 when it attends that tile (its softmax runs
// first), else by warpgroup 1; the MMA warp waits for that warpgroup's P before issuing either PV
// on the tile.
// Epilogue: each softmax warp stages its 32 output rows, 64 columns at a time, in its own 4 KB of
// shared memory (16-byte chunks XOR-swizzled by row), and writes them back as whole 128-byte row
// segments, four rows per store instruction.
// Every wait is bounded; an expired wait records B200_DEVICE_TIMEOUT and stops the CTA.
#include <type_traits>

#include "attention.cuh"
#include "softmax_sm100.cuh"
#include "tc05.cuh"

namespace b200 {

namespace {

constexpr int kBN = 128;
constexpr int kKStages = 2;
constexpr int kVStages = 2;
// Register split (setmaxnreg): each softmax thread holds its whole 128-column S row in registers
// (one TMEM wait per tile); 256 x kRegsSoftmax + 128 x kRegsOther = 384 x 168, the registers the
// CTA is launched with (the launcher checks the compiled count before the first launch).
constexpr uint32_t kRegsSoftmax = 200;
constexpr uint32_t kRegsOther = 104;
constexpr int kWarpK = 8, kWarpMma = 9, kWarpV = 10;

struct SmemLayout {
  uint32_t q, k0, v0, o, bars, total;
};

// epilogue staging: 32 rows x 128 bytes per softmax warp
constexpr uint32_t kOStageWarp = 32 * 128;

template <int D>
__host__ __device__ constexpr SmemLayout q2_layout() {
  constexpr uint32_t SUB = D / 64;
  constexpr uint32_t QT = SUB * 128 * 128;  // one 128-row query tile
  constexpr uint32_t KT = SUB * kBN * 128;  // one 128-key K or V tile
  constexpr uint32_t KV = (kKStages + kVStages) * KT;
  constexpr uint32_t OS = 8 * kOStageWarp;
  return SmemLayout{0, 2 * QT, 2 * QT + kKStages * KT, 2 * QT + KV, 2 * QT + KV + OS,
                    2 * QT + KV + OS + 512};
}

enum : int {
  kBarQFull = 0,
  kBarQEmpty,
  kBarKFull,                          // + K stage
  kBarKEmpty = kBarKFull + kKStages,
  kBarVFull = kBarKEmpty + kKStages,  // + V stage
  kBarVEmpty = kBarVFull + kVStages,
  kBarSFull = kBarVEmpty + kVStages,  // + warpgroup
  kBarPFull = kBarSFull + 2,          // + warpgroup (4 arrivals)
  kBarPvDone = kBarPFull + 2,         // + warpgroup
  kBarOEmpty = kBarPvDone + 2,        // + warpgroup (4 arrivals)
  kBarBegin = kBarOEmpty + 2,         // + warpgroup (1 arrival)
  kBarFinal = kBarBegin + 2,
  kNumBars
};

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

// One work item: sequence s, KV head h, query tiles w = 0, 1 of TQ tokens starting at q_row0.
struct Q2Item {
  int s, h, q_row0, pos0;  // pos0: position of tile 0's first token
  int n_q[2];              // tokens of tile w (tile 1 may be empty)
  int kv_end[2];           // keys attended by tile w's last token + 1
  int n_kv[2];             // KV tiles of warpgroup w (0 if the tile is empty)
  int n_kv_all, kv_end_all;
};

__device__ __forceinline__ Q2Item q2_decode(const PrefillArgs& a, int item) {
  Q2Item it;
  const int pair = item / a.hkv;
  it.h = item - pair * a.hkv;
  const int2 w = a.work[pair];
  it.s = w.x;
  const int64_t q0 = a.cu_q[it.s];
  const int count = static_cast<int>(a.cu_q[it.s + 1] - q0);
  const int ctx = a.ctx_lens[it.s];
  const int t_begin = w.y * 2 * a.tq;
  it.q_row0 = static_cast<int>(q0) + t_begin;
  it.pos0 = ctx - count + t_begin;
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int n = count - t_begin - t * a.tq;
    it.n_q[t] = n < 0 ? 0 : (n > a.tq ? a.tq : n);
    it.kv_end[t] = it.pos0 + t * a.tq + it.n_q[t];
    it.n_kv[t] = it.n_q[t] > 0 ? (it.kv_end[t] + kBN - 1) / kBN : 0;
  }
  it.n_kv_all = it.n_kv[0] > it.n_kv[1] ? it.n_kv[0] : it.n_kv[1];
  it.kv_end_all = it.n_q[1] > 0 ? it.kv_end[1] : it.kv_end[0];
  return it;
}

// The warpgroup that zeroes the V rows past kv_end_all in the item's last KV tile: warpgroup 0
// when it attends that tile, else warpgroup 1 (which then holds the item's latest rows).
__device__ __forceinline__ int q2_zero_wg(const Q2Item& it) {
  return it.n_kv[0] == it.n_kv_all ? 0 : 1;
}

}  // namespace

// kPolyMask: bit i set = pair i of every 8 consecutive exponential pairs of a row is computed by
// exp2_poly2 on the FMA pipe instead of ex2 on the SFU.
template <typename T, int D, uint32_t kPolyMask>
__global__ void __launch_bounds__(kPrefillThreads, 1)
    prefill_q2_kernel(const __grid_constant__ CUtensorMap qmap,
                      const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap, PrefillArgs a) {
  constexpr int SUB = D / 64;
  constexpr int kChunks = kBN / 16;
  constexpr SmemLayout L = q2_layout<D>();
  constexpr uint32_t KT = SUB * kBN * 128;
  constexpr uint32_t QT = SUB * 128 * 128;
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
      mbar_init(&bars[kBarPFull + w], 4);
      mbar_init(&bars[kBarPvDone + w], 1);
      mbar_init(&bars[kBarOEmpty + w], 4);
      mbar_init(&bars[kBarBegin + w], 1);
    }
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
  // Each warpgroup changes its register count inside its own branch, so that the compiler
  // allocates the softmax code against kRegsSoftmax and the producer / MMA code against
  // kRegsOther.
  if (warp >= 8) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsOther));
    if (warp == kWarpK || warp == kWarpV) {
      // ------------------------------------------------------------------ TMA producers
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
          const Q2Item it = q2_decode(a, item);
          if (is_k) {
            if (!wait_or_abort(&bars[kBarQEmpty], (n_items & 1u) ^ 1u, abort_flag, a.status)) break;
            ++q_issued;
            if (leader) {
              // both tiles, always: rows past the batch read the fill value, rows of the next
              // sequence are never stored (their t >= n_q)
              mbar_arrive_expect_tx(&bars[kBarQFull], 2 * QT);
              for (int w = 0; w < 2; ++w)
                for (int g = 0; g < a.group; ++g)
#pragma unroll
                  for (int sub = 0; sub < SUB; ++sub)
                    tc05::tma_load_4d(smem + L.q + w * QT + sub * 16384 + g * a.tq * 128, &qmap,
                                      &bars[kBarQFull], 0, sub, it.h * a.group + g,
                                      it.q_row0 + w * a.tq);
            }
          }
          const int32_t* bt_row = a.bt + static_cast<int64_t>(it.s) * a.bt_stride;
          const int n_kv = it.n_kv_all;
          const int kv_end = it.kv_end_all;
          bool ok = true;
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
                              it.h * SUB + sub, rows[b]);
            }
          }
          if (!ok) break;
          ++n_items;
        }
        for (uint32_t f = kv_it > nst ? kv_it - nst : 0; f < kv_it; ++f)
          mbar_wait_bounded(&full[f % nst], (f / nst) & 1u);
        if (q_issued > 0) mbar_wait_bounded(&bars[kBarQFull], (q_issued - 1) & 1u);
      }
      __syncwarp();
    } else if (warp == kWarpMma) {
      // ------------------------------------------------------------------ MMA issuer
      {
        const bool leader = elect_one_sync();
        uint32_t n_items = 0, kv_it = 0;
        uint32_t c_tile[2] = {0u, 0u};  // tiles issued to warpgroup w so far (phase index)
        constexpr uint32_t kHi = tc05::desc_hi_sw128(1024);
        const uint32_t q_lo0 = tc05::desc_lo(base + L.q, 16);
        const uint32_t k_lo0 = tc05::desc_lo(base + L.k0, 16);
        const uint32_t v_lo0 = tc05::desc_lo(base + L.v0, kBN * 128);
        auto issue_s = [&](uint32_t wg, uint32_t stage) {
          const uint32_t q_lo = q_lo0 + wg * (QT >> 4);
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
          const uint32_t p_t = tmem + wg * kBN + 64;
          const uint32_t d = tmem + kColO + wg * D;
          if (!leader) return;
#pragma unroll
          for (int kk = 0; kk < kBN / 16; ++kk) {
            const uint32_t vrow16 = kk;  // P columns hold the keys in order: 16 keys per K step
            tc05::mma_f16_ts(d, p_t + kk * 8, tc05::desc_join(v_lo + vrow16 * (2048 >> 4), kHi),
                             idesc_o, (acc || kk > 0) ? 1u : 0u);
          }
        };
        auto wait_k = [&](uint32_t f) {
          return wait_or_abort(&bars[kBarKFull + f % kKStages], (f / kKStages) & 1u, abort_flag,
                               a.status);
        };
        bool ok = true;
        for (int round = 0, item = snake_item(0); item < total && ok; item = snake_item(++round)) {
          const Q2Item it = q2_decode(a, item);
          const int n_kv = it.n_kv_all;
          const int zw = q2_zero_wg(it);
          const bool needs_zero = it.kv_end_all < n_kv * kBN;
          if (!wait_or_abort(&bars[kBarQFull], n_items & 1u, abort_flag, a.status)) break;
          tc05::fence_after_sync();
          // prologue: S_w(0) of this item (it may overlap the previous item's epilogues: S/P_w is
          // free once PV_w of the previous item's last tile was issued, which came before)
          if (!wait_k(kv_it)) break;
          tc05::fence_after_sync();
#pragma unroll
          for (uint32_t w = 0; w < 2; ++w) {
            if (it.n_kv[w] == 0) continue;
            issue_s(w, kv_it % kKStages);
            if (leader) tc05::commit(&bars[kBarSFull + w]);
          }
          if (leader) {
            tc05::commit(&bars[kBarKEmpty + kv_it % kKStages]);
            if (n_kv == 1) tc05::commit(&bars[kBarQEmpty]);
          }
          // each warpgroup's previous epilogue must have read O_w before PV_w(0) overwrites it;
          // then the warpgroup may begin this item
#pragma unroll
          for (uint32_t w = 0; w < 2; ++w) {
            if (!ok) break;
            ok = wait_or_abort(&bars[kBarOEmpty + w], (n_items & 1u) ^ 1u, abort_flag, a.status);
            if (ok && leader && it.n_kv[w] == 0) tc05::mbar_arrive(&bars[kBarBegin + w]);
          }
          if (!ok) break;
          tc05::fence_after_sync();
          for (int j = 0; j < n_kv && ok; ++j) {
            const uint32_t f = kv_it + j;
            const bool zero_here = needs_zero && j == n_kv - 1;
            if (!wait_or_abort(&bars[kBarVFull + f % kVStages], (f / kVStages) & 1u, abort_flag,
                               a.status)) {
              ok = false;
              break;
            }
            if (zero_here && !wait_or_abort(&bars[kBarPFull + zw], ((zw ? c_tile[1] : c_tile[0]) + j) & 1u,
                                            abort_flag, a.status)) {
              ok = false;
              break;
            }
#pragma unroll
            for (uint32_t w = 0; w < 2; ++w) {
              if (j >= it.n_kv[w]) continue;
              if (!wait_or_abort(&bars[kBarPFull + w], (c_tile[w] + j) & 1u, abort_flag, a.status)) {
                ok = false;
                break;
              }
              tc05::fence_after_sync();
              issue_pv(f % kVStages, w, j > 0);
              if (leader) tc05::commit(&bars[kBarPvDone + w]);
              if (j + 1 < it.n_kv[w]) {
                // the first warpgroup needing K tile j+1 waits for it; the last releases it
                const bool first = (w == 0) || (j + 1 >= it.n_kv[0]);
                const bool last = (w == 1) || (j + 1 >= it.n_kv[1]);
                if (first && !wait_k(f + 1)) {
                  ok = false;
                  break;
                }
                tc05::fence_after_sync();
                issue_s(w, (f + 1) % kKStages);
                if (leader) {
                  tc05::commit(&bars[kBarSFull + w]);
                  if (last) {
                    tc05::commit(&bars[kBarKEmpty + (f + 1) % kKStages]);
                    if (j + 1 == n_kv - 1) tc05::commit(&bars[kBarQEmpty]);
                  }
                }
              }
            }
            if (ok && leader) tc05::commit(&bars[kBarVEmpty + f % kVStages]);
          }
          if (!ok) break;
          kv_it += n_kv;
          c_tile[0] += it.n_kv[0];
          c_tile[1] += it.n_kv[1];
          ++n_items;
        }
        if (leader) tc05::commit(&bars[kBarFinal]);
        mbar_wait_bounded(&bars[kBarFinal], 0);
      }
      __syncwarp();
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
    // ------------------------------------------------------------------ softmax / epilogue
    const uint32_t wg = static_cast<uint32_t>(warp) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int g = row / a.tq;
    const int t = row - g * a.tq;
    const uint32_t trow = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t s_self = trow + wg * kBN;
    const uint32_t o_self = trow + kColO + wg * D;
    const int sm_tid = quarter * 32 + lane;
    uint32_t c_tile = 0, kv_it = 0, n_items = 0, n_idle = 0;
    Q2Item nx{};
    if (snake_item(0) < total) nx = q2_decode(a, snake_item(0));
    for (int round = 0, item = snake_item(0); item < total; item = snake_item(++round)) {
      const Q2Item it = nx;
      const int n_kv = wg ? it.n_kv[1] : it.n_kv[0];
      const int n_q = wg ? it.n_q[1] : it.n_q[0];
      const bool valid = t < n_q;
      const int pos = valid ? it.pos0 + static_cast<int>(wg) * a.tq + t : -1;
      const bool zeroer = static_cast<int>(wg) == q2_zero_wg(it) &&
                          it.kv_end_all < it.n_kv_all * kBN;
      bool ok = true;
      if (n_kv == 0) {
        ok = wait_or_abort(&bars[kBarBegin + wg], n_idle & 1u, abort_flag, a.status);
        ++n_idle;
        if (!__all_sync(0xffffffffu, ok)) break;
      }
      float m = -INFINITY, l = 0.f;
      int j = 0;
      for (; j < n_kv; ++j) {
        const uint32_t gt = c_tile + j;
        ok = wait_or_abort(&bars[kBarSFull + wg], gt & 1u, abort_flag, a.status);
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        tc05::fence_after_sync();
        const bool need_mask = __any_sync(0xffffffffu, j * kBN + kBN - 1 > pos);
        const int lim = pos - j * kBN;
        // the whole S row of this thread: four 32-column loads, one wait
        float sa[32], sb[32], sc[32], sd[32];
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
          for (int c = 0; c < 32; c += 2) mx8[(c >> 1) & 7] = fmax3(mx8[(c >> 1) & 7], v[c], v[c + 1]);
        };
        tc05::ld_32x32b_x32(s_self, sa);
        tc05::ld_32x32b_x32(s_self + 32, sb);
        tc05::ld_32x32b_x32(s_self + 64, sc);
        tc05::ld_32x32b_x32(s_self + 96, sd);
        tc05::wait_ld();
        mask_chunk(sa, 0);
        mask_chunk(sb, 1);
        mask_chunk(sc, 2);
        mask_chunk(sd, 3);
        max_chunk(sa);
        max_chunk(sb);
        max_chunk(sc);
        max_chunk(sd);
        const float smax = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                                 fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
        const float tmax = smax * a.scale_log2;
        float alpha = 1.f;
        if (m == -INFINITY) {
          m = tmax;
        } else if (tmax > m + 8.f) {
          alpha = fast_exp2(m - tmax);
          m = tmax;
        }
        const float mu = m == -INFINITY ? 0.f : m;
        // p = 2^(s*scale - m) for pairs of keys: the argument by one packed FMA, the
        // exponential on the SFU or (pairs selected by kPolyMask) by exp2_poly2, the row sum by
        // packed adds into four accumulators
        const uint64_t scale2 = f2_pack(a.scale_log2, a.scale_log2);
        const uint64_t negmu2 = f2_pack(-mu, -mu);
        uint64_t rs2[4] = {0ull, 0ull, 0ull, 0ull};
        auto exp_chunk = [&](const float (&x)[32], int group) {
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            float pk[8];
#pragma unroll
            for (int c = 0; c < 16; c += 2) {
              const int pi = c >> 1;
              const uint64_t arg = f2_fma(f2_pack(x[16 * hh + c], x[16 * hh + c + 1]), scale2, negmu2);
              float p0, p1;
              if ((kPolyMask >> pi) & 1u) {
                exp2_poly2(arg, p0, p1);
              } else {
                float a0, a1;
                f2_unpack(arg, a0, a1);
                p0 = fast_exp2(a0);
                p1 = fast_exp2(a1);
              }
              rs2[pi & 3] = f2_add(rs2[pi & 3], f2_pack(p0, p1));
              pk[pi] = __uint_as_float(MmaOp<T>::pack(p0, p1));
            }
            tc05::st_32x32b_x8(s_self + 64 + group * 16 + hh * 8, pk);
          }
        };
        // P over the S columns 64..127, keys in order (all of S is in registers by now)
        exp_chunk(sa, 0);
        exp_chunk(sb, 1);
        exp_chunk(sc, 2);
        exp_chunk(sd, 3);
        float rsl[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) f2_unpack(rs2[k], rsl[2 * k], rsl[2 * k + 1]);
        const float rs = ((rsl[0] + rsl[1]) + (rsl[2] + rsl[3])) + ((rsl[4] + rsl[5]) + (rsl[6] + rsl[7]));
        l = l * alpha + rs;
        // PV_w(j - 1), the last MMA into O_w, was issued before S_w(j) and is covered by the
        // commit that signalled S_w(j)
        if (j >= 1 && __any_sync(0xffffffffu, alpha != 1.f)) {
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
        if (zeroer && j == it.n_kv_all - 1) {
          const uint32_t fv = kv_it + j;
          ok = wait_or_abort(&bars[kBarVFull + fv % kVStages], (fv / kVStages) & 1u, abort_flag,
                             a.status);
          if (!__all_sync(0xffffffffu, ok)) {
            ok = false;
            break;
          }
          uint8_t* vst = smem + L.v0 + (fv % kVStages) * KT;
          const int r0 = it.kv_end_all - j * kBN;
          const int nz = (kBN - r0) * SUB * 8;
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
      // the next item's indices load here, ahead of this item's output stores (loads issued after
      // them queue behind them)
      if (snake_item(round + 1) < total) nx = q2_decode(a, snake_item(round + 1));
      // ---- epilogue: this warpgroup's rows only
      if (n_kv > 0) {
        ok = wait_or_abort(&bars[kBarPvDone + wg], (c_tile + n_kv - 1) & 1u, abort_flag, a.status);
        if (!__all_sync(0xffffffffu, ok)) break;
        tc05::fence_after_sync();
        const float inv = l > 0.f ? 1.f / l : 0.f;
        if (a.vec_out) {
          // stage 64 columns of the warp's 32 rows, then write 4 rows x 128 B per instruction
          uint8_t* stage = smem + L.o + warp * kOStageWarp;
          const int64_t head0 = static_cast<int64_t>(it.h * a.group);
          const int tok0 = it.q_row0 + static_cast<int>(wg) * a.tq;
#pragma unroll
          for (int half = 0; half < D / 64; ++half) {
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) {
              float o[16];
              tc05::ld_32x32b_x16(o_self + half * 64 + ch * 16, o);
              tc05::wait_ld();
#pragma unroll
              for (int c8 = 0; c8 < 2; ++c8) {
                uint4 v;
                v.x = MmaOp<T>::pack(o[c8 * 8 + 0] * inv, o[c8 * 8 + 1] * inv);
                v.y = MmaOp<T>::pack(o[c8 * 8 + 2] * inv, o[c8 * 8 + 3] * inv);
                v.z = MmaOp<T>::pack(o[c8 * 8 + 4] * inv, o[c8 * 8 + 5] * inv);
                v.w = MmaOp<T>::pack(o[c8 * 8 + 6] * inv, o[c8 * 8 + 7] * inv);
                const int k = ch * 2 + c8;
                *reinterpret_cast<uint4*>(stage + lane * 128 + ((k ^ (lane & 7)) << 4)) = v;
              }
            }
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int rr = i * 4 + (lane >> 3);  // row within the warp
              const int k = lane & 7;              // 16-byte chunk within the 128-byte segment
              const uint4 v =
                  *reinterpret_cast<const uint4*>(stage + rr * 128 + ((k ^ (rr & 7)) << 4));
              const int wrow = quarter * 32 + rr;  // row within the warpgroup's tile
              const int gg = wrow / a.tq;
              const int tt = wrow - gg * a.tq;
              if (tt < n_q) {
                T* dst = static_cast<T*>(a.out) + static_cast<int64_t>(tok0 + tt) * a.o_stok +
                         (head0 + gg) * a.o_shead + half * 64 + k * 8;
                *reinterpret_cast<uint4*>(dst) = v;
              }
            }
            __syncwarp();
          }
        } else {
          T* orow = static_cast<T*>(a.out) +
                    static_cast<int64_t>(it.q_row0 + static_cast<int>(wg) * a.tq + t) * a.o_stok +
                    static_cast<int64_t>(it.h * a.group + g) * a.o_shead;
#pragma unroll
          for (int ch = 0; ch < D / 16; ++ch) {
            float o[16];
            tc05::ld_32x32b_x16(o_self + ch * 16, o);
            tc05::wait_ld();
            if (valid) {
#pragma unroll
              for (int c = 0; c < 16; ++c) orow[ch * 16 + c] = from_f32<T>(o[c] * inv);
            }
          }
        }
      }
      tc05::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc05::mbar_arrive(&bars[kBarOEmpty + wg]);
      c_tile += n_kv;
      kv_it += it.n_kv_all;
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

// Host side: the plan kernel counts items in pairs of query tiles (launch_prefill_plan with
// tq = 2 * TQ; PrefillArgs.tq stays TQ), max_work = num_tokens / (2 * TQ) + num_seqs.
template <typename T, int D, uint32_t kPolyMask>
static cudaError_t launch_prefill_q2_t(const CUtensorMap& qm, const CUtensorMap& km,
                                       const CUtensorMap& vm, const PrefillArgs& a,
                                       int max_items, int num_sms, cudaStream_t stream) {
  constexpr SmemLayout L = q2_layout<D>();
  const int smem = static_cast<int>(L.total) + 1024;
  static bool configured = false;
  auto kern = prefill_q2_kernel<T, D, kPolyMask>;
  if (!configured) {
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

template <typename T, int D>
static cudaError_t launch_prefill_q2_mode(int poly_mode, const CUtensorMap& qm,
                                          const CUtensorMap& km, const CUtensorMap& vm,
                                          const PrefillArgs& a, int max_items, int num_sms,
                                          cudaStream_t stream) {
  switch (poly_mode) {
    case 0: return launch_prefill_q2_t<T, D, 0x00u>(qm, km, vm, a, max_items, num_sms, stream);
    case 2: return launch_prefill_q2_t<T, D, 0xAAu>(qm, km, vm, a, max_items, num_sms, stream);
    default: return launch_prefill_q2_t<T, D, 0x88u>(qm, km, vm, a, max_items, num_sms, stream);
  }
}

cudaError_t launch_prefill_q2(int dtype, int head_dim, const CUtensorMap& qm,
                              const CUtensorMap& km, const CUtensorMap& vm, const PrefillArgs& a,
                              int max_items, int num_sms, int poly_mode, cudaStream_t stream) {
  if (dtype == B200_DTYPE_BF16) {
    if (head_dim == 128)
      return launch_prefill_q2_mode<__nv_bfloat16, 128>(poly_mode, qm, km, vm, a, max_items,
                                                        num_sms, stream);
    if (head_dim == 64)
      return launch_prefill_q2_mode<__nv_bfloat16, 64>(poly_mode, qm, km, vm, a, max_items,
                                                       num_sms, stream);
  } else if (dtype == B200_DTYPE_F16) {
    if (head_dim == 128)
      return launch_prefill_q2_mode<__half, 128>(poly_mode, qm, km, vm, a, max_items, num_sms,
                                                 stream);
    if (head_dim == 64)
      return launch_prefill_q2_mode<__half, 64>(poly_mode, qm, km, vm, a, max_items, num_sms,
                                                stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace b200
