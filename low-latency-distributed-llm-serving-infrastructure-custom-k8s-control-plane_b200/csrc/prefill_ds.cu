// K3, dual-stream form: ragged causal attention on the 5th-generation tensor cores with two
// independent work streams per CTA.
//
// One work item = (sequence, tile of TQ = 128/G query tokens, KV head): 128 query rows, the G
// query heads sharing the KV head x TQ tokens (row = g*TQ + t).  The CTA runs two streams, each a
// complete pipeline of its own: stream w has its own items, its own Q tile, K and V rings, TMEM
// S/P buffer and O accumulator, its own TMA producer warp, MMA-issuing warp and softmax
// warpgroup.  The streams share only the tensor core and the SM's issue slots, so one stream's
// item transition (epilogue, next Q tile, pipeline refill) overlaps the other stream's steady
// state instead of stalling the whole CTA.
//
// Roles (384 threads, three warpgroups; setmaxnreg inside each role's branch):
//   warps 0-3 / 4-7   softmax + epilogue of stream 0 / 1 (one query row per thread, TMEM lane =
//                     row): the whole 128-column S row in registers (one TMEM wait), causal mask,
//                     online softmax with a lazily moved reference max (O and l are rescaled only
//                     when the row max grows by more than 2^8), P packed to 16-bit pairs and
//                     stored over the upper half of S; at the item's end O / l to global memory.
//   warp 8 / 10       TMA producer of stream 0 / 1: the item's Q tile, then per 128-key tile the
//                     K tile and the V tile through the block table (one 16-row box per block and
//                     64-column half).
//   warp 9 / 11       MMA issuer of stream 0 / 1 (warp 9 also owns TMEM): S = Q.K^T (M=128,
//                     N=128, K=D) into the stream's S buffer; O += P.V with P read from TMEM.
//                     S(j+1) is issued right after PV(j): tcgen05.mma executes in issue order, so
//                     PV(j) has read P(j) before S(j+1) overwrites the columns.
// TMEM (512 columns): S/P of stream w at [128w, 128w + 128) (P in the upper 64 columns, keys in
// order), O of stream w at [256 + w*D, 256 + (w+1)*D).
// Shared memory per stream: Q (D/64 x 16 KB) + kStages K tiles + kStages V tiles; one stage per
// ring at D = 128 (2 x 96 KB), two at D = 64.  A stream's K(j+1) is loaded while its softmax
// works on S(j), its V(j+1) while S(j+1) and that softmax run.
// Work: the plan kernel sorts the items by decreasing cost (KV tiles); the 2 x gridDim.x streams
// take them in snake order.  Every wait is bounded; an expired wait records B200_DEVICE_TIMEOUT
// and stops the CTA.
#include <type_traits>

#include "attention.cuh"
#include "softmax_sm100.cuh"
#include "tc05.cuh"

namespace b200 {

namespace {

constexpr int kBN = 128;
constexpr uint32_t kRegsSoftmax = 200;
constexpr uint32_t kRegsOther = 104;

template <int D>
struct DsConfig {
  static constexpr int kStages = D == 128 ? 1 : 2;  // K and V ring depth per stream
  static constexpr uint32_t QT = (D / 64) * 128 * 128;   // one 128-row query tile
  static constexpr uint32_t KT = (D / 64) * kBN * 128;   // one 128-key K or V tile
  static constexpr uint32_t kStream = QT + 2 * kStages * KT;
  static constexpr uint32_t kBars = 2 * kStream;         // barriers after both streams' buffers
  static constexpr uint32_t kTotal = kBars + 512;
};

// Barriers of stream w start at w * kBarsPerStream.
enum : int {
  kBarQFull = 0,
  kBarQEmpty,
  kBarSFull,
  kBarPFull,   // 4 arrivals (the warps of the softmax warpgroup)
  kBarPvDone,
  kBarOEmpty,  // 4 arrivals
  kBarFinal,
  kBarKFull,   // + stage
  kBarKEmpty = kBarKFull + 2,
  kBarVFull = kBarKEmpty + 2,
  kBarVEmpty = kBarVFull + 2,
  kBarsPerStream = kBarVEmpty + 2
};

__device__ __forceinline__ bool ds_wait(uint64_t* bar, uint32_t phase, volatile int* abort_flag,
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

struct DsItem {
  int s, h, q_row0, n_q, pos0, kv_end, n_kv;
};

__device__ __forceinline__ DsItem ds_decode(const PrefillArgs& a, int item) {
  DsItem it;
  const int tile = item / a.hkv;
  it.h = item - tile * a.hkv;
  const int2 w = a.work[tile];
  it.s = w.x;
  const int64_t q0 = a.cu_q[it.s];
  const int count = static_cast<int>(a.cu_q[it.s + 1] - q0);
  const int t_begin = w.y * a.tq;
  it.n_q = min(a.tq, count - t_begin);
  it.q_row0 = static_cast<int>(q0) + t_begin;
  it.pos0 = a.ctx_lens[it.s] - count + t_begin;
  it.kv_end = it.pos0 + it.n_q;
  it.n_kv = (it.kv_end + kBN - 1) / kBN;
  return it;
}

// Item of stream `w` of this CTA in traversal round `round`: the 2 x gridDim.x streams walk the
// cost-sorted work list in snake order.
__device__ __forceinline__ int ds_item(int round, int w) {
  const int n = 2 * static_cast<int>(gridDim.x);
  const int v = 2 * static_cast<int>(blockIdx.x) + w;
  return round * n + ((round & 1) ? (n - 1 - v) : v);
}

}  // namespace

// kPolyMask: bit i set = pair i of every 8 consecutive exponential pairs of a row is computed by
// exp2_poly2 on the FMA pipe instead of ex2 on the SFU.
template <typename T, int D, uint32_t kPolyMask>
__global__ void __launch_bounds__(kPrefillThreads, 1)
    prefill_ds_kernel(const __grid_constant__ CUtensorMap qmap,
                      const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap, PrefillArgs a) {
  using C = DsConfig<D>;
  constexpr int SUB = D / 64;
  constexpr int kChunks = kBN / 16;
  constexpr int NST = C::kStages;
  constexpr uint32_t kTmemCols = 512;
  constexpr uint32_t kColO = 256;
  constexpr uint32_t ab_fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  constexpr uint32_t idesc_s = tc05::idesc_f16(ab_fmt, 128, kBN, 0);
  constexpr uint32_t idesc_o = tc05::idesc_f16(ab_fmt, 128, D, 1);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base = (raw_u32 + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_u32);
  uint64_t* bars_all = reinterpret_cast<uint64_t*>(smem + C::kBars);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars_all + 2 * kBarsPerStream);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int w = 0; w < 2; ++w) {
      uint64_t* b = bars_all + w * kBarsPerStream;
      mbar_init(&b[kBarQFull], 1);
      mbar_init(&b[kBarQEmpty], 1);
      mbar_init(&b[kBarSFull], 1);
      mbar_init(&b[kBarPFull], 4);
      mbar_init(&b[kBarPvDone], 1);
      mbar_init(&b[kBarOEmpty], 4);
      mbar_init(&b[kBarFinal], 1);
      for (int st = 0; st < 2; ++st) {
        mbar_init(&b[kBarKFull + st], 1);
        mbar_init(&b[kBarKEmpty + st], 1);
        mbar_init(&b[kBarVFull + st], 1);
        mbar_init(&b[kBarVEmpty + st], 1);
      }
    }
    *abort_flag = 0;
    fence_proxy_async_smem();
  }
  if (warp == 9) {
    tc05::tmem_alloc(tmem_slot, kTmemCols);
    tc05::tmem_relinquish();
  }
  tc05::fence_before_sync();
  __syncthreads();
  tc05::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const int total = a.hdr->total_items;

  if (warp >= 8) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsOther));
    const int w = (warp - 8) >> 1;                 // warps 8, 9 -> stream 0; 10, 11 -> stream 1
    uint64_t* bars = bars_all + w * kBarsPerStream;
    uint8_t* sq = smem + w * C::kStream;           // this stream's Q tile
    uint8_t* sk = sq + C::QT;                      // K ring
    uint8_t* sv = sk + NST * C::KT;                // V ring
    const bool leader = elect_one_sync();
    if ((warp & 1) == 0) {
      // ------------------------------------------------------------------ TMA producer
      if (leader) {
        prefetch_tensormap(&qmap);
        prefetch_tensormap(&kmap);
        prefetch_tensormap(&vmap);
      }
      const int32_t layer_base = a.layer * a.nb;
      uint32_t n_items = 0, kv_it = 0;
      uint32_t k_fills = 0, v_fills = 0;  // fills issued (the drain below waits for each ring's)
      bool ok = true;
      for (int round = 0, item = ds_item(0, w); item < total && ok; item = ds_item(++round, w)) {
        const DsItem it = ds_decode(a, item);
        if (!ds_wait(&bars[kBarQEmpty], (n_items & 1u) ^ 1u, abort_flag, a.status)) break;
        if (leader) {
          // rows past the batch read the fill value, rows of the next sequence are never stored
          mbar_arrive_expect_tx(&bars[kBarQFull], C::QT);
          for (int g = 0; g < a.group; ++g)
#pragma unroll
            for (int sub = 0; sub < SUB; ++sub)
              tc05::tma_load_4d(sq + sub * 16384 + g * a.tq * 128, &qmap, &bars[kBarQFull], 0, sub,
                                it.h * a.group + g, it.q_row0);
        }
        const int32_t* bt_row = a.bt + static_cast<int64_t>(it.s) * a.bt_stride;
        // cache rows of the next tile's 16-row chunks, read one tile ahead; chunks past kv_end
        // load (masked) rows of the sequence's first block
        int fb = 0, fw = 0;
        int32_t nrow[kChunks];
        auto fetch_rows = [&](int jj) {
#pragma unroll
          for (int b = 0; b < kChunks; ++b) {
            const bool real = jj * kBN + 16 * b < it.kv_end;
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
        for (int j = 0; j < it.n_kv; ++j, ++kv_it) {
          const uint32_t st = kv_it % NST;
          const uint32_t ph = ((kv_it / NST) & 1u) ^ 1u;
          int32_t rows[kChunks];
#pragma unroll
          for (int b = 0; b < kChunks; ++b) rows[b] = nrow[b];
          if (j + 1 < it.n_kv) fetch_rows(j + 1);
          if (!ds_wait(&bars[kBarKEmpty + st], ph, abort_flag, a.status)) {
            ok = false;
            break;
          }
          ++k_fills;
          if (leader) {
            mbar_arrive_expect_tx(&bars[kBarKFull + st], C::KT);
#pragma unroll
            for (int b = 0; b < kChunks; ++b)
#pragma unroll
              for (int sub = 0; sub < SUB; ++sub)
                tma_load_3d(sk + st * C::KT + sub * (kBN * 128) + b * 2048, &kmap,
                            &bars[kBarKFull + st], 0, it.h * SUB + sub, rows[b]);
          }
          if (!ds_wait(&bars[kBarVEmpty + st], ph, abort_flag, a.status)) {
            ok = false;
            break;
          }
          ++v_fills;
          if (leader) {
            mbar_arrive_expect_tx(&bars[kBarVFull + st], C::KT);
#pragma unroll
            for (int b = 0; b < kChunks; ++b)
#pragma unroll
              for (int sub = 0; sub < SUB; ++sub)
                tma_load_3d(sv + st * C::KT + sub * (kBN * 128) + b * 2048, &vmap,
                            &bars[kBarVFull + st], 0, it.h * SUB + sub, rows[b]);
          }
        }
        ++n_items;
      }
      // every fill this warp issued has landed before the CTA retires (bounded waits)
      for (uint32_t f = k_fills > NST ? k_fills - NST : 0; f < k_fills; ++f)
        mbar_wait_bounded(&bars[kBarKFull + f % NST], (f / NST) & 1u);
      for (uint32_t f = v_fills > NST ? v_fills - NST : 0; f < v_fills; ++f)
        mbar_wait_bounded(&bars[kBarVFull + f % NST], (f / NST) & 1u);
      if (n_items > 0) mbar_wait_bounded(&bars[kBarQFull], (n_items - 1) & 1u);
    } else {
      // ------------------------------------------------------------------ MMA issuer
      uint32_t n_items = 0, kv_it = 0;
      constexpr uint32_t kHi = tc05::desc_hi_sw128(1024);
      const uint32_t q_lo = tc05::desc_lo(base + w * C::kStream, 16);
      const uint32_t k_lo0 = tc05::desc_lo(base + w * C::kStream + C::QT, 16);
      const uint32_t v_lo0 = tc05::desc_lo(base + w * C::kStream + C::QT + NST * C::KT, kBN * 128);
      const uint32_t s_t = tmem + w * kBN;
      const uint32_t p_t = s_t + 64;
      const uint32_t o_t = tmem + kColO + w * D;
      auto issue_s = [&](uint32_t stage) {
        const uint32_t k_lo = k_lo0 + stage * (C::KT >> 4);
        if (!leader) return;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t qo = static_cast<uint32_t>(((kk >> 2) * 16384 + (kk & 3) * 32) >> 4);
          const uint32_t ko = static_cast<uint32_t>(((kk >> 2) * (kBN * 128) + (kk & 3) * 32) >> 4);
          tc05::mma_f16(s_t, tc05::desc_join(q_lo + qo, kHi), tc05::desc_join(k_lo + ko, kHi),
                        idesc_s, kk > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](uint32_t stage, bool acc) {
        const uint32_t v_lo = v_lo0 + stage * (C::KT >> 4);
        if (!leader) return;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk)  // 16 keys per K step, P columns in key order
          tc05::mma_f16_ts(o_t, p_t + kk * 8, tc05::desc_join(v_lo + kk * (2048 >> 4), kHi),
                           idesc_o, (acc || kk > 0) ? 1u : 0u);
      };
      auto s_tile = [&](uint32_t f, bool last) -> bool {
        if (!ds_wait(&bars[kBarKFull + f % NST], (f / NST) & 1u, abort_flag, a.status))
          return false;
        tc05::fence_after_sync();
        issue_s(f % NST);
        if (leader) {
          tc05::commit(&bars[kBarSFull]);
          tc05::commit(&bars[kBarKEmpty + f % NST]);
          if (last) tc05::commit(&bars[kBarQEmpty]);  // the item's last S has read Q
        }
        return true;
      };
      bool ok = true;
      for (int round = 0, item = ds_item(0, w); item < total && ok; item = ds_item(++round, w)) {
        const DsItem it = ds_decode(a, item);
        if (!ds_wait(&bars[kBarQFull], n_items & 1u, abort_flag, a.status)) break;
        tc05::fence_after_sync();
        // S(0) overlaps the previous item's epilogue (it writes S/P, not O)
        if (!s_tile(kv_it, it.n_kv == 1)) break;
        // O is free once the previous epilogue has read it
        if (!ds_wait(&bars[kBarOEmpty], (n_items & 1u) ^ 1u, abort_flag, a.status)) break;
        tc05::fence_after_sync();
        for (int j = 0; j < it.n_kv; ++j) {
          const uint32_t f = kv_it + j;
          if (!ds_wait(&bars[kBarPFull], f & 1u, abort_flag, a.status) ||
              !ds_wait(&bars[kBarVFull + f % NST], (f / NST) & 1u, abort_flag, a.status)) {
            ok = false;
            break;
          }
          tc05::fence_after_sync();
          issue_pv(f % NST, j > 0);
          if (leader) {
            tc05::commit(&bars[kBarPvDone]);
            tc05::commit(&bars[kBarVEmpty + f % NST]);
          }
          if (j + 1 < it.n_kv && !s_tile(f + 1, j + 1 == it.n_kv - 1)) {
            ok = false;
            break;
          }
        }
        kv_it += it.n_kv;
        ++n_items;
      }
      // all tcgen05 work this warp issued completes before TMEM is released
      if (leader) tc05::commit(&bars[kBarFinal]);
      mbar_wait_bounded(&bars[kBarFinal], 0);
    }
    __syncwarp();
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
    // ------------------------------------------------------------------ softmax / epilogue
    const int w = warp >> 2;
    uint64_t* bars = bars_all + w * kBarsPerStream;
    uint8_t* sv = smem + w * C::kStream + C::QT + NST * C::KT;  // V ring (for the tail zeroing)
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int g = row / a.tq;
    const int t = row - g * a.tq;
    const uint32_t trow = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t s_self = trow + w * kBN;
    const uint32_t o_self = trow + kColO + w * D;
    const int sm_tid = quarter * 32 + lane;
    uint32_t kv_it = 0, n_items = 0;
    for (int round = 0, item = ds_item(0, w); item < total; item = ds_item(++round, w)) {
      const DsItem it = ds_decode(a, item);
      const bool valid = t < it.n_q;
      const int pos = valid ? it.pos0 + t : -1;
      float m = -INFINITY, l = 0.f;
      bool ok = true;
      for (int j = 0; j < it.n_kv; ++j) {
        const uint32_t f = kv_it + j;
        ok = ds_wait(&bars[kBarSFull], f & 1u, abort_flag, a.status);
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        tc05::fence_after_sync();
        const bool need_mask = __any_sync(0xffffffffu, j * kBN + kBN - 1 > pos);
        const int lim = pos - j * kBN;  // columns c > lim are in the future of this row
        float sa[32], sb[32], sc[32], sd[32];
        tc05::ld_32x32b_x32(s_self, sa);
        tc05::ld_32x32b_x32(s_self + 32, sb);
        tc05::ld_32x32b_x32(s_self + 64, sc);
        tc05::ld_32x32b_x32(s_self + 96, sd);
        tc05::wait_ld();
        auto mask_chunk = [&](float (&v)[32], int chunk) {
          if (need_mask) {
#pragma unroll
            for (int c = 0; c < 32; ++c)
              if (chunk * 32 + c > lim) v[c] = -INFINITY;
          }
        };
        mask_chunk(sa, 0);
        mask_chunk(sb, 1);
        mask_chunk(sc, 2);
        mask_chunk(sd, 3);
        float mx8[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) mx8[k] = -INFINITY;
        auto max_chunk = [&](const float (&v)[32]) {
#pragma unroll
          for (int c = 0; c < 32; c += 2)
            mx8[(c >> 1) & 7] = fmax3(mx8[(c >> 1) & 7], v[c], v[c + 1]);
        };
        max_chunk(sa);
        max_chunk(sb);
        max_chunk(sc);
        max_chunk(sd);
        const float smax = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                                 fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
        // Lazily moved reference max: the row keeps its reference m until the tile max exceeds
        // it by more than 8 (log2 units), so p stays below 2^8 and O / l are rescaled only on
        // such jumps; O and l always share the same m, so O / l is exact whichever m was used.
        const float tmax = smax * a.scale_log2;  // scale > 0: max commutes with scaling
        float alpha = 1.f;
        if (m == -INFINITY) {
          m = tmax;
        } else if (tmax > m + 8.f) {
          alpha = fast_exp2(m - tmax);
          m = tmax;
        }
        const float mu = m == -INFINITY ? 0.f : m;
        // p = 2^(s*scale - m) for pairs of keys: the argument by one packed FMA, the exponential
        // on the SFU or (pairs selected by kPolyMask) by exp2_poly2, the row sum by packed adds
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
              const uint64_t arg =
                  f2_fma(f2_pack(x[16 * hh + c], x[16 * hh + c + 1]), scale2, negmu2);
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
        exp_chunk(sa, 0);
        exp_chunk(sb, 1);
        exp_chunk(sc, 2);
        exp_chunk(sd, 3);
        float rsl[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) f2_unpack(rs2[k], rsl[2 * k], rsl[2 * k + 1]);
        const float rs = ((rsl[0] + rsl[1]) + (rsl[2] + rsl[3])) +
                         ((rsl[4] + rsl[5]) + (rsl[6] + rsl[7]));
        l = l * alpha + rs;
        // O rescale: PV(j-1), the last MMA into O, was issued before S(j) and is covered by the
        // commit that signalled S(j), so O can be read and written here
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
        if (j == it.n_kv - 1 && it.kv_end < j * kBN + kBN) {
          // keys past kv_end are masked for every row (P = 0), but their V rows may hold
          // anything, and 0 * NaN is not 0: zero them once the V tile has landed
          ok = ds_wait(&bars[kBarVFull + f % NST], (f / NST) & 1u, abort_flag, a.status);
          if (!__all_sync(0xffffffffu, ok)) {
            ok = false;
            break;
          }
          uint8_t* vst = sv + (f % NST) * C::KT;
          const int r0 = it.kv_end - j * kBN;
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
        if (lane == 0) tc05::mbar_arrive(&bars[kBarPFull]);
      }
      if (!ok) break;
      // ---- epilogue: wait for the item's last PV, then O / l (all of O in one TMEM wait)
      ok = ds_wait(&bars[kBarPvDone], (kv_it + it.n_kv - 1) & 1u, abort_flag, a.status);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc05::fence_after_sync();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      T* orow = static_cast<T*>(a.out) + static_cast<int64_t>(it.q_row0 + t) * a.o_stok +
                static_cast<int64_t>(it.h * a.group + g) * a.o_shead;
#pragma unroll
      for (int half = 0; half < D / 64; ++half) {
        float oa[32], ob[32];
        tc05::ld_32x32b_x32(o_self + half * 64, oa);
        tc05::ld_32x32b_x32(o_self + half * 64 + 32, ob);
        tc05::wait_ld();
        if (valid) {
          auto put = [&](const float (&o)[32], int c0) {
            if (a.vec_out) {
#pragma unroll
              for (int c8 = 0; c8 < 4; ++c8) {
                uint4 v;
                v.x = MmaOp<T>::pack(o[c8 * 8 + 0] * inv, o[c8 * 8 + 1] * inv);
                v.y = MmaOp<T>::pack(o[c8 * 8 + 2] * inv, o[c8 * 8 + 3] * inv);
                v.z = MmaOp<T>::pack(o[c8 * 8 + 4] * inv, o[c8 * 8 + 5] * inv);
                v.w = MmaOp<T>::pack(o[c8 * 8 + 6] * inv, o[c8 * 8 + 7] * inv);
                *reinterpret_cast<uint4*>(orow + c0 + c8 * 8) = v;
              }
            } else {
#pragma unroll
              for (int c = 0; c < 32; ++c) orow[c0 + c] = from_f32<T>(o[c] * inv);
            }
          };
          put(oa, half * 64);
          put(ob, half * 64 + 32);
        }
      }
      tc05::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc05::mbar_arrive(&bars[kBarOEmpty]);
      kv_it += it.n_kv;
      ++n_items;
    }
  }

  tc05::fence_before_sync();
  __syncthreads();
  if (warp == 9) {
    tc05::fence_after_sync();
    tc05::tmem_dealloc(tmem, kTmemCols);
  }
}

template <typename T, int D, uint32_t kPolyMask>
static cudaError_t launch_prefill_ds_t(const CUtensorMap& qm, const CUtensorMap& km,
                                       const CUtensorMap& vm, const PrefillArgs& a,
                                       int max_items, int num_sms, cudaStream_t stream) {
  const int smem = static_cast<int>(DsConfig<D>::kTotal) + 1024;
  static bool configured = false;
  auto kern = prefill_ds_kernel<T, D, kPolyMask>;
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
  // two streams per CTA: enough CTAs for every item to have a stream, at most one per SM
  int grid = num_sms;
  const int need = (max_items + 1) / 2;
  if (need < grid) grid = need;
  if (grid < 1) grid = 1;
  kern<<<grid, kPrefillThreads, smem, stream>>>(qm, km, vm, a);
  return cudaGetLastError();
}

template <typename T, int D>
static cudaError_t launch_prefill_ds_mode(int poly_mode, const CUtensorMap& qm,
                                          const CUtensorMap& km, const CUtensorMap& vm,
                                          const PrefillArgs& a, int max_items, int num_sms,
                                          cudaStream_t stream) {
  switch (poly_mode) {
    case 0: return launch_prefill_ds_t<T, D, 0x00u>(qm, km, vm, a, max_items, num_sms, stream);
    case 2: return launch_prefill_ds_t<T, D, 0xAAu>(qm, km, vm, a, max_items, num_sms, stream);
    default: return launch_prefill_ds_t<T, D, 0x88u>(qm, km, vm, a, max_items, num_sms, stream);
  }
}

cudaError_t launch_prefill_ds(int dtype, int head_dim, const CUtensorMap& qm,
                              const CUtensorMap& km, const CUtensorMap& vm, const PrefillArgs& a,
                              int max_items, int num_sms, int poly_mode, cudaStream_t stream) {
  if (dtype == B200_DTYPE_BF16) {
    if (head_dim == 128)
      return launch_prefill_ds_mode<__nv_bfloat16, 128>(poly_mode, qm, km, vm, a, max_items,
                                                        num_sms, stream);
    if (head_dim == 64)
      return launch_prefill_ds_mode<__nv_bfloat16, 64>(poly_mode, qm, km, vm, a, max_items,
                                                       num_sms, stream);
  } else if (dtype == B200_DTYPE_F16) {
    if (head_dim == 128)
      return launch_prefill_ds_mode<__half, 128>(poly_mode, qm, km, vm, a, max_items, num_sms,
                                                 stream);
    if (head_dim == 64)
      return launch_prefill_ds_mode<__half, 64>(poly_mode, qm, km, vm, a, max_items, num_sms,
                                                stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace b200
