// Paged attention kernels for sm_100a.
//
//  * plan_kernel        -- split plan for decode: per-sequence split counts (block-wide prefix sum),
//                          work list, merge counters reset, zero output for empty contexts.
//  * decode_tc_kernel   -- K1: bf16/f16 decode through block tables.  Persistent CTAs pull
//                          (sequence, split, kv head) items from an atomic counter; each of the 4
//                          warps streams its share of the split's 16-token units through its own
//                          TMA -> shared-memory ring (128B swizzle, mbarrier completion), computes
//                          S^T = K.Q^T and O^T += V^T.P^T with mma.sync m16n8k16 (tokens in M,
//                          the GQA heads in N, P transposed in registers by movmatrix), keeps an
//                          online softmax, merges its warps in shared memory and, for split
//                          sequences, the last CTA of a (sequence, kv head) merges the partials
//                          (atomic counter, no spin-waits).
//  * row_attn_kernel    -- CUDA-core path, one CTA of 4-16 warps per (query row, kv head, head
//                          chunk): fp32 caches, and shapes outside the tensor-core tile rules.
//                          Block-table decode or ragged causal prefill; positions in groups, the
//                          next group's K/V rows loading while the current group is computed.
//  * mask_attn_kernel   -- the reference's gather-slot + mask form (csrc/src/paged_kernels.cpp:
//                          7-105 semantics), one CTA of 4-16 warps per (query row, kv head, head
//                          chunk): the allowed slots of each 2048-slot chunk are compacted in
//                          shared memory, then attended in groups, the next group's K/V rows
//                          loading while the current group is computed.
#include "attention.cuh"

namespace b200 {

// ============================================================================================
// Split plan
// ============================================================================================

__global__ void __launch_bounds__(1024) plan_kernel(PlanArgs a) {
  __shared__ int32_t warp_sums[32];
  __shared__ int32_t carry_s;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) carry_s = 0;
  __syncthreads();
  for (int base = 0; base < a.S; base += 1024) {
    const int s = base + tid;
    int32_t n = 0;
    bool decoded = true;
    if (s < a.S) {
      int32_t ctx = a.ctx_lens[s];
      if (ctx > a.max_ctx) {
        flag_status(a.status, B200_DEVICE_BAD_OP);
        ctx = a.max_ctx;
      }
      if (a.cu_q != nullptr && a.cu_q[s + 1] - a.cu_q[s] != 1) decoded = false;
      n = (decoded && ctx > 0) ? (ctx + a.split_tokens - 1) / a.split_tokens : 0;
    }
    // block-wide inclusive scan: warp shuffles, then one warp over the warp totals
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
    const int32_t carry = carry_s;
    const int32_t incl = v + (warp > 0 ? warp_sums[warp - 1] : 0) + carry;
    const int32_t excl = incl - n;
    if (s < a.S) {
      a.cu_splits[s] = excl;
      for (int32_t p = 0; p < n; ++p) a.work_sp[excl + p] = make_int2(s, p);
      if (n == 0 && decoded) {  // empty context: the reference writes zeros (paged_kernels.cpp:30-34)
        const int64_t row = a.cu_q ? a.cu_q[s] : (a.query_rows ? a.query_rows[s] : s);
        char* orow = static_cast<char*>(a.out) + row * a.o_srow * a.esize;
        for (int h = 0; h < a.hq; ++h)
          for (int d = 0; d < a.head_dim; ++d)
            for (int b = 0; b < a.esize; ++b) orow[(h * a.o_shead + d) * a.esize + b] = 0;
      }
    }
    __syncthreads();
    if (tid == 1023) carry_s = incl;
    __syncthreads();
  }
  if (tid == 0) {
    a.cu_splits[a.S] = carry_s;
    a.hdr->total_splits = carry_s;
    a.hdr->total_items = carry_s * a.items_per_split;
    a.hdr->next_item = 0;
  }
  for (int i = tid; i < a.S * a.items_per_split; i += 1024) a.counters[i] = 0;
}

// ============================================================================================
// K1: tensor-core decode
// ============================================================================================

template <typename T, int D, int NS>
__global__ void __launch_bounds__(kDecodeThreads, 2)
    decode_tc_kernel(const __grid_constant__ CUtensorMap kmap,
                     const __grid_constant__ CUtensorMap vmap, DecodeArgs a) {
  using Cfg = TcTile<D>;
  constexpr int NW = kDecodeWarps;
  constexpr int OSTR = D + 4;  // padded row of the merge buffer (bank-conflict free)
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_u32 - raw_u32);
  // Each warp's [8][OSTR] merge rows alias its own TMA stage region: the ring of a warp is
  // drained (every fill consumed) before it writes them, and refilled only after the merge.
  static_assert(8 * OSTR * 4 <= NS * Cfg::kStage, "merge rows must fit a warp's stage region");
  auto o_w_of = [&](int w) { return reinterpret_cast<float*>(smem + w * NS * Cfg::kStage); };
  float* m_w = reinterpret_cast<float*>(smem + NW * NS * Cfg::kStage);       // [NW][8]
  float* l_w = m_w + NW * 8;                                                 // [NW][8]
  uint64_t* bars = reinterpret_cast<uint64_t*>(l_w + NW * 8);                // [NW][NS]
  int32_t* item_s = reinterpret_cast<int32_t*>(bars + NW * NS);              // [4]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r = lane >> 2, c = lane & 3;
  const int mi = lane >> 3, rr = lane & 7;
  const int items_per_split = a.hkv * a.nchunks;

  if (tid == 0) {
    item_s[2] = 0;
    for (int i = 0; i < NW * NS; ++i) mbar_init(&bars[i], 1);
    fence_proxy_async_smem();
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
  }
  __syncthreads();

  uint32_t fill_it = 0;  // fills this warp has consumed so far (stage / phase bookkeeping)
  const uint32_t my_stage0 = base_u32 + warp * NS * Cfg::kStage;
  uint8_t* my_stage0_ptr = smem + warp * NS * Cfg::kStage;
  uint64_t* my_bars = bars + warp * NS;
  const int total_items = a.hdr->total_items;

  // per-lane ldmatrix coordinates
  const int ktok = rr + 8 * (mi & 1);
  const int kcol = mi >> 1;
  const int vtok = rr + 8 * (mi >> 1);
  const int vcol = mi & 1;

  while (true) {
    if (tid == 0) item_s[0] = atomicAdd(&a.hdr->next_item, 1);
    __syncthreads();
    const int item = item_s[0];
    if (item >= total_items || item_s[2] != 0) break;
    const int sp = item / items_per_split;
    const int rem = item - sp * items_per_split;
    const int h = rem / a.nchunks;
    const int cch = rem - h * a.nchunks;
    const int2 sp_pair = a.work_sp[sp];
    const int s = sp_pair.x, p = sp_pair.y;
    const int nsplit = a.cu_splits[s + 1] - a.cu_splits[s];
    const int ctx = min(a.ctx_lens[s], a.max_ctx);
    const int tok_begin = p * a.split_tokens;
    const int tok_end = min(ctx, tok_begin + a.split_tokens);
    const int nunits = (tok_end - tok_begin + 15) >> 4;
    const int nh = min(8, a.group - cch * 8);  // q heads of this chunk
    const int hq0 = h * a.group + cch * 8;
    const int64_t qrow = a.cu_q ? a.cu_q[s] : (a.query_rows ? a.query_rows[s] : s);
    const int32_t* bt_row = a.bt + static_cast<int64_t>(s) * a.bt_stride;
    const int n_my = nunits > warp ? (nunits - warp + NW - 1) / NW : 0;

    // ---- producer: lane 0 of each warp issues its own TMA fills --------------------------
    auto issue = [&](int j, uint32_t it) {
      const int u = warp + j * NW;
      const int tok0 = tok_begin + 16 * u;
      const int st = it % NS;
      uint64_t* bar = &my_bars[st];
      const uint32_t kdst = my_stage0 + st * Cfg::kStage;
      const uint32_t vdst = kdst + Cfg::kHalf;
      const int rows_valid = min(16, tok_end - tok0);
      const int nbox = a.bs >= 16 ? 1 : (rows_valid > 8 ? 2 : 1);
      const int box_rows = a.bs >= 16 ? 16 : 8;
      mbar_arrive_expect_tx(bar, nbox * box_rows * D * 2 * 2);
      for (int b = 0; b < nbox; ++b) {
        const int t = tok0 + b * 8;
        int32_t blk = bt_row[t / a.bs];
        if (blk < 0 || blk >= a.nb) {
          flag_status(a.status, B200_DEVICE_BAD_BLOCK);
          blk = 0;
        }
        const int32_t row = (a.layer * a.nb + blk) * a.bs + (t % a.bs);
#pragma unroll
        for (int sub = 0; sub < Cfg::kSub; ++sub) {
          const int c1 = h * Cfg::kSub + sub;
          tma_load_3d(smem + (kdst - base_u32) + sub * 2048 + b * 1024, &kmap, bar, 0, c1, row);
          tma_load_3d(smem + (vdst - base_u32) + sub * 2048 + b * 1024, &vmap, bar, 0, c1, row);
        }
      }
    };
    if (lane == 0) {
      // the stage region was last written and read through the generic proxy (merge rows,
      // V zeroing): order that before the async-proxy fills
      fence_proxy_async_smem();
      const int pre = min(NS, n_my);
      for (int j = 0; j < pre; ++j) issue(j, fill_it + j);
    }
    __syncwarp();

    // ---- Q fragments (B operand: k = head dim, n = q head) ------------------------------
    uint32_t qf[D / 16][2];
    {
      const T* q = static_cast<const T*>(a.q) + qrow * a.q_srow;
      if (r < nh) {
        const T* qh = q + static_cast<int64_t>(hq0 + r) * a.q_shead;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          qf[ks][0] = *reinterpret_cast<const uint32_t*>(qh + 16 * ks + 2 * c);
          qf[ks][1] = *reinterpret_cast<const uint32_t*>(qh + 16 * ks + 8 + 2 * c);
        }
      } else {
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) qf[ks][0] = qf[ks][1] = 0u;
      }
    }

    float acc[D / 16][4];
#pragma unroll
    for (int mt = 0; mt < D / 16; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    bool timed_out = false;
    int fail_j = 0;

    for (int j = 0; j < n_my; ++j) {
      const uint32_t it = fill_it + j;
      const int st = it % NS;
      const uint32_t ph = (it / NS) & 1u;
      const int tok0 = tok_begin + 16 * (warp + j * NW);
      if (!mbar_wait_bounded(&my_bars[st], ph)) {
        timed_out = true;
        fail_j = j;
        break;
      }
      const uint32_t kb = my_stage0 + st * Cfg::kStage;
      const uint32_t vb = kb + Cfg::kHalf;
      const int rows_valid = tok_end - tok0;
      if (rows_valid < 16) {
        // rows past the context may hold anything (including NaN bit patterns): zero V there
        uint8_t* vptr = my_stage0_ptr + st * Cfg::kStage + Cfg::kHalf;
        const int nz = (16 - rows_valid) * (D / 8);
        for (int idx = lane; idx < nz; idx += 32) {
          const int row = rows_valid + idx / (D / 8);
          const int chunk = idx % (D / 8);
          const int sub = chunk >> 3, cc = chunk & 7;
          *reinterpret_cast<uint4*>(vptr + sub * 2048 + row * 128 + ((cc ^ (row & 7)) << 4)) =
              make_uint4(0u, 0u, 0u, 0u);
        }
        __syncwarp();
      }

      // S^T = K . Q^T  (16 tokens x 8 heads)
      float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        const int sub = ks >> 2;
        const int chunk = (2 * ks + kcol) & 7;
        const uint32_t addr = kb + sub * 2048 + ktok * 128 + ((chunk ^ (ktok & 7)) << 4);
        uint32_t a0, a1, a2, a3;
        ldmatrix_x4(addr, a0, a1, a2, a3);
        MmaOp<T>::run(sc, a0, a1, a2, a3, qf[ks][0], qf[ks][1]);
      }
      float x0 = sc[0] * a.scale_log2, x1 = sc[1] * a.scale_log2;
      float x2 = sc[2] * a.scale_log2, x3 = sc[3] * a.scale_log2;
      if (tok0 + r >= tok_end) x0 = x1 = -INFINITY;
      if (tok0 + r + 8 >= tok_end) x2 = x3 = -INFINITY;
      float t0 = fmaxf(x0, x2), t1 = fmaxf(x1, x3);
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        t0 = fmaxf(t0, __shfl_xor_sync(0xffffffffu, t0, o));
        t1 = fmaxf(t1, __shfl_xor_sync(0xffffffffu, t1, o));
      }
      const float n0 = fmaxf(m0, t0), n1 = fmaxf(m1, t1);
      const float u0 = n0 == -INFINITY ? 0.f : n0;
      const float u1 = n1 == -INFINITY ? 0.f : n1;
      const float al0 = fast_exp2(m0 - u0), al1 = fast_exp2(m1 - u1);
      const float p0 = fast_exp2(x0 - u0), p1 = fast_exp2(x1 - u1);
      const float p2 = fast_exp2(x2 - u0), p3 = fast_exp2(x3 - u1);
      l0 = l0 * al0 + p0 + p2;
      l1 = l1 * al1 + p1 + p3;
      m0 = n0;
      m1 = n1;
      if (!__all_sync(0xffffffffu, al0 == 1.f && al1 == 1.f)) {
#pragma unroll
        for (int mt = 0; mt < D / 16; ++mt) {
          acc[mt][0] *= al0;
          acc[mt][1] *= al1;
          acc[mt][2] *= al0;
          acc[mt][3] *= al1;
        }
      }
      const uint32_t pb0 = movmatrix_trans(MmaOp<T>::pack(p0, p1));
      const uint32_t pb1 = movmatrix_trans(MmaOp<T>::pack(p2, p3));

      // O^T += V^T . P^T  (D dims x 8 heads)
#pragma unroll
      for (int mt = 0; mt < D / 16; ++mt) {
        const int sub = mt >> 2;
        const int chunk = (2 * mt + vcol) & 7;
        const uint32_t addr = vb + sub * 2048 + vtok * 128 + ((chunk ^ (vtok & 7)) << 4);
        uint32_t a0, a1, a2, a3;
        ldmatrix_x4_trans(addr, a0, a1, a2, a3);
        MmaOp<T>::run(acc[mt], a0, a1, a2, a3, pb0, pb1);
      }
      __syncwarp();
      if (lane == 0 && j + NS < n_my) {
        fence_proxy_async_smem();
        issue(j + NS, it + NS);
      }
    }
    if (timed_out) {
      // The fills this warp still has in flight for this item are [fail_j, min(n_my, fail_j+NS)):
      // wait for them (bounded) so no TMA lands in shared memory after the CTA stops, then
      // make every warp leave the item loop at its next check.
      flag_status(a.status, B200_DEVICE_TIMEOUT);
      for (int j = fail_j; j < min(n_my, fail_j + NS); ++j) {
        const uint32_t it = fill_it + j;
        mbar_wait_bounded(&my_bars[it % NS], (it / NS) & 1u);
      }
      item_s[2] = 1;
    }
    fill_it += n_my;

    // ---- merge the 4 warps in shared memory ---------------------------------------------
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, o);
      l1 += __shfl_xor_sync(0xffffffffu, l1, o);
    }
    if (r == 0) {
      m_w[warp * 8 + 2 * c] = m0;
      m_w[warp * 8 + 2 * c + 1] = m1;
      l_w[warp * 8 + 2 * c] = l0;
      l_w[warp * 8 + 2 * c + 1] = l1;
    }
#pragma unroll
    for (int mt = 0; mt < D / 16; ++mt) {
      const int d0 = 16 * mt + r;
      float* ow = o_w_of(warp);
      ow[(2 * c) * OSTR + d0] = acc[mt][0];
      ow[(2 * c + 1) * OSTR + d0] = acc[mt][1];
      ow[(2 * c) * OSTR + d0 + 8] = acc[mt][2];
      ow[(2 * c + 1) * OSTR + d0 + 8] = acc[mt][3];
    }
    __syncthreads();

    const int pidx = (a.cu_splits[s] + p) * items_per_split + h * a.nchunks + cch;
    for (int idx = tid; idx < nh * D; idx += kDecodeThreads) {
      const int hh = idx / D, d = idx - hh * D;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < NW; ++w) M = fmaxf(M, m_w[w * 8 + hh]);
      const float Mu = M == -INFINITY ? 0.f : M;
      float o = 0.f, L = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        const float wt = fast_exp2(m_w[w * 8 + hh] - Mu);
        o += wt * o_w_of(w)[hh * OSTR + d];
        L += wt * l_w[w * 8 + hh];
      }
      const float val = L > 0.f ? o / L : 0.f;
      if (nsplit == 1) {
        T* orow = static_cast<T*>(a.out) + qrow * a.o_srow + (hq0 + hh) * a.o_shead;
        orow[d] = from_f32<T>(val);
      } else {
        a.part_o[(static_cast<int64_t>(pidx) * a.hpc + hh) * D + d] = val;
        if (d == 0) a.part_lse[pidx * a.hpc + hh] = L > 0.f ? M + __log2f(L) : -INFINITY;
      }
    }

    if (nsplit > 1) {
      __threadfence();
      __syncthreads();
      const int cidx = s * items_per_split + h * a.nchunks + cch;
      if (tid == 0) item_s[1] = (atomicAdd(&a.counters[cidx], 1) == nsplit - 1) ? 1 : 0;
      __syncthreads();
      if (item_s[1]) {
        __threadfence();
        const int pbase = a.cu_splits[s] * items_per_split + h * a.nchunks + cch;
        for (int idx = tid; idx < nh * D; idx += kDecodeThreads) {
          const int hh = idx / D, d = idx - hh * D;
          float M = -INFINITY;
          for (int q = 0; q < nsplit; ++q)
            M = fmaxf(M, __ldcg(&a.part_lse[(pbase + q * items_per_split) * a.hpc + hh]));
          const float Mu = M == -INFINITY ? 0.f : M;
          float o = 0.f, W = 0.f;
          for (int q = 0; q < nsplit; ++q) {
            const int pi = pbase + q * items_per_split;
            const float wt = fast_exp2(__ldcg(&a.part_lse[pi * a.hpc + hh]) - Mu);
            o += wt * __ldcg(&a.part_o[(static_cast<int64_t>(pi) * a.hpc + hh) * D + d]);
            W += wt;
          }
          T* orow = static_cast<T*>(a.out) + qrow * a.o_srow + (hq0 + hh) * a.o_shead;
          orow[d] = from_f32<T>(W > 0.f ? o / W : 0.f);
        }
        if (tid == 0) a.counters[cidx] = 0;
      }
    }
    __syncthreads();
  }
}

// ============================================================================================
// CUDA-core row kernel (fp32 exactness path and shapes outside the tensor-core rules)
// ============================================================================================

constexpr int kRowPassBlocks = 256;  // block ids of a row staged in shared memory per pass

// One CTA of NW warps per (query row, kv head, head chunk).  The row's context positions are
// taken in groups of U consecutive positions per warp: a group's block ids and K/V rows are loaded
// together, its U dot products reduced together, and the next group's loads are issued before the
// current group is computed (the same schedule as mask_attn_kernel below).
template <typename T, int NPL, int U, int NW>
__global__ void __launch_bounds__(NW * 32) row_attn_kernel(RowArgs a) {
  constexpr int kThreads = NW * 32;
  extern __shared__ float rsm[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row = blockIdx.x;
  const int h = blockIdx.y / a.nchunks;
  const int cch = blockIdx.y - h * a.nchunks;
  const int nh = min(8, a.group - cch * 8);
  const int hq0 = h * a.group + cch * 8;
  const int D = a.head_dim;
  float* o_w = rsm;                      // [NW][8][D]
  float* m_w = o_w + NW * 8 * D;         // [NW][8]
  float* l_w = m_w + NW * 8;             // [NW][8]

  // Which context does this query row attend?
  int64_t qrow = row;
  int32_t pos = 0, seq = 0;
  if (a.cu_q == nullptr) {
    seq = row;
    qrow = a.query_rows ? a.query_rows[row] : row;
    pos = a.ctx_lens[seq] - 1;
  } else {
    int lo = 0, hi = a.S - 1;  // last s with cu_q[s] <= row
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (a.cu_q[mid] <= row) lo = mid; else hi = mid - 1;
    }
    seq = lo;
    const int32_t count = static_cast<int32_t>(a.cu_q[seq + 1] - a.cu_q[seq]);
    pos = a.ctx_lens[seq] - count + static_cast<int32_t>(row - a.cu_q[seq]);
  }
  const int32_t n_ctx = pos + 1;
  const int32_t* bt_row = a.bt + static_cast<int64_t>(seq) * a.bt_stride;

  float q[8][NPL];
  float acc[8][NPL];
  float m[8], l[8];
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
      const int d = lane + 32 * i;
      acc[g][i] = 0.f;
      q[g][i] = 0.f;
      if (g < nh && d < D) {
        const T* qp = static_cast<const T*>(a.q) + qrow * a.q_srow +
                      static_cast<int64_t>(hq0 + g) * a.q_shead;
        q[g][i] = to_f32<T>(qp[d]);
      }
    }
  }

  const int64_t row_elems = static_cast<int64_t>(a.hkv) * D;
  const int64_t layer_base = static_cast<int64_t>(a.layer) * a.nb * a.bs * row_elems;
  // The row's block ids, kRowPassBlocks per pass, are staged in shared memory first, so a group's
  // K/V addresses need no global load.  K/V rows of positions [c0, c0 + U) of the pass that starts
  // at p0 and ends at pend (positions at or past pend are skipped; a block id outside the pool
  // sets a status bit and skips the position):
  __shared__ int32_t blk_s[kRowPassBlocks];
  int p0 = 0, pend = 0;
  auto load_group = [&](int c0, float (&kv)[U][NPL], float (&vv)[U][NPL], bool (&ok)[U]) {
    // one division per group: the block index and offset of c0, then stepped position by position
    int bi = (c0 - p0) / a.bs;
    int off = (c0 - p0) - bi * a.bs;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int cpos = c0 + u;
      const int32_t blk = cpos < pend ? blk_s[bi] : 0;
      ok[u] = cpos < pend && blk >= 0 && blk < a.nb;
      if (cpos < pend && !ok[u] && lane == 0) flag_status(a.status, B200_DEVICE_BAD_BLOCK);
      const int64_t slot = ok[u] ? static_cast<int64_t>(blk) * a.bs + off : 0;
      if (++off == a.bs) {
        off = 0;
        ++bi;
      }
      const T* kp = static_cast<const T*>(a.kc) + layer_base + slot * row_elems + h * D;
      const T* vp = static_cast<const T*>(a.vc) + layer_base + slot * row_elems + h * D;
#pragma unroll
      for (int i = 0; i < NPL; ++i) {
        const int d = lane + 32 * i;
        kv[u][i] = ok[u] && d < D ? to_f32<T>(kp[d]) : 0.f;
        vv[u][i] = ok[u] && d < D ? to_f32<T>(vp[d]) : 0.f;
      }
    }
  };
  const int pass_pos = kRowPassBlocks * a.bs;
  for (p0 = 0; p0 < n_ctx; p0 += pass_pos) {
    pend = min(n_ctx, p0 + pass_pos);
    {
      const int b0 = p0 / a.bs, nblk = (pend - p0 + a.bs - 1) / a.bs;
      for (int b = tid; b < nblk; b += kThreads) blk_s[b] = bt_row[b0 + b];
    }
    __syncthreads();
    float kv[U][NPL], vv[U][NPL];
    bool ok[U];
    load_group(p0 + warp * U, kv, vv, ok);
    for (int c0 = p0 + warp * U; c0 < pend; c0 += NW * U) {
      float kv2[U][NPL], vv2[U][NPL];
      bool ok2[U];
      load_group(c0 + NW * U, kv2, vv2, ok2);
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        if (g >= nh) break;
        float sv[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          float part = 0.f;
#pragma unroll
          for (int i = 0; i < NPL; ++i) part = fmaf(q[g][i], kv[u][i], part);
          sv[u] = part;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
          for (int u = 0; u < U; ++u) sv[u] += __shfl_xor_sync(0xffffffffu, sv[u], o);
        float mx = m[g];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          sv[u] *= a.scale;
          if (ok[u]) mx = fmaxf(mx, sv[u]);
        }
        if (mx == -INFINITY) continue;  // no valid position in the group yet
        const float alpha = m[g] == -INFINITY ? 0.f : expf(m[g] - mx);
        l[g] *= alpha;
#pragma unroll
        for (int i = 0; i < NPL; ++i) acc[g][i] *= alpha;
#pragma unroll
        for (int u = 0; u < U; ++u) {
          if (!ok[u]) continue;
          const float pw = expf(sv[u] - mx);
          l[g] += pw;
#pragma unroll
          for (int i = 0; i < NPL; ++i) acc[g][i] = fmaf(pw, vv[u][i], acc[g][i]);
        }
        m[g] = mx;
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        ok[u] = ok2[u];
#pragma unroll
        for (int i = 0; i < NPL; ++i) {
          kv[u][i] = kv2[u][i];
          vv[u][i] = vv2[u][i];
        }
      }
    }
    __syncthreads();  // the next pass rewrites the staged block ids
  }

  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      m_w[warp * 8 + g] = m[g];
      l_w[warp * 8 + g] = l[g];
    }
  }
#pragma unroll
  for (int g = 0; g < 8; ++g)
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
      const int d = lane + 32 * i;
      if (d < D) o_w[(warp * 8 + g) * D + d] = acc[g][i];
    }
  __syncthreads();
  for (int idx = tid; idx < nh * D; idx += kThreads) {
    const int g = idx / D, d = idx - g * D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, m_w[w * 8 + g]);
    float o = 0.f, L = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        const float mw = m_w[w * 8 + g];
        if (mw == -INFINITY) continue;
        const float wt = expf(mw - M);
        o += wt * o_w[(w * 8 + g) * D + d];
        L += wt * l_w[w * 8 + g];
      }
    }
    T* op = static_cast<T*>(a.out) + qrow * a.o_srow + static_cast<int64_t>(hq0 + g) * a.o_shead;
    op[d] = from_f32<T>(L > 0.f ? o / L : 0.f);
  }
}

// ============================================================================================
// Gather-slot + mask form (the reference's paged_attention signature)
// ============================================================================================

constexpr int kMaskChunk = 2048;  // context positions compacted per pass

// One CTA of NW warps per (query row, kv head, head chunk).  Each pass compacts the positions of
// kMaskChunk context slots that the row's mask allows into a shared-memory list of gather slots
// (per-thread counts, block-wide prefix sum), so a masked-out position costs one byte load here
// only.  The warps then take groups of U list entries: a group's K/V rows are loaded together
// and its U dot products reduced together, and the next group's rows are loaded before the
// current group is computed, so each warp keeps two groups of loads in flight.  Per group and
// head the running max moves once: one rescale, then the U exponentials against the new max.
// NW is 16 for D <= 64, 8 for D = 128 and 4 for D = 256 (the merge buffers stay at 32 KB).
template <typename T, int NPL, int U, int NW>
__global__ void __launch_bounds__(NW * 32) mask_attn_kernel(RowArgs a) {
  constexpr int kThreads = NW * 32;
  constexpr int kPer = kMaskChunk / kThreads;
  static_assert(kPer * kThreads == kMaskChunk && kPer <= 32, "compaction split");
  extern __shared__ float rsm[];
  __shared__ int32_t list[kMaskChunk];
  __shared__ int32_t warp_tot[NW];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row = blockIdx.x;
  const int h = blockIdx.y / a.nchunks;
  const int cch = blockIdx.y - h * a.nchunks;
  const int nh = min(8, a.group - cch * 8);
  const int hq0 = h * a.group + cch * 8;
  const int D = a.head_dim;
  float* o_w = rsm;                      // [NW][8][D]
  float* m_w = o_w + NW * 8 * D;         // [NW][8]
  float* l_w = m_w + NW * 8;             // [NW][8]

  float q[8][NPL], acc[8][NPL], m[8], l[8];
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
      const int d = lane + 32 * i;
      acc[g][i] = 0.f;
      q[g][i] = 0.f;
      if (g < nh && d < D)
        q[g][i] = to_f32<T>(static_cast<const T*>(a.q)[static_cast<int64_t>(hq0 + g) * a.q_shead +
                                                       row * a.q_srow + d]);
    }
  }

  const int64_t row_elems = static_cast<int64_t>(a.hkv) * D;
  const int64_t layer_base = static_cast<int64_t>(a.layer) * a.nb * a.bs * row_elems;
  const int64_t n_slots = static_cast<int64_t>(a.nb) * a.bs;
  const uint8_t* mrow = a.mask + static_cast<int64_t>(row) * a.num_ctx;

  // K/V rows of list entries [e0, e0 + U) (entries at or past `total`, and slots outside the
  // cache, are skipped; the latter set a status bit)
  auto load_group = [&](int e0, int total, float (&kv)[U][NPL], float (&vv)[U][NPL],
                        bool (&ok)[U]) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int e = e0 + u;
      const int64_t slot = e < total ? static_cast<int64_t>(list[e]) : 0;
      ok[u] = e < total && slot >= 0 && slot < n_slots;
      if (e < total && !ok[u] && lane == 0) flag_status(a.status, B200_DEVICE_BAD_SLOT);
      const int64_t base = layer_base + (ok[u] ? slot : 0) * row_elems + h * D;
      const T* kp = static_cast<const T*>(a.kc) + base;
      const T* vp = static_cast<const T*>(a.vc) + base;
#pragma unroll
      for (int i = 0; i < NPL; ++i) {
        const int d = lane + 32 * i;
        kv[u][i] = ok[u] && d < D ? to_f32<T>(kp[d]) : 0.f;
        vv[u][i] = ok[u] && d < D ? to_f32<T>(vp[d]) : 0.f;
      }
    }
  };

  for (int c0 = 0; c0 < a.num_ctx; c0 += kMaskChunk) {
    // ---- compaction: this thread's kPer positions (their gather slots load together with the
    // mask bytes), then its offset in the pass's list
    const int p0 = c0 + tid * kPer;
    uint32_t bits = 0;
    int32_t gv[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const bool in = p0 + i < a.num_ctx;
      gv[i] = in ? a.gather[p0 + i] : 0;
      if (in && mrow[p0 + i]) bits |= 1u << i;
    }
    const int cnt = __popc(bits);
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    int off = incl - cnt, total = 0;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const int t = warp_tot[w];
      if (w < warp) off += t;
      total += t;
    }
#pragma unroll
    for (int i = 0; i < kPer; ++i)
      if ((bits >> i) & 1u) list[off++] = gv[i];
    __syncthreads();

    // ---- attention over the pass's allowed slots: group e0 computed while group e0 + NW*U loads
    float kv[U][NPL], vv[U][NPL];
    bool ok[U];
    load_group(warp * U, total, kv, vv, ok);
    for (int e0 = warp * U; e0 < total; e0 += NW * U) {
      float kv2[U][NPL], vv2[U][NPL];
      bool ok2[U];
      load_group(e0 + NW * U, total, kv2, vv2, ok2);
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        if (g >= nh) break;
        float sv[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          float part = 0.f;
#pragma unroll
          for (int i = 0; i < NPL; ++i) part = fmaf(q[g][i], kv[u][i], part);
          sv[u] = part;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
          for (int u = 0; u < U; ++u) sv[u] += __shfl_xor_sync(0xffffffffu, sv[u], o);
        float mx = m[g];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          sv[u] *= a.scale;
          if (ok[u]) mx = fmaxf(mx, sv[u]);
        }
        if (mx == -INFINITY) continue;  // no allowed slot in the group yet
        const float alpha = m[g] == -INFINITY ? 0.f : expf(m[g] - mx);
        l[g] *= alpha;
#pragma unroll
        for (int i = 0; i < NPL; ++i) acc[g][i] *= alpha;
#pragma unroll
        for (int u = 0; u < U; ++u) {
          if (!ok[u]) continue;
          const float pw = expf(sv[u] - mx);
          l[g] += pw;
#pragma unroll
          for (int i = 0; i < NPL; ++i) acc[g][i] = fmaf(pw, vv[u][i], acc[g][i]);
        }
        m[g] = mx;
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        ok[u] = ok2[u];
#pragma unroll
        for (int i = 0; i < NPL; ++i) {
          kv[u][i] = kv2[u][i];
          vv[u][i] = vv2[u][i];
        }
      }
    }
    __syncthreads();  // the next pass rewrites the list and the warp totals
  }

  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      m_w[warp * 8 + g] = m[g];
      l_w[warp * 8 + g] = l[g];
    }
  }
#pragma unroll
  for (int g = 0; g < 8; ++g)
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
      const int d = lane + 32 * i;
      if (d < D) o_w[(warp * 8 + g) * D + d] = acc[g][i];
    }
  __syncthreads();
  for (int idx = tid; idx < nh * D; idx += kThreads) {
    const int g = idx / D, d = idx - g * D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, m_w[w * 8 + g]);
    float o = 0.f, L = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        const float mw = m_w[w * 8 + g];
        if (mw == -INFINITY) continue;
        const float wt = expf(mw - M);
        o += wt * o_w[(w * 8 + g) * D + d];
        L += wt * l_w[w * 8 + g];
      }
    }
    T* op = static_cast<T*>(a.out) + static_cast<int64_t>(row) * a.o_srow +
            static_cast<int64_t>(hq0 + g) * a.o_shead;
    op[d] = from_f32<T>(L > 0.f ? o / L : 0.f);
  }
}

// ============================================================================================
// Launchers
// ============================================================================================

template <typename T, int D, int NS>
static int decode_tc_smem_bytes() {
  using Cfg = TcTile<D>;
  return 1024 + kDecodeWarps * NS * Cfg::kStage + 2 * kDecodeWarps * 8 * 4 +
         kDecodeWarps * NS * 8 + 16;
}

template <typename T, int D, int NS>
static cudaError_t launch_decode_tc_t(const CUtensorMap& km, const CUtensorMap& vm,
                                      const DecodeArgs& a, int max_items, cudaStream_t stream) {
  static int occupancy = -1;
  static int num_sms = 0;
  const int smem = decode_tc_smem_bytes<T, D, NS>();
  auto kern = decode_tc_kernel<T, D, NS>;
  if (occupancy < 0) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev);
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occupancy, kern, kDecodeThreads, smem);
    if (e != cudaSuccess) return e;
    if (occupancy < 1) occupancy = 1;
  }
  int grid = num_sms * occupancy;
  if (max_items < grid) grid = max_items;
  if (grid < 1) grid = 1;
  kern<<<grid, kDecodeThreads, smem, stream>>>(km, vm, a);
  return cudaGetLastError();
}

cudaError_t launch_plan(const PlanArgs& a, cudaStream_t stream) {
  plan_kernel<<<1, 1024, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_decode_tc(int dtype, int head_dim, const CUtensorMap& km, const CUtensorMap& vm,
                             const DecodeArgs& a, int max_items, cudaStream_t stream) {
  constexpr int NS = kDecodeStages;
  if (dtype == B200_DTYPE_BF16) {
    if (head_dim == 128) return launch_decode_tc_t<__nv_bfloat16, 128, NS>(km, vm, a, max_items, stream);
    if (head_dim == 64) return launch_decode_tc_t<__nv_bfloat16, 64, NS>(km, vm, a, max_items, stream);
  } else if (dtype == B200_DTYPE_F16) {
    if (head_dim == 128) return launch_decode_tc_t<__half, 128, NS>(km, vm, a, max_items, stream);
    if (head_dim == 64) return launch_decode_tc_t<__half, 64, NS>(km, vm, a, max_items, stream);
  }
  return cudaErrorInvalidValue;
}

template <typename T>
static cudaError_t launch_row_t(const RowArgs& a, int rows, cudaStream_t stream) {
  const dim3 grid(rows, a.hkv * a.nchunks);
  const int npl = (a.head_dim + 31) / 32;
  // NW warps: 16 / 16 / 8 / 4 for NPL 1 / 2 / 4 / 8; merge buffers (NW * 8 * D + 2 * NW * 8)
  // floats, <= 33.8 KB
  auto mask_smem = [&](int nw) { return (nw * 8 * a.head_dim + 2 * nw * 8) * 4; };
  if (a.mode == kRowMask) {
    if (npl <= 1) mask_attn_kernel<T, 1, 4, 16><<<grid, 512, mask_smem(16), stream>>>(a);
    else if (npl <= 2) mask_attn_kernel<T, 2, 4, 16><<<grid, 512, mask_smem(16), stream>>>(a);
    else if (npl <= 4) mask_attn_kernel<T, 4, 2, 8><<<grid, 256, mask_smem(8), stream>>>(a);
    else if (npl <= 8) mask_attn_kernel<T, 8, 1, 4><<<grid, 128, mask_smem(4), stream>>>(a);
    else return cudaErrorInvalidValue;
    return cudaGetLastError();
  }
  if (npl <= 1) row_attn_kernel<T, 1, 4, 16><<<grid, 512, mask_smem(16), stream>>>(a);
  else if (npl <= 2) row_attn_kernel<T, 2, 4, 16><<<grid, 512, mask_smem(16), stream>>>(a);
  else if (npl <= 4) row_attn_kernel<T, 4, 2, 8><<<grid, 256, mask_smem(8), stream>>>(a);
  else if (npl <= 8) row_attn_kernel<T, 8, 1, 4><<<grid, 128, mask_smem(4), stream>>>(a);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

cudaError_t launch_row(int dtype, const RowArgs& a, int rows, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  if (dtype == B200_DTYPE_F32) return launch_row_t<float>(a, rows, stream);
  if (dtype == B200_DTYPE_BF16) return launch_row_t<__nv_bfloat16>(a, rows, stream);
  if (dtype == B200_DTYPE_F16) return launch_row_t<__half>(a, rows, stream);
  return cudaErrorInvalidValue;
}

}  // namespace b200
