// attn_bwd.cu -- GQA flash-attention backward for sm_100a (tcgen05 + TMEM + TMA).
//
// Replaces k_gqa_flash_attn_tc_bwd<HEAD_DIM> (src/tkm_gpu.cu:440-598 of the
// reference): same inputs (packed QKV, O, dO, LSE) and math
// (Delta = rowsum(O*dO), P = exp(s*scale - LSE), dS = P*(dP - Delta)),
// with the true dK = scale * dS^T Q and dV = P^T dO summed over the query
// heads of each kv head (the reference writes dK := dQ, dV := dO at
// src/tkm_gpu.cu:588-596) and a correctly laid-out dQ = scale * dS K.
//
// Two kernels, no atomics, deterministic (three with a dS workspace, below):
//  * attn_bwd_dkdv_kernel: one CTA per 128-key tile of a (batch, kv head);
//    K, V and the dK, dV accumulators stay resident while the CTA walks every
//    (query head of the group, 128-row query tile) pair that sees the keys.
//    Four MMAs per step, all M = 128 keys: S^T = K Q^T, dP^T = V dO^T,
//    dV += P^T dO and dK += dS^T Q (P^T and dS^T read straight from TMEM).
//  * attn_bwd_dq_kernel: one CTA per 128-row query tile of a (batch, q head),
//    Q, dO and the dQ accumulator resident, K/V blocks streamed.  Three MMAs
//    per block, M = 128 queries: S = Q K^T, dP = dO V^T, dQ += dS K (dS from
//    TMEM).
//  * with a dS workspace the dK/dV kernel also stores dS (16-bit, 32 KB per
//    128x128 tile) and attn_bwd_dsk_kernel computes dQ = scale * dS K as a
//    plain tcgen05 GEMM over the stored tiles, in place of the dQ kernel and
//    its recomputation of S, P and dP.  A tile is kept in the MMA's
//    no-swizzle core-matrix order (see ds_tile), so that each warp store
//    writes whole 128-byte lines and the GEMM fetches a tile with one bulk copy.
// In both kernels warps 0-7 are two compute warpgroups (one thread per TMEM
// lane/row, each group owning half of the 128 columns), warp 8 issues TMA,
// warp 9 issues tcgen05.mma.  The MMA order lets the next step's S/dP MMAs
// run while the compute warps still work on the current step.
#include "tkb_common.cuh"
#include "tkb_internal.h"

// Groups of four exponentials (of 16 per thread and step) that the dK/dV
// kernel computes with the FMA-pipe polynomial instead of ex2.  Same-box
// A/B at the headline shape: 2 and 4 groups within noise of none (backward
// 1.664-1.677 vs 1.650-1.671 ms), 8 groups slower (1.689-1.694); off.
#ifndef TKB_BWD_EMU
#define TKB_BWD_EMU 0
#endif

namespace tkb {

TKB_DEVFN void wait_ld_dep32(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
                 "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),
                 "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]),
                 "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]),
                 "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// Packed 16-bit column in TMEM of K-step kk (16 rows of the reduction dim) when
// compute warpgroup 0 stores its half at columns [0,32) and group 1 at [64,96).
TKB_DEVFN uint32_t half_split_col(int kk) { return kk < 4 ? kk * 8 : 64 + (kk - 4) * 8; }

// Index of the dS tile (query tile i, key tile j) within one (batch, q head):
// causal rows hold only j <= i (lower triangle, row-major), else all nq tiles.
// Inside a tile, dS[q][k] (16-bit) sits at byte (k / 8) * 2048 + (q / 8) * 128
// + (k % 8) * 16 + (q % 8) * 2: core matrices of 8 queries x 8 keys (128
// bytes), 16 consecutive ones along the queries per group of 8 keys.
TKB_DEVFN long long ds_tile(int i, int j, int nq, bool causal) {
  return causal ? static_cast<long long>(i) * (i + 1) / 2 + j : static_cast<long long>(i) * nq + j;
}

// CTA -> (key tile jt, batch x kv head bg), longest first.  At D = 128 the
// heads go in groups of four, longest first inside a group: the CTAs that run
// at the same time then walk the Q and dO tiles of a few heads, which stay in
// L2, instead of those of up to 148 different heads (2.07 -> 1.85 ms per
// backward at B=8, H=16, S=4096; groups of 2, 4 and 8 measured alike).  At
// D = 64 the plain longest-first order over all heads is kept: grouping gave
// nothing there.
template <int D>
TKB_DEVFN void dkv_cta_order(int cta, int BG, int nkt, int& jt, int& bg) {
  constexpr int HG = 4;
  if (D != 128) {
    jt = cta / BG;
    bg = cta % BG;
    return;
  }
  const int full = BG / HG, per = HG * nkt;
  if (cta < full * per) {
    const int r = cta % per;
    jt = r / HG;
    bg = (cta / per) * HG + r % HG;
  } else {
    const int hr = BG - full * HG, r = cta - full * per;
    jt = r / hr;
    bg = full * HG + r % hr;
  }
}

// ============================================================================ dK / dV
template <int D>
struct DkvCfg {
  static constexpr int TILE = 128 * D * 2;
  static constexpr int SLAB = 128 * 128;
  // D = 64 leaves room for two S^T buffers in TMEM and four Q/dO stages: the
  // next step's S^T is computed while this step's P^T still feeds dV, so the
  // exponentials of consecutive steps follow each other without waiting on
  // the tensor pipe.  D = 128 has neither (512 TMEM columns, 227 KB).
  static constexpr bool DBL = (D == 64);
  static constexpr int NSTQ = DBL ? 4 : 2;
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + TILE;
  static constexpr int OFF_Q = OFF_V + TILE;
  static constexpr int OFF_DO = OFF_Q + NSTQ * TILE;
  static constexpr int OFF_LSE = OFF_DO + NSTQ * TILE;  // NSTQ x 128 floats
  static constexpr int OFF_DEL = OFF_LSE + NSTQ * 512;
  static constexpr int OFF_BAR = OFF_DEL + NSTQ * 512;
  // kv_full, q_full[NSTQ], q_empty[NSTQ], st_full[2], dp_full, p_ready[2], ds_ready, kv_done, drain
  static constexpr int NBAR = 1 + 2 * NSTQ + 8;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int SMEM = OFF_MISC + 16 + 1024;
  static constexpr uint32_t TM_DP = 128, TM_DK = 256, TM_DV = 256 + D;
  // S^T buffer of step it (the second one at D = 64 only)
  static TKB_DEVFN uint32_t tm_st(int it) { return (DBL && (it & 1)) ? 384u : 0u; }
};

template <int D, bool BF16>
__global__ void __launch_bounds__(320, 1) attn_bwd_dkdv_kernel(const __grid_constant__ BwdParams p) {
  using C = DkvCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* kv_full = bars;
  uint64_t* q_full = bars + 1;
  uint64_t* q_empty = q_full + C::NSTQ;
  uint64_t* st_full = q_empty + C::NSTQ;  // [S^T buffer]
  uint64_t* dp_full = st_full + 2;
  uint64_t* p_ready = dp_full + 1;  // [half]: P^T of queries 0-31 / 32-63 of each compute warpgroup
  uint64_t* ds_ready = p_ready + 2;
  uint64_t* kv_done = ds_ready + 1;
  uint64_t* mma_drain = kv_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);

  const int warp = warp_id(), lane = lane_id();
  const int BG = p.B * p.Hkv;
  int jt, bg;  // key tile (tile 0 sees the most queries), batch x kv head
  dkv_cta_order<D>(blockIdx.x, BG, gridDim.x / BG, jt, bg);
  const int b = bg / p.Hkv, g = bg % p.Hkv;
  const int G = p.Hq / p.Hkv;
  const int nq = p.S_pad >> 7;
  const int i0 = p.causal ? jt : 0;
  const int n_i = nq - i0;
  const int n_steps = G * n_i;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < C::NSTQ; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], 1);
    }
    mbar_init(&st_full[0], 1);
    mbar_init(&st_full[1], 1);
    mbar_init(dp_full, 1);
    mbar_init(&p_ready[0], 256);
    mbar_init(&p_ready[1], 256);
    mbar_init(ds_ready, 256);
    mbar_init(kv_done, 1);
    mbar_init(mma_drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      prefetch_tmap(&p.tmQ);
      prefetch_tmap(&p.tmK);
      prefetch_tmap(&p.tmV);
      prefetch_tmap(&p.tmdO);
      const uint64_t pol_kv = policy_evict_first(), pol_q = policy_evict_last();
      mbar_arrive_expect_tx(kv_full, 2 * C::TILE);
#pragma unroll
      for (int hh = 0; hh < D / 64; ++hh) {
        tma_load_3d(smem + C::OFF_K + hh * C::SLAB, &p.tmK, kv_full, g * D + hh * 64, jt * 128, b, pol_kv);
        tma_load_3d(smem + C::OFF_V + hh * C::SLAB, &p.tmV, kv_full, g * D + hh * 64, jt * 128, b, pol_kv);
      }
      int issued = 0;
      for (int it = 0; it < n_steps; ++it) {
        const int s = it % C::NSTQ;
        const uint32_t ph = (it / C::NSTQ) & 1;
        const int hq = g * G + it / n_i, i = i0 + it % n_i;
        if (!mbar_wait(&q_empty[s], ph ^ 1, abort_flag)) break;
        mbar_arrive_expect_tx(&q_full[s], 2 * C::TILE + 1024);
#pragma unroll
        for (int hh = 0; hh < D / 64; ++hh) {
          tma_load_3d(smem + C::OFF_Q + s * C::TILE + hh * C::SLAB, &p.tmQ, &q_full[s], hq * D + hh * 64,
                      i * 128, b, pol_q);
          tma_load_3d(smem + C::OFF_DO + s * C::TILE + hh * C::SLAB, &p.tmdO, &q_full[s], hq * D + hh * 64,
                      i * 128, b, pol_q);
        }
        const long long ro = (static_cast<long long>(b) * p.Hq + hq) * p.S_pad + i * 128;
        bulk_load(smem + C::OFF_LSE + s * 512, p.nlse2 + ro, 512, &q_full[s]);
        bulk_load(smem + C::OFF_DEL + s * 512, p.delta + ro, 512, &q_full[s]);
        issued = it + 1;
      }
      if (*abort_flag) {
        volatile int never = 0;
        mbar_wait(kv_full, 0, &never);
        for (int it = max(0, issued - C::NSTQ); it < issued; ++it)
          mbar_wait(&q_full[it % C::NSTQ], (it / C::NSTQ) & 1, &never);
      }
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = idesc_f16kind(128, 128, BF16, false, false);  // S^T, dP^T
      constexpr uint32_t idKV = idesc_f16kind(128, D, BF16, false, true);    // dV, dK (A in TMEM)
      const uint32_t sK = sbase + C::OFF_K, sV = sbase + C::OFF_V;
      auto sQ = [&](int s) { return sbase + C::OFF_Q + s * C::TILE; };
      auto sO = [&](int s) { return sbase + C::OFF_DO + s * C::TILE; };
      auto issue_nt = [&](uint32_t d, uint32_t a, uint32_t bm) {  // D(128x128) = A(128xD) B(128xD)^T
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * C::SLAB + (kk & 3) * 32;
          umma_ss(d, sdesc_sw128(a + off, 16, 1024), sdesc_sw128(bm + off, 16, 1024), idS, kk > 0 ? 1u : 0u);
        }
      };
      auto issue_acc = [&](uint32_t d, uint32_t a_tm, uint32_t bm, bool acc) {  // D += A(tmem) B(smem, MN-major)
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_ts(d, a_tm + half_split_col(kk), sdesc_sw128(bm + kk * 2048, C::SLAB, 1024), idKV,
                  (acc || kk > 0) ? 1u : 0u);
      };
      // the same over the K-steps of one half of each warpgroup's queries:
      // half 0 = K-steps 0, 1 (group 0) and 4, 5 (group 1), half 1 = the rest
      auto issue_acc_half = [&](uint32_t d, uint32_t a_tm, uint32_t bm, bool acc, int half) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int kk = (i >> 1) * 4 + half * 2 + (i & 1);
          umma_ts(d, a_tm + half_split_col(kk), sdesc_sw128(bm + kk * 2048, C::SLAB, 1024), idKV,
                  (acc || i > 0) ? 1u : 0u);
        }
      };
      // S^T of step n into its buffer; st_full[buffer] completes once per use
      auto issue_st = [&](int n) {
        issue_nt(tmem + C::tm_st(n), sK, sQ(n % C::NSTQ));
        umma_commit(&st_full[C::DBL ? (n & 1) : 0]);
      };
      bool ok = mbar_wait(kv_full, 0, abort_flag) && mbar_wait(&q_full[0], 0, abort_flag);
      if (ok) {
        tc_fence_after();
        issue_st(0);
        issue_nt(tmem + C::TM_DP, sV, sO(0));
        umma_commit(dp_full);
        if (C::DBL && n_steps > 1) {
          if ((ok = mbar_wait(&q_full[1 % C::NSTQ], 0, abort_flag))) {
            tc_fence_after();
            issue_st(1);
          }
        }
      }
      for (int it = 0; ok && it < n_steps; ++it) {
        const int s = it % C::NSTQ, s1 = (it + 1) % C::NSTQ;
        const bool more = it + 1 < n_steps;
        // dV += P^T dO, in two halves as the compute warps publish P^T
        if (!(ok = mbar_wait(&p_ready[0], it & 1, abort_flag))) break;
        tc_fence_after();
        issue_acc_half(tmem + C::TM_DV, tmem + C::tm_st(it), sO(s), it > 0, 0);
        if (!(ok = mbar_wait(&p_ready[1], it & 1, abort_flag))) break;
        tc_fence_after();
        issue_acc_half(tmem + C::TM_DV, tmem + C::tm_st(it), sO(s), true, 1);
        // the S^T MMA that reuses this buffer (step it + 2 with two buffers,
        // it + 1 with one) follows the dV MMA that reads P^T from it
        const int nxt = C::DBL ? it + 2 : it + 1;
        if (nxt < n_steps) {
          const int sn = nxt % C::NSTQ;
          if (!(ok = mbar_wait(&q_full[sn], (nxt / C::NSTQ) & 1, abort_flag))) break;
          tc_fence_after();
          issue_st(nxt);
        }
        if (!(ok = mbar_wait(ds_ready, it & 1, abort_flag))) break;
        tc_fence_after();
        issue_acc(tmem + C::TM_DK, tmem + C::TM_DP, sQ(s), it > 0);           // dK += dS^T Q
        umma_commit(&q_empty[s]);
        if (more) {
          issue_nt(tmem + C::TM_DP, sV, sO(s1));                              // dP^T for the next step
          umma_commit(dp_full);
        }
      }
      if (ok) umma_commit(kv_done);
      else {
        volatile int never = 0;
        umma_commit(mma_drain);
        mbar_wait(mma_drain, 0, &never);
      }
    }
  } else {
    // ---------------------------------------------------------------- compute warpgroups
    const int w = warp >> 2;              // which half of the 128 query columns
    const int kr = threadIdx.x & 127;     // key row = TMEM lane
    const int key = jt * 128 + kr;
    const bool key_ok = key < p.S;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t cb = static_cast<uint32_t>(w * 64);
    const uint32_t tDP = tmem + lane_off + C::TM_DP + cb;
    const float sl2 = p.scale_log2;
    bool ok = true;
    for (int it = 0; it < n_steps; ++it) {
      const int s = it % C::NSTQ;
      const int i = i0 + it % n_i;
      const float4* lse4 = reinterpret_cast<const float4*>(smem + C::OFF_LSE + s * 512) + w * 16;
      const float4* del4 = reinterpret_cast<const float4*>(smem + C::OFF_DEL + s * 512) + w * 16;
      // keys above the diagonal of a diagonal tile see no query of this half below qmin
      const int qmin = (p.causal && i == jt) ? kr - w * 64 : -1;
      const uint32_t tST = tmem + lane_off + C::tm_st(it) + cb;
      if (!(ok = mbar_wait_warp(&q_full[s], (it / C::NSTQ) & 1, abort_flag))) break;
      if (!(ok = mbar_wait_warp(&st_full[C::DBL ? (it & 1) : 0], C::DBL ? ((it >> 1) & 1) : (it & 1), abort_flag)))
        break;
      tc_fence_after();
      uint32_t pk[32];
      {
        uint32_t v0[32], v1[32];
        tmem_ld32(tST, v0);
        tmem_ld32(tST + 32, v1);
        wait_ld_dep32(v0);
        wait_ld_dep32(v1);
        // masked keys (sequence tail) and the diagonal tile need the per-element test
        const bool need_mask = !key_ok || qmin > 0;
        const uint64_t sl2x2 = f2(sl2, sl2);
        // P^T of queries 0-31 of this warpgroup first (K-steps released to the
        // dV MMA while queries 32-63 are computed), then the rest
        auto exp4 = [&](int e4) {
          const float4 l = lse4[e4];  // -LSE * log2(e) of queries 4 e4 .. 4 e4 + 3
          const uint32_t* src = e4 < 8 ? &v0[e4 * 4] : &v1[(e4 - 8) * 4];
          const int q0 = e4 * 4;
          float a0, a1, a2, a3;
          f2_split(fma_f2(f2(__uint_as_float(src[0]), __uint_as_float(src[1])), sl2x2, f2(l.x, l.y)), a0, a1);
          f2_split(fma_f2(f2(__uint_as_float(src[2]), __uint_as_float(src[3])), sl2x2, f2(l.z, l.w)), a2, a3);
          if ((e4 * TKB_BWD_EMU) % 16 + TKB_BWD_EMU >= 16) {
            ex2_poly_f2(a0, a1, a0, a1);
            ex2_poly_f2(a2, a3, a2, a3);
          } else {
            a0 = ex2(a0);
            a1 = ex2(a1);
            a2 = ex2(a2);
            a3 = ex2(a3);
          }
          if (need_mask) {
            if (!key_ok || q0 < qmin) a0 = 0.f;
            if (!key_ok || q0 + 1 < qmin) a1 = 0.f;
            if (!key_ok || q0 + 2 < qmin) a2 = 0.f;
            if (!key_ok || q0 + 3 < qmin) a3 = 0.f;
          }
          pk[e4 * 2] = pack2<BF16>(a0, a1);
          pk[e4 * 2 + 1] = pack2<BF16>(a2, a3);
        };
#pragma unroll
        for (int e4 = 0; e4 < 8; ++e4) exp4(e4);
        tmem_st16(tST, pk);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_ready[0]);
#pragma unroll
        for (int e4 = 8; e4 < 16; ++e4) exp4(e4);
        tmem_st16(tST + 16, pk + 16);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_ready[1]);
      }

      if (!(ok = mbar_wait_warp(dp_full, it & 1, abort_flag))) break;
      tc_fence_after();
      uint32_t ds[32];
      {
        uint32_t v0[32], v1[32];
        tmem_ld32(tDP, v0);
        tmem_ld32(tDP + 32, v1);
        wait_ld_dep32(v0);
        wait_ld_dep32(v1);
#pragma unroll
        for (int e4 = 0; e4 < 16; ++e4) {
          const float4 dl = del4[e4];
          const uint32_t* src = e4 < 8 ? &v0[e4 * 4] : &v1[(e4 - 8) * 4];
          const float2 p01 = unpack2<BF16>(pk[e4 * 2]), p23 = unpack2<BF16>(pk[e4 * 2 + 1]);
          float d0, d1, d2, d3;  // dS = P (dP - Delta), two lanes per instruction
          f2_split(mul_f2(f2(p01.x, p01.y),
                          sub_f2(f2(__uint_as_float(src[0]), __uint_as_float(src[1])), f2(dl.x, dl.y))), d0, d1);
          f2_split(mul_f2(f2(p23.x, p23.y),
                          sub_f2(f2(__uint_as_float(src[2]), __uint_as_float(src[3])), f2(dl.z, dl.w))), d2, d3);
          ds[e4 * 2] = pack2<BF16>(d0, d1);
          ds[e4 * 2 + 1] = pack2<BF16>(d2, d3);
        }
      }
      tmem_st32(tDP, ds);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(ds_ready);
      if (p.ds) {
        // key kr of the dS tile (i, jt), this warpgroup's 64 queries: eight
        // 16-byte core-matrix rows; per store a warp's 32 keys fill four
        // whole 128-byte core matrices.  Issued while the dK MMA runs.
        const int hq = g * G + it / n_i;
        const long long tile = (static_cast<long long>(b) * p.Hq + hq) * p.ds_tiles + ds_tile(i, jt, nq, p.causal);
        uint8_t* dst = reinterpret_cast<uint8_t*>(p.ds) + tile * 32768 + (kr >> 3) * 2048 + (kr & 7) * 16 + w * 1024;
        const uint64_t pol = policy_evict_first();  // streamed once: keep Q, dO resident in L2
#pragma unroll
        for (int c = 0; c < 8; ++c)
          st_global_hint(dst + c * 128, make_uint4(ds[4 * c], ds[4 * c + 1], ds[4 * c + 2], ds[4 * c + 3]), pol);
      }
    }
    // epilogue: warpgroup 0 stores dK (scaled), warpgroup 1 stores dV
    if (ok && mbar_wait_warp(kv_done, 0, abort_flag)) {
      tc_fence_after();
      const float mul = w == 0 ? p.scale : 1.0f;
      uint8_t* dst = reinterpret_cast<uint8_t*>(w == 0 ? p.dk : p.dv) +
                     2 * (static_cast<long long>(b) * p.dkv_batch_stride +
                          static_cast<long long>(key) * p.dkv_row_stride + static_cast<long long>(g) * D);
      const uint32_t src_col = w == 0 ? C::TM_DK : C::TM_DV;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_off + src_col + c * 32, v);
        wait_ld_dep32(v);
        uint4 o[4];
        uint32_t* ow = reinterpret_cast<uint32_t*>(o);
#pragma unroll
        for (int e = 0; e < 16; ++e)
          ow[e] = pack2<BF16>(__uint_as_float(v[2 * e]) * mul, __uint_as_float(v[2 * e + 1]) * mul);
        if (key_ok) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c * 64);
#pragma unroll
          for (int e = 0; e < 4; ++e) d4[e] = o[e];
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================================ dQ
template <int D>
struct DqCfg {
  static constexpr int TILE = 128 * D * 2;
  static constexpr int SLAB = 128 * 128;
  static constexpr int NST = (D == 64) ? 4 : 2;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_DO = OFF_Q + TILE;
  static constexpr int OFF_K = OFF_DO + TILE;
  static constexpr int OFF_V = OFF_K + NST * TILE;
  static constexpr int OFF_BAR = OFF_V + NST * TILE;
  // q_full, kv_full[NST], kv_empty[NST], s_full[2], dp_full, ds_ready, dq_done, drain
  static constexpr int NBAR = 1 + 2 * NST + 6;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int SMEM = OFF_MISC + 16 + 1024;
  static constexpr uint32_t TM_S0 = 0, TM_S1 = 128, TM_DP = 256, TM_DQ = 384;
};

template <int D, bool BF16>
__global__ void __launch_bounds__(320, 1) attn_bwd_dq_kernel(const __grid_constant__ BwdParams p) {
  using C = DqCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + C::NST;
  uint64_t* s_full = kv_empty + C::NST;
  uint64_t* dp_full = s_full + 2;
  uint64_t* ds_ready = dp_full + 1;
  uint64_t* dq_done = ds_ready + 1;
  uint64_t* mma_drain = dq_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);

  const int warp = warp_id(), lane = lane_id();
  const int BH = p.B * p.Hq;
  const int nq = p.S_pad >> 7;
  // longest (causal) query tile first; at D = 128 the (batch, q head) units go
  // in groups of eight (a GQA group of the long-context shape), so the CTAs
  // resident together stream the K and V tiles of one or two kv heads through
  // L2 (same-box A/B: 58.1 -> 56.9 ms at S=32768, 64/8 heads; 2.20 -> 2.06 ms
  // at the B=8, H=16, S=4096 shape; identical results)
  int qt, bh;
  {
    constexpr int HG = 8;
    const int full = BH / HG, per = HG * nq, cta = blockIdx.x;
    if (D != 128) {
      qt = nq - 1 - cta / BH;
      bh = cta % BH;
    } else if (cta < full * per) {
      const int r = cta % per;
      qt = nq - 1 - r / HG;
      bh = (cta / per) * HG + r % HG;
    } else {
      const int hr = BH - full * HG, r = cta - full * per;
      qt = nq - 1 - r / hr;
      bh = full * HG + r % hr;
    }
  }
  const int b = bh / p.Hq, h = bh % p.Hq;
  const int g = h / (p.Hq / p.Hkv);
  const int nkv = (p.S + 127) >> 7;
  const int nb = p.causal ? min(qt + 1, nkv) : nkv;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < C::NST; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(dp_full, 1);
    mbar_init(ds_ready, 256);
    mbar_init(dq_done, 1);
    mbar_init(mma_drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      prefetch_tmap(&p.tmQ);
      prefetch_tmap(&p.tmK);
      prefetch_tmap(&p.tmV);
      prefetch_tmap(&p.tmdO);
      const uint64_t pol_q = policy_evict_first(), pol_kv = policy_evict_last();
      mbar_arrive_expect_tx(q_full, 2 * C::TILE);
#pragma unroll
      for (int hh = 0; hh < D / 64; ++hh) {
        tma_load_3d(smem + C::OFF_Q + hh * C::SLAB, &p.tmQ, q_full, h * D + hh * 64, qt * 128, b, pol_q);
        tma_load_3d(smem + C::OFF_DO + hh * C::SLAB, &p.tmdO, q_full, h * D + hh * 64, qt * 128, b, pol_q);
      }
      int issued = 0;
      for (int j = 0; j < nb; ++j) {
        const int s = j % C::NST;
        if (!mbar_wait(&kv_empty[s], ((j / C::NST) & 1) ^ 1, abort_flag)) break;
        mbar_arrive_expect_tx(&kv_full[s], 2 * C::TILE);
#pragma unroll
        for (int hh = 0; hh < D / 64; ++hh) {
          tma_load_3d(smem + C::OFF_K + s * C::TILE + hh * C::SLAB, &p.tmK, &kv_full[s], g * D + hh * 64, j * 128,
                      b, pol_kv);
          tma_load_3d(smem + C::OFF_V + s * C::TILE + hh * C::SLAB, &p.tmV, &kv_full[s], g * D + hh * 64, j * 128,
                      b, pol_kv);
        }
        issued = j + 1;
      }
      if (*abort_flag) {
        volatile int never = 0;
        mbar_wait(q_full, 0, &never);
        for (int j = max(0, issued - C::NST); j < issued; ++j)
          mbar_wait(&kv_full[j % C::NST], (j / C::NST) & 1, &never);
      }
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = idesc_f16kind(128, 128, BF16, false, false);  // S, dP
      constexpr uint32_t idQ = idesc_f16kind(128, D, BF16, false, true);     // dQ (A = dS in TMEM)
      const uint32_t sQ = sbase + C::OFF_Q, sO = sbase + C::OFF_DO;
      auto sK = [&](int s) { return sbase + C::OFF_K + s * C::TILE; };
      auto sV = [&](int s) { return sbase + C::OFF_V + s * C::TILE; };
      auto tS = [&](int j) { return tmem + ((j & 1) ? C::TM_S1 : C::TM_S0); };
      auto issue_nt = [&](uint32_t d, uint32_t a, uint32_t bm) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * C::SLAB + (kk & 3) * 32;
          umma_ss(d, sdesc_sw128(a + off, 16, 1024), sdesc_sw128(bm + off, 16, 1024), idS, kk > 0 ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(q_full, 0, abort_flag) && mbar_wait(&kv_full[0], 0, abort_flag);
      if (ok) {
        tc_fence_after();
        issue_nt(tS(0), sQ, sK(0));
        umma_commit(&s_full[0]);
        issue_nt(tmem + C::TM_DP, sO, sV(0));
        umma_commit(dp_full);
      }
      for (int j = 0; ok && j < nb; ++j) {
        const int s = j % C::NST, s1 = (j + 1) % C::NST;
        const bool more = j + 1 < nb;
        if (more) {
          if (!(ok = mbar_wait(&kv_full[s1], ((j + 1) / C::NST) & 1, abort_flag))) break;
          tc_fence_after();
          issue_nt(tS(j + 1), sQ, sK(s1));                                    // S for the next block
          umma_commit(&s_full[(j + 1) & 1]);
        }
        if (!(ok = mbar_wait(ds_ready, j & 1, abort_flag))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)                                         // dQ += dS K
          umma_ts(tmem + C::TM_DQ, tS(j) + half_split_col(kk), sdesc_sw128(sK(s) + kk * 2048, C::SLAB, 1024), idQ,
                  (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&kv_empty[s]);
        if (more) {
          issue_nt(tmem + C::TM_DP, sO, sV(s1));                              // dP for the next block
          umma_commit(dp_full);
        }
      }
      if (ok) umma_commit(dq_done);
      else {
        volatile int never = 0;
        umma_commit(mma_drain);
        mbar_wait(mma_drain, 0, &never);
      }
    }
  } else {
    // ---------------------------------------------------------------- compute warpgroups
    const int w = warp >> 2;             // which half of the 128 keys of a block
    const int r = threadIdx.x & 127;     // query row = TMEM lane
    const int qrow = qt * 128 + r;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t cb = static_cast<uint32_t>(w * 64);
    const long long rowi = static_cast<long long>(bh) * p.S_pad + qrow;
    const float nlse2 = p.nlse2[rowi], dlt = p.delta[rowi];
    const float sl2 = p.scale_log2;
    bool ok = true;
    for (int j = 0; j < nb; ++j) {
      const uint32_t tSj = tmem + lane_off + ((j & 1) ? C::TM_S1 : C::TM_S0) + cb;
      const int kbase = j * 128 + w * 64;
      // keys >= lim are masked (sequence end, causal diagonal)
      const int lim = min(p.S - kbase, p.causal ? qrow - kbase + 1 : 64);
      if (!(ok = mbar_wait_warp(&s_full[j & 1], (j >> 1) & 1, abort_flag))) break;
      tc_fence_after();
      float pv[64];
      {
        uint32_t v0[32], v1[32];
        tmem_ld32(tSj, v0);
        tmem_ld32(tSj + 32, v1);
        wait_ld_dep32(v0);
        wait_ld_dep32(v1);
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          pv[c] = ex2(fmaf(__uint_as_float(v0[c]), sl2, nlse2));
          pv[c + 1] = ex2(fmaf(__uint_as_float(v0[c + 1]), sl2, nlse2));
          pv[32 + c] = ex2(fmaf(__uint_as_float(v1[c]), sl2, nlse2));
          pv[32 + c + 1] = ex2(fmaf(__uint_as_float(v1[c + 1]), sl2, nlse2));
        }
        if (lim < 64) {
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (c >= lim) pv[c] = 0.f;
        }
      }
      if (!(ok = mbar_wait_warp(dp_full, j & 1, abort_flag))) break;
      tc_fence_after();
      uint32_t ds[32];
      {
        uint32_t v0[32], v1[32];
        tmem_ld32(tmem + lane_off + C::TM_DP + cb, v0);
        tmem_ld32(tmem + lane_off + C::TM_DP + cb + 32, v1);
        wait_ld_dep32(v0);
        wait_ld_dep32(v1);
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          ds[e] = pack2<BF16>(pv[2 * e] * (__uint_as_float(v0[2 * e]) - dlt),
                                   pv[2 * e + 1] * (__uint_as_float(v0[2 * e + 1]) - dlt));
          ds[16 + e] = pack2<BF16>(pv[32 + 2 * e] * (__uint_as_float(v1[2 * e]) - dlt),
                                        pv[32 + 2 * e + 1] * (__uint_as_float(v1[2 * e + 1]) - dlt));
        }
      }
      tmem_st32(tSj, ds);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(ds_ready);
    }
    // epilogue: each warpgroup stores half of the D columns of dQ (scaled)
    if (ok && mbar_wait_warp(dq_done, 0, abort_flag)) {
      tc_fence_after();
      uint8_t* dst = reinterpret_cast<uint8_t*>(p.dq) +
                     2 * (static_cast<long long>(b) * p.dkv_batch_stride +
                          static_cast<long long>(qrow) * p.dkv_row_stride + static_cast<long long>(h) * D);
#pragma unroll 1
      for (int c = w * (D / 64); c < (w + 1) * (D / 64); ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_off + C::TM_DQ + c * 32, v);
        wait_ld_dep32(v);
        uint4 o[4];
        uint32_t* ow = reinterpret_cast<uint32_t*>(o);
#pragma unroll
        for (int e = 0; e < 16; ++e)
          ow[e] = pack2<BF16>(__uint_as_float(v[2 * e]) * p.scale, __uint_as_float(v[2 * e + 1]) * p.scale);
        if (qrow < p.S) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c * 64);
#pragma unroll
          for (int e = 0; e < 4; ++e) d4[e] = o[e];
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================================ dQ = dS K
// Persistent: one CTA per SM walks the (query tile, batch x q head) items in
// longest-first order (heads grouped at D = 128, see dsk_item), item t of the
// order at CTA t mod gridDim.  For each
// item the stored dS tiles of its query row (A, 128 queries x 128 keys in
// core-matrix order, one bulk copy each) and the matching K tiles (B, TMA,
// 128-byte swizzle) stream through an NST-stage ring that runs on across
// items; one thread issues the tcgen05 MMAs into one of two TMEM
// accumulators; four warps scale and store dQ of the previous item while the
// next one accumulates.
template <int D>
struct DskCfg {
  static constexpr int SLAB = 128 * 128;
  static constexpr int TILE_A = 2 * SLAB;       // 128 keys x 128 queries
  static constexpr int TILE_K = 128 * D * 2;    // 128 keys x D
  static constexpr int STAGE = TILE_A + TILE_K;
  static constexpr int NST = (D == 64) ? 4 : 3;
  static constexpr int OFF_BAR = NST * STAGE;
  // full[NST], empty[NST], acc_full[2], acc_empty[2], drain
  static constexpr int NBAR = 2 * NST + 5;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int SMEM = OFF_MISC + 16 + 1024;
  static constexpr uint32_t TM_COLS = 2 * D;    // two accumulators
};

struct DskItem {
  int qt, bh, nb;
};

// Item t of the walk.  At D = 128 the (batch, q head) units go in groups of
// eight, longest query tile first inside a group, so that the items resident
// at the same time read the K tiles of a few heads from L2 while the dS tiles
// stream past (same-box A/B at B=8, H=16, S=4096: 1.84 -> 1.69 ms per
// backward, identical results).  At D = 64 the plain longest-first order over
// all heads is kept (grouping gave nothing there).
template <int D>
TKB_DEVFN DskItem dsk_item(const BwdParams& p, int t) {
  const int BH = p.B * p.Hq, nq = p.S_pad >> 7;
  DskItem it;
  constexpr int HG = 8;
  const int full = BH / HG, per = HG * nq;
  if (D != 128) {
    it.qt = nq - 1 - t / BH;
    it.bh = t % BH;
  } else if (t < full * per) {
    const int r = t % per;
    it.qt = nq - 1 - r / HG;
    it.bh = (t / per) * HG + r % HG;
  } else {
    const int hr = BH - full * HG, r = t - full * per;
    it.qt = nq - 1 - r / hr;
    it.bh = full * HG + r % hr;
  }
  it.nb = p.causal ? it.qt + 1 : nq;
  return it;
}

template <int D, bool BF16>
__global__ void __launch_bounds__(192, 1) attn_bwd_dsk_kernel(const __grid_constant__ BwdParams p) {
  using C = DskCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* full = bars;
  uint64_t* empty = full + C::NST;
  uint64_t* acc_full = empty + C::NST;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* mma_drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);

  const int warp = warp_id(), lane = lane_id();
  const int nq = p.S_pad >> 7;
  const int n_items = p.B * p.Hq * nq;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 128);
    }
    mbar_init(mma_drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, C::TM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      prefetch_tmap(&p.tmK);
      const uint64_t pol_ds = policy_evict_first(), pol_k = policy_evict_last();
      int n = 0;  // ring position, continuous across items
      bool ok = true;
      for (int t = blockIdx.x; ok && t < n_items; t += gridDim.x) {
        const DskItem it = dsk_item<D>(p, t);
        const int b = it.bh / p.Hq, g = (it.bh % p.Hq) / (p.Hq / p.Hkv);
        // the tiles of one query row are consecutive
        const long long tile0 = static_cast<long long>(it.bh) * p.ds_tiles + ds_tile(it.qt, 0, nq, p.causal);
        for (int j = 0; j < it.nb; ++j, ++n) {
          const int s = n % C::NST;
          if (!(ok = mbar_wait(&empty[s], ((n / C::NST) & 1) ^ 1, abort_flag))) break;
          mbar_arrive_expect_tx(&full[s], C::STAGE);
          uint8_t* st = smem + s * C::STAGE;
          bulk_load_hint(st, reinterpret_cast<const uint8_t*>(p.ds) + (tile0 + j) * 32768, C::TILE_A, &full[s],
                         pol_ds);
#pragma unroll
          for (int hh = 0; hh < D / 64; ++hh)
            tma_load_3d(st + C::TILE_A + hh * C::SLAB, &p.tmK, &full[s], g * D + hh * 64, j * 128, b, pol_k);
        }
      }
      if (!ok) {
        // let the copies in flight land before the CTA exits
        volatile int never = 0;
        for (int m = max(0, n - C::NST); m < n; ++m) mbar_wait(&full[m % C::NST], (m / C::NST) & 1, &never);
      }
    }
  } else if (warp == 5) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t id = idesc_f16kind(128, D, BF16, true, true);  // A query-major, B key-major
      int n = 0, k = 0;  // ring position; item count of this CTA
      bool ok = true;
      for (int t = blockIdx.x; ok && t < n_items; t += gridDim.x, ++k) {
        const DskItem it = dsk_item<D>(p, t);
        const int a = k & 1;
        // the epilogue has emptied this accumulator (item k - 2)
        if (!(ok = mbar_wait(&acc_empty[a], ((k >> 1) & 1) ^ 1, abort_flag))) break;
        tc_fence_after();
        const uint32_t acc = tmem + a * D;
        for (int j = 0; j < it.nb; ++j, ++n) {
          const int s = n % C::NST;
          if (!(ok = mbar_wait(&full[s], (n / C::NST) & 1, abort_flag))) break;
          tc_fence_after();
          const uint32_t sa = sbase + s * C::STAGE, sk = sa + C::TILE_A;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_ss(acc, sdesc_interleave(sa + kk * 4096, 2048, 128), sdesc_sw128(sk + kk * 2048, C::SLAB, 1024), id,
                    (j > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&acc_full[a]);
      }
      if (!ok) {
        volatile int never = 0;
        umma_commit(mma_drain);
        mbar_wait(mma_drain, 0, &never);
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue: warps 0-3, one query row each
    const int r = threadIdx.x;  // TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    int k = 0;
    for (int t = blockIdx.x; t < n_items; t += gridDim.x, ++k) {
      const DskItem it = dsk_item<D>(p, t);
      const int a = k & 1;
      if (!mbar_wait_warp(&acc_full[a], (k >> 1) & 1, abort_flag)) break;
      tc_fence_after();
      const int b = it.bh / p.Hq, h = it.bh % p.Hq;
      const int qrow = it.qt * 128 + r;
      uint8_t* dst = reinterpret_cast<uint8_t*>(p.dq) +
                     2 * (static_cast<long long>(b) * p.dkv_batch_stride +
                          static_cast<long long>(qrow) * p.dkv_row_stride + static_cast<long long>(h) * D);
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_off + a * D + c * 32, v);
        wait_ld_dep32(v);
        uint4 o[4];
        uint32_t* ow = reinterpret_cast<uint32_t*>(o);
#pragma unroll
        for (int e = 0; e < 16; ++e)
          ow[e] = pack2<BF16>(__uint_as_float(v[2 * e]) * p.scale, __uint_as_float(v[2 * e + 1]) * p.scale);
        if (qrow < p.S) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c * 64);
#pragma unroll
          for (int e = 0; e < 4; ++e) d4[e] = o[e];
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[a]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TM_COLS);
  }
}

template <int D, bool BF16>
static cudaError_t launch_bwd(const BwdParams& p, cudaStream_t stream) {
  {
    using C = DkvCfg<D>;
    auto kern = attn_bwd_dkdv_kernel<D, BF16>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    kern<<<static_cast<unsigned>(p.B * p.Hkv * (p.S_pad / 128)), 320, C::SMEM, stream>>>(p);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  if (p.ds) {
    using C = DskCfg<D>;
    auto kern = attn_bwd_dsk_kernel<D, BF16>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int items = p.B * p.Hq * (p.S_pad / 128);
    kern<<<static_cast<unsigned>(items < sms ? items : sms), 192, C::SMEM, stream>>>(p);
    return cudaGetLastError();
  }
  {
    using C = DqCfg<D>;
    auto kern = attn_bwd_dq_kernel<D, BF16>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    kern<<<static_cast<unsigned>(p.B * p.Hq * (p.S_pad / 128)), 320, C::SMEM, stream>>>(p);
    return cudaGetLastError();
  }
}

cudaError_t attn_bwd_tc(const BwdParams& p, int D, bool bf16, cudaStream_t stream) {
  if (D == 128) return bf16 ? launch_bwd<128, true>(p, stream) : launch_bwd<128, false>(p, stream);
  if (D == 64) return bf16 ? launch_bwd<64, true>(p, stream) : launch_bwd<64, false>(p, stream);
  return cudaErrorInvalidValue;
}

}  // namespace tkb
