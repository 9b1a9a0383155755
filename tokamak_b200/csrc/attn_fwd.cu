// attn_fwd.cu -- GQA flash-attention forward for sm_100a (tcgen05 + TMEM + TMA).
//
// Replaces k_gqa_flash_attn_tc_fwd<HEAD_DIM> (src/tkm_gpu.cu:302-438 of the
// reference), same semantics: O = softmax(Q K^T * scale, causal key>query
// masked) V per head, LSE = ln(sum exp) per (b, q-head, row), kv head =
// q head / (Hq/Hkv).
//
// One CTA owns two 128-row query tiles of one (batch, q-head) and streams the
// 128-key K/V blocks of the matching kv head through shared memory.
//   warps 0-3  softmax warpgroup for query tile 0 (thread = query row)
//   warps 4-7  softmax warpgroup for query tile 1
//   warp 8     TMA producer (Q once, K and V rings of NSTK / NSTV stages)
//   warp 9     tcgen05 MMA issuer, TMEM owner
// TMEM (512 columns): S0 [0,128) S1 [128,256) O0 [256,256+D) O1 [256+D,256+2D).
// The softmax warps overwrite the first 64 columns of S with P (16-bit pairs),
// which the P*V MMA reads straight from TMEM.  Causal blocks above the
// diagonal are never loaded or computed.
#include "tkb_common.cuh"
#include "tkb_internal.h"

// V stages at D = 128 (2 or 3) and heads per CTA group (0: all heads'
// query-tile pairs longest first).  Same-box A/B at the headline shape:
// forward 0.624 ms with (2, 0), 0.633 with (3, 0), 0.601 with (2, 4),
// 0.559 with (2, 8), 0.567 with (2, 16), 0.566 with (3, 8).
#ifndef TKB_FWD_NSTV
#define TKB_FWD_NSTV 2
#endif
#ifndef TKB_FWD_HG
#define TKB_FWD_HG 8
#endif

namespace tkb {

template <int D>
struct FwdCfg {
  static constexpr int TILE = 128 * D * 2;  // bytes of one 128-row x D tile
  static constexpr int SLAB = 128 * 128;    // bytes of one 64-column swizzle slab
  // K and V rings counted apart: at D = 128 a third V stage (224 KB of tiles
  // in all) fits beside two K stages; it measured no faster once the CTAs of
  // a head group read K/V from L2.
  static constexpr int NSTK = (D == 64) ? 4 : 2;
  static constexpr int NSTV = (D == 64) ? 4 : TKB_FWD_NSTV;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + 2 * TILE;
  static constexpr int OFF_V = OFF_K + NSTK * TILE;
  static constexpr int OFF_BAR = OFF_V + NSTV * TILE;
  // q_full, k_full[NSTK], k_empty[NSTK], v_full[NSTV], v_empty[NSTV], s_full[2], p_ready[2][2], o_done[2], drain
  static constexpr int NBAR = 1 + 2 * NSTK + 2 * NSTV + 9;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int SMEM = OFF_MISC + 16 + 1024;  // + slack for 1024-byte alignment
  static_assert(SMEM <= 232448, "forward tiles exceed 227 KB of shared memory");
  static constexpr uint32_t TM_S0 = 0, TM_S1 = 128, TM_O0 = 256, TM_O1 = 256 + D;
};

TKB_DEVFN void wait_ld_dep(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
                 "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),
                 "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]),
                 "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]),
                 "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// CTA -> (batch x q head bh, query-tile pair t).  Heads go in groups of hg,
// longest pair first inside a group (causal), so that the CTAs running at
// the same time read the K/V tiles of a few heads, which then come from L2;
// hg = 0 orders all heads' pairs longest first.
TKB_DEVFN void fwd_cta_order(int cta, int BH, int npairs, int hg, int& bh, int& t) {
  if (hg <= 0) {
    bh = cta % BH;
    t = npairs - 1 - cta / BH;
    return;
  }
  const int full = BH / hg, per = hg * npairs;
  if (cta < full * per) {
    const int r = cta % per;
    t = npairs - 1 - r / hg;
    bh = (cta / per) * hg + r % hg;
  } else {
    const int hr = BH - full * hg, r = cta - full * per;
    t = npairs - 1 - r / hr;
    bh = full * hg + r % hr;
  }
}

// One key block of the online softmax for this thread's query row: S from
// TMEM, the causal and sequence-end masks, the running max raised when this
// block's exceeds it by more than 8 (rescaling O in TMEM), P written over S
// in two halves, and release(h) once half h (keys 64h .. 64h+63) is in TMEM.
template <int D, bool BF16, typename Release>
TKB_DEVFN void softmax_block(uint32_t tS, uint32_t tO, float sl2, int j, int qt, int qrow, int S, int causal,
                             float& m_used, float& l, Release&& release) {
  uint32_t r0[32], r1[32], r2[32], r3[32];
  tmem_ld32(tS + 0, r0);
  tmem_ld32(tS + 32, r1);
  tmem_ld32(tS + 64, r2);
  tmem_ld32(tS + 96, r3);
  wait_ld_dep(r0);
  wait_ld_dep(r1);
  wait_ld_dep(r2);
  wait_ld_dep(r3);
  float sv[128];
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    sv[i] = __uint_as_float(r0[i]);
    sv[32 + i] = __uint_as_float(r1[i]);
    sv[64 + i] = __uint_as_float(r2[i]);
    sv[96 + i] = __uint_as_float(r3[i]);
  }
  const int kbase = j * 128;
  if ((causal && kbase + 127 > qt * 128) || kbase + 128 > S) {
    const int lim = min(S - kbase, causal ? qrow - kbase + 1 : 128);
#pragma unroll
    for (int c = 0; c < 128; ++c)
      if (c >= lim) sv[c] = -INFINITY;
  }
  float mx0 = sv[0], mx1 = sv[1], mx2 = sv[2], mx3 = sv[3];
#pragma unroll
  for (int c = 4; c < 128; c += 8) {
    mx0 = fmax3(mx0, sv[c], sv[c + 1]);
    mx1 = fmax3(mx1, sv[c + 2], sv[c + 3]);
    mx2 = fmax3(mx2, sv[c + 4], sv[c + 5]);
    mx3 = fmax3(mx3, sv[c + 6], sv[c + 7]);
  }
  const float mx = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * sl2;
  // Raise the running max when this block's exceeds it by more than 8
  // (2^8 headroom in fp32): the row sum now, the partial O row below,
  // after the first half's exponentials, when half of S is no longer
  // live in registers (the O chunks then fit without spilling).
  float resc = 1.f;
  bool raised = false;
  if (j == 0) {
    m_used = (mx == -INFINITY) ? 0.f : mx;
  } else if (mx > m_used + 8.0f) {
    resc = ex2(m_used - mx);  // may be 0 for a jump past 2^126: O is then cleared
    l *= resc;
    m_used = mx;
    raised = true;
  }
  const uint64_t sl2x2 = f2(sl2, sl2), nmx2 = f2(-m_used, -m_used);
  uint32_t pk0[32], pk1[32];
  uint64_t ls0 = f2(0.f, 0.f), ls1 = f2(0.f, 0.f);
  // exponentials of keys 2i, 2i+1 (pair i of the half at sv + base): the
  // scale and the row sums in packed f32x2 instructions
  auto exp_pair = [&](int base, int i, uint32_t& pk, uint64_t& ls) {
    float x0, x1, a, c;
    f2_split(fma_f2(f2(sv[base + 2 * i], sv[base + 2 * i + 1]), sl2x2, nmx2), x0, x1);
    a = ex2(x0);
    c = ex2(x1);
    ls = add_f2(ls, f2(a, c));
    pk = pack2_int<BF16>(a, c);
  };
  // P for keys 0-63 goes to TMEM first so that the P*V MMA can start on
  // that half while the exponentials of keys 64-127 are computed.
#pragma unroll
  for (int i = 0; i < 32; ++i) exp_pair(0, i, pk0[i], (i & 1) ? ls1 : ls0);
  if (__any_sync(0xffffffffu, raised)) {
    // The warp rescales its 32 rows of O if any of them raised its maximum
    // (rows that did not multiply by 1): tcgen05.ld / st are warp-collective
    // and must not run under a per-row condition.  O of the previous blocks
    // is complete: s_full of this block was committed after their P*V MMAs.
    // P*V of this block waits for p_ready.
#pragma unroll 1
    for (int c = 0; c < D / 32; ++c) {
      uint32_t o[32];
      tmem_ld32(tO + c * 32, o);
      wait_ld_dep(o);
#pragma unroll
      for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * resc);
      tmem_st32(tO + c * 32, o);
    }
  }
  tmem_st32(tS + 0, pk0);
  tmem_wait_st();
  tc_fence_before();
  release(0);
#pragma unroll
  for (int i = 0; i < 32; ++i) exp_pair(64, i, pk1[i], (i & 1) ? ls1 : ls0);
  {
    float a0, a1, b0, b1;
    f2_split(ls0, a0, a1);
    f2_split(ls1, b0, b1);
    l += (a0 + b0) + (a1 + b1);
  }
  tmem_st32(tS + 32, pk1);
  tmem_wait_st();
  tc_fence_before();
  release(1);
}

template <int D, bool BF16>
__global__ void __launch_bounds__(320, 1) attn_fwd_tc_kernel(const __grid_constant__ FwdParams p) {
  using C = FwdCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + C::NSTK;
  uint64_t* v_full = k_empty + C::NSTK;
  uint64_t* v_empty = v_full + C::NSTV;
  uint64_t* s_full = v_empty + C::NSTV;
  uint64_t* p_ready = s_full + 2;  // [w][half]: P of keys 0-63 / 64-127 of the block is in TMEM
  uint64_t* o_done = p_ready + 4;
  uint64_t* mma_drain = o_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);

  const int warp = warp_id(), lane = lane_id();
  const int BH = p.B * p.Hq;
  int bh, t;  // (batch, q head), query-tile pair
  fwd_cta_order(blockIdx.x, BH, p.n_pairs, TKB_FWD_HG, bh, t);
  const int b = bh / p.Hq, h = bh % p.Hq;
  const int g = h / (p.Hq / p.Hkv);
  const int nkv = (p.S + 127) >> 7;
  int nb[2];
#pragma unroll
  for (int w = 0; w < 2; ++w) {
    const int qt = 2 * t + w;
    nb[w] = (qt * 128 >= p.S) ? 0 : (p.causal ? min(qt + 1, nkv) : nkv);
  }
  const int nblk = max(nb[0], nb[1]);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < C::NSTK; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < C::NSTV; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int w = 0; w < 2; ++w) {
      mbar_init(&s_full[w], 1);
      mbar_init(&p_ready[2 * w], 128);
      mbar_init(&p_ready[2 * w + 1], 128);
      mbar_init(&o_done[w], 1);
    }
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
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&p.tmQ);
      prefetch_tmap(&p.tmK);
      prefetch_tmap(&p.tmV);
      const uint64_t pol_q = policy_evict_first(), pol_kv = policy_evict_last();
      mbar_arrive_expect_tx(q_full, 2 * C::TILE);
#pragma unroll
      for (int w = 0; w < 2; ++w)
#pragma unroll
        for (int hh = 0; hh < D / 64; ++hh)
          tma_load_3d(smem + C::OFF_Q + w * C::TILE + hh * C::SLAB, &p.tmQ, q_full, h * D + hh * 64,
                      (2 * t + w) * 128, b, pol_q);
      int issued = 0;
      for (int j = 0; j < nblk; ++j) {
        const int sk = j % C::NSTK, sv = j % C::NSTV;
        if (!mbar_wait(&k_empty[sk], ((j / C::NSTK) & 1) ^ 1, abort_flag)) break;
        mbar_arrive_expect_tx(&k_full[sk], C::TILE);
#pragma unroll
        for (int hh = 0; hh < D / 64; ++hh)
          tma_load_3d(smem + C::OFF_K + sk * C::TILE + hh * C::SLAB, &p.tmK, &k_full[sk], g * D + hh * 64,
                      j * 128, b, pol_kv);
        if (!mbar_wait(&v_empty[sv], ((j / C::NSTV) & 1) ^ 1, abort_flag)) {
          issued = -(j + 1);  // K of block j is in flight, V is not
          break;
        }
        mbar_arrive_expect_tx(&v_full[sv], C::TILE);
#pragma unroll
        for (int hh = 0; hh < D / 64; ++hh)
          tma_load_3d(smem + C::OFF_V + sv * C::TILE + hh * C::SLAB, &p.tmV, &v_full[sv], g * D + hh * 64,
                      j * 128, b, pol_kv);
        issued = j + 1;
      }
      if (*abort_flag) {
        // Let every copy this CTA started land before the CTA exits.
        volatile int never = 0;
        mbar_wait(q_full, 0, &never);
        const int nk = issued < 0 ? -issued : issued, nv = issued < 0 ? -issued - 1 : issued;
        for (int j = max(0, nk - C::NSTK); j < nk; ++j) mbar_wait(&k_full[j % C::NSTK], (j / C::NSTK) & 1, &never);
        for (int j = max(0, nv - C::NSTV); j < nv; ++j) mbar_wait(&v_full[j % C::NSTV], (j / C::NSTV) & 1, &never);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && nblk > 0) {
      constexpr uint32_t idS = idesc_f16kind(128, 128, BF16, false, false);
      constexpr uint32_t idO = idesc_f16kind(128, D, BF16, false, true);
      const uint32_t sQ = sbase + C::OFF_Q, sK = sbase + C::OFF_K, sV = sbase + C::OFF_V;
      auto issue_S = [&](int w, int s) {
        const uint32_t qa = sQ + w * C::TILE, ka = sK + s * C::TILE;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * C::SLAB + (kk & 3) * 32;
          umma_ss(tmem + (w ? C::TM_S1 : C::TM_S0), sdesc_sw128(qa + off, 16, 1024),
                  sdesc_sw128(ka + off, 16, 1024), idS, kk > 0 ? 1u : 0u);
        }
      };
      // O += P V over the keys of one half of the block (k-steps 4*half .. 4*half+3)
      auto issue_PV = [&](int w, int s, int half, bool acc) {
        const uint32_t va = sV + s * C::TILE;
        const uint32_t tP = tmem + (w ? C::TM_S1 : C::TM_S0);
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {
          const int kk = half * 4 + k4;
          umma_ts(tmem + (w ? C::TM_O1 : C::TM_O0), tP + kk * 8, sdesc_sw128(va + kk * 2048, C::SLAB, 1024), idO,
                  (acc || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(q_full, 0, abort_flag) && mbar_wait(&k_full[0], 0, abort_flag);
      if (ok) {
        tc_fence_after();
        for (int w = 0; w < 2; ++w)
          if (nb[w] > 0) {
            issue_S(w, 0);
            umma_commit(&s_full[w]);
          }
        umma_commit(&k_empty[0]);
      }
      for (int j = 0; ok && j < nblk; ++j) {
        const int s = j % C::NSTV, s1 = (j + 1) % C::NSTK;  // V stage of block j, K stage of block j + 1
        if (!(ok = mbar_wait(&v_full[s], (j / C::NSTV) & 1, abort_flag))) break;
        bool k_next = false;
        for (int w = 0; w < 2 && ok; ++w) {
          if (j >= nb[w]) continue;
          if (!(ok = mbar_wait(&p_ready[2 * w], j & 1, abort_flag))) break;
          tc_fence_after();
          issue_PV(w, s, 0, j > 0);
          if (!(ok = mbar_wait(&p_ready[2 * w + 1], j & 1, abort_flag))) break;
          tc_fence_after();
          issue_PV(w, s, 1, true);
          if (j == nb[w] - 1) umma_commit(&o_done[w]);
          if (j + 1 < nb[w]) {
            if (!k_next) {
              if (!(ok = mbar_wait(&k_full[s1], ((j + 1) / C::NSTK) & 1, abort_flag))) break;
              tc_fence_after();
              k_next = true;
            }
            issue_S(w, s1);
            umma_commit(&s_full[w]);
          }
        }
        umma_commit(&v_empty[s]);
        if (k_next) umma_commit(&k_empty[s1]);
      }
      if (!ok) {
        // Make sure no MMA is still running when TMEM is released.
        volatile int never = 0;
        umma_commit(mma_drain);
        mbar_wait(mma_drain, 0, &never);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax warpgroups
    const int w = warp >> 2;
    const int r = threadIdx.x & 127;
    const int qt = 2 * t + w;
    const int qrow = qt * 128 + r;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_off + (w ? C::TM_S1 : C::TM_S0);
    const uint32_t tO = tmem + lane_off + (w ? C::TM_O1 : C::TM_O0);
    const float sl2 = p.scale_log2;
    float m_used = 0.f, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nb[w]; ++j) {
      if (!(ok = mbar_wait_warp(&s_full[w], j & 1, abort_flag))) break;
      tc_fence_after();
      softmax_block<D, BF16>(tS, tO, sl2, j, qt, qrow, p.S, p.causal, m_used, l,
                             [&](int hh) { mbar_arrive(&p_ready[2 * w + hh]); });
    }
    if (ok && nb[w] > 0 && mbar_wait_warp(&o_done[w], 0, abort_flag)) {
      tc_fence_after();
      const float inv_l = l > 0.f ? 1.0f / l : 0.f;
      const bool valid = qrow < p.S;
      uint8_t* orow = reinterpret_cast<uint8_t*>(p.out) +
                      2 * (static_cast<long long>(b) * p.out_batch_stride +
                           static_cast<long long>(qrow) * p.out_row_stride + static_cast<long long>(h) * D);
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(tO + c * 32, o);
        wait_ld_dep(o);
        uint4 v[4];
        uint32_t* vw = reinterpret_cast<uint32_t*>(v);
#pragma unroll
        for (int i = 0; i < 16; ++i)
          vw[i] = pack2<BF16>(__uint_as_float(o[2 * i]) * inv_l, __uint_as_float(o[2 * i + 1]) * inv_l);
        if (valid) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 64);
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[i] = v[i];
        }
      }
      if (valid && p.lse)
        p.lse[static_cast<long long>(bh) * p.S + qrow] = (m_used + lg2(l)) * 0.69314718055994531f;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D, bool BF16>
static cudaError_t launch_fwd(const FwdParams& p, cudaStream_t stream) {
  using C = FwdCfg<D>;
  auto kern = attn_fwd_tc_kernel<D, BF16>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  const unsigned grid = static_cast<unsigned>(p.B * p.Hq * p.n_pairs);
  kern<<<grid, 320, C::SMEM, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t attn_fwd_tc(const FwdParams& p, int D, bool bf16, cudaStream_t stream) {
  if (D == 128) return bf16 ? launch_fwd<128, true>(p, stream) : launch_fwd<128, false>(p, stream);
  if (D == 64) return bf16 ? launch_fwd<64, true>(p, stream) : launch_fwd<64, false>(p, stream);
  return cudaErrorInvalidValue;
}

}  // namespace tkb
