// attn_bwd.cu -- GQA flash-attention backward for sm_100a (tcgen05 + TMEM + TMA).
//
// Replaces k_gqa_flash_attn_tc_bwd<HEAD_DIM> (src/tkm_gpu.cu:440-598 of the
// reference).  Same inputs (packed QKV, O, dO, LSE) and the same dQ math
// (D = rowsum(O*dO), P = exp(s*scale - LSE), dS = P*(dP - D)*scale,
// dQ = dS K), but with the true dK = dS^T Q and dV = P^T dO summed over the
// query heads of each KV head (the reference writes dK := dQ, dV := dO at
// src/tkm_gpu.cu:588-596).
//
// One CTA owns a 128-key tile of one (batch, kv-head); it keeps K, V and the
// dK, dV accumulators resident and walks every (query head of the group,
// 128-row query tile) pair that can see those keys (causal: tiles at or
// below the diagonal only).
//   warps 0-3  compute warpgroup (thread = key row): P^T, dS^T
//   warps 4-7  dQ warpgroup: drains dQ tiles from TMEM into fp32 global sums
//   warp 8     TMA producer (K, V once; Q, dO, LSE, Delta ring)
//   warp 9     tcgen05 MMA issuer, TMEM owner
// Five MMAs per step, all M = 128:
//   S^T = K Q^T, dP^T = V dO^T, dV += P^T dO (A from TMEM),
//   dK += dS^T Q (A from TMEM), dQ = dS K (A = dS in shared memory).
#include "tkb_common.cuh"
#include "tkb_internal.h"

namespace tkb {

template <int D>
struct BwdCfg {
  static constexpr int TILE = 128 * D * 2;
  static constexpr int SLAB = 128 * 128;
  static constexpr int NSTQ = 2;
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + TILE;
  static constexpr int OFF_Q = OFF_V + TILE;           // NSTQ tiles
  static constexpr int OFF_DO = OFF_Q + NSTQ * TILE;   // NSTQ tiles
  static constexpr int OFF_DS = OFF_DO + NSTQ * TILE;  // 128 x 128 16-bit, MN-major
  static constexpr int OFF_LSE = OFF_DS + 128 * 128 * 2;  // NSTQ x 128 floats
  static constexpr int OFF_DEL = OFF_LSE + NSTQ * 512;    // NSTQ x 128 floats
  static constexpr int OFF_BAR = OFF_DEL + NSTQ * 512;
  // kv_full, q_full[NSTQ], q_empty[NSTQ], st_full, dp_full, p_ready, ds_ready, dq_full, dq_empty, kv_done, drain
  static constexpr int NBAR = 1 + 2 * NSTQ + 8;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int USED = OFF_MISC + 16;
  static constexpr int SLACK = (232448 - USED) < 1024 ? (232448 - USED) : 1024;
  static constexpr int SMEM = USED + SLACK;
  static constexpr uint32_t TM_ST = 0, TM_DP = 128;
  static constexpr uint32_t TM_DQ = (D == 128) ? 128 : 256;
  static constexpr uint32_t TM_DK = (D == 128) ? 256 : 320;
  static constexpr uint32_t TM_DV = TM_DK + D;
  static_assert(USED <= 232448, "shared memory budget");
};

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

template <int D, bool BF16>
__global__ void __launch_bounds__(320, 1) attn_bwd_tc_kernel(const __grid_constant__ BwdParams p) {
  using C = BwdCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw_s = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (raw_s & 1023u)) & 1023u;
  if (pad > static_cast<uint32_t>(C::SLACK)) {
    if (threadIdx.x == 0) atomicOr(&g_device_error, ERR_BAD_LAUNCH);
    return;
  }
  uint8_t* smem = smem_raw + pad;
  const uint32_t sbase = raw_s + pad;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* kv_full = bars;
  uint64_t* q_full = bars + 1;
  uint64_t* q_empty = q_full + C::NSTQ;
  uint64_t* st_full = q_empty + C::NSTQ;
  uint64_t* dp_full = st_full + 1;
  uint64_t* p_ready = dp_full + 1;
  uint64_t* ds_ready = p_ready + 1;
  uint64_t* dq_full = ds_ready + 1;
  uint64_t* dq_empty = dq_full + 1;
  uint64_t* kv_done = dq_empty + 1;
  uint64_t* mma_drain = kv_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  const float* s_lse = reinterpret_cast<const float*>(smem + C::OFF_LSE);
  const float* s_del = reinterpret_cast<const float*>(smem + C::OFF_DEL);

  const int warp = warp_id(), lane = lane_id();
  const int BG = p.B * p.Hkv;
  const int jt = static_cast<int>(blockIdx.x / BG);  // kv tile; tile 0 has the most work
  const int bg = blockIdx.x % BG;
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
    mbar_init(st_full, 1);
    mbar_init(dp_full, 1);
    mbar_init(p_ready, 128);
    mbar_init(ds_ready, 128);
    mbar_init(dq_full, 1);
    mbar_init(dq_empty, 128);
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
    // ------------------------------------------------------------ TMA producer
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
        bulk_load(smem + C::OFF_LSE + s * 512, p.lse2 + ro, 512, &q_full[s]);
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
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = idesc_f16kind(128, 128, BF16, false, false);  // S^T, dP^T
      constexpr uint32_t idKV = idesc_f16kind(128, D, BF16, false, true);    // dV, dK (A in TMEM)
      constexpr uint32_t idQ = idesc_f16kind(128, D, BF16, true, true);      // dQ (A = dS, MN-major)
      const uint32_t sK = sbase + C::OFF_K, sV = sbase + C::OFF_V, sDS = sbase + C::OFF_DS;
      bool ok = mbar_wait(kv_full, 0, abort_flag);
      for (int it = 0; ok && it < n_steps; ++it) {
        const int s = it % C::NSTQ;
        const uint32_t sQ = sbase + C::OFF_Q + s * C::TILE, sO = sbase + C::OFF_DO + s * C::TILE;
        if (!(ok = mbar_wait(&q_full[s], (it / C::NSTQ) & 1, abort_flag))) break;
        tc_fence_after();
        // S^T = K Q^T
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * C::SLAB + (kk & 3) * 32;
          umma_ss(tmem + C::TM_ST, sdesc_sw128(sK + off, 16, 1024), sdesc_sw128(sQ + off, 16, 1024), idS,
                  kk > 0 ? 1u : 0u);
        }
        umma_commit(st_full);
        // dP^T = V dO^T  (for D = 128 the dP region also holds the previous dQ tile)
        if (C::TM_DQ == C::TM_DP && it > 0) {
          if (!(ok = mbar_wait(dq_empty, (it - 1) & 1, abort_flag))) break;
          tc_fence_after();
        }
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * C::SLAB + (kk & 3) * 32;
          umma_ss(tmem + C::TM_DP, sdesc_sw128(sV + off, 16, 1024), sdesc_sw128(sO + off, 16, 1024), idS,
                  kk > 0 ? 1u : 0u);
        }
        umma_commit(dp_full);
        // dV += P^T dO
        if (!(ok = mbar_wait(p_ready, it & 1, abort_flag))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_ts(tmem + C::TM_DV, tmem + C::TM_ST + kk * 8, sdesc_sw128(sO + kk * 2048, C::SLAB, 1024), idKV,
                  (it > 0 || kk > 0) ? 1u : 0u);
        // dK += dS^T Q
        if (!(ok = mbar_wait(ds_ready, it & 1, abort_flag))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_ts(tmem + C::TM_DK, tmem + C::TM_DP + kk * 8, sdesc_sw128(sQ + kk * 2048, C::SLAB, 1024), idKV,
                  (it > 0 || kk > 0) ? 1u : 0u);
        // dQ = dS K  (M = queries, K = keys)
        if (C::TM_DQ != C::TM_DP && it > 0) {
          if (!(ok = mbar_wait(dq_empty, (it - 1) & 1, abort_flag))) break;
          tc_fence_after();
        }
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_ss(tmem + C::TM_DQ, sdesc_sw128(sDS + kk * 2048, C::SLAB, 1024),
                  sdesc_sw128(sK + kk * 2048, C::SLAB, 1024), idQ, kk > 0 ? 1u : 0u);
        umma_commit(dq_full);
        umma_commit(&q_empty[s]);
      }
      if (ok) umma_commit(kv_done);
      else {
        volatile int never = 0;
        umma_commit(mma_drain);
        mbar_wait(mma_drain, 0, &never);
      }
    }
  } else if (warp < 4) {
    // ------------------------------------------------------------ compute warpgroup
    const int kr = threadIdx.x;  // key row within the tile
    const int key = jt * 128 + kr;
    const bool key_ok = key < p.S;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const uint32_t tST = tmem + lane_off + C::TM_ST, tDP = tmem + lane_off + C::TM_DP;
    const float sl2 = p.scale_log2;
    uint8_t* ds_row = smem + C::OFF_DS + kr * 128;
    const int sw = kr & 7;
    bool ok = true;
    for (int it = 0; it < n_steps; ++it) {
      const int s = it % C::NSTQ;
      const int i = i0 + it % n_i;
      const float* lse = s_lse + s * 128;
      const float* del = s_del + s * 128;
      // keys above the diagonal of a diagonal tile see nothing
      const int qmin = (p.causal && i == jt) ? kr : 0;
      // LSE / Delta of this stage were written by the bulk copy: observe its barrier directly.
      if (!(ok = mbar_wait(&q_full[s], (it / C::NSTQ) & 1, abort_flag))) break;
      if (!(ok = mbar_wait(st_full, it & 1, abort_flag))) break;
      tc_fence_after();
      uint32_t pk[64];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld32(tST + c * 32, v);
        wait_ld_dep32(v);
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int q0 = c * 32 + 2 * e;
          float a = ex2(fmaf(__uint_as_float(v[2 * e]), sl2, -lse[q0]));
          float d = ex2(fmaf(__uint_as_float(v[2 * e + 1]), sl2, -lse[q0 + 1]));
          if (!key_ok || q0 < qmin) a = 0.f;
          if (!key_ok || q0 + 1 < qmin) d = 0.f;
          pk[c * 16 + e] = pack2<BF16>(a, d);
        }
      }
      tmem_st32(tST, *reinterpret_cast<uint32_t(*)[32]>(&pk[0]));
      tmem_st32(tST + 32, *reinterpret_cast<uint32_t(*)[32]>(&pk[32]));
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(p_ready);

      if (!(ok = mbar_wait(dp_full, it & 1, abort_flag))) break;
      tc_fence_after();
      uint32_t ds[64];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld32(tDP + c * 32, v);
        wait_ld_dep32(v);
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int q0 = c * 32 + 2 * e;
          const float2 pp = unpack2<BF16>(pk[c * 16 + e]);
          const float a = pp.x * (__uint_as_float(v[2 * e]) - del[q0]);
          const float d = pp.y * (__uint_as_float(v[2 * e + 1]) - del[q0 + 1]);
          ds[c * 16 + e] = pack2<BF16>(a, d);
        }
      }
      tmem_st32(tDP, *reinterpret_cast<uint32_t(*)[32]>(&ds[0]));
      tmem_st32(tDP + 32, *reinterpret_cast<uint32_t(*)[32]>(&ds[32]));
      // dS row -> shared memory, [query slab][key][64 queries] with 128-byte swizzle
#pragma unroll
      for (int qh = 0; qh < 2; ++qh)
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const int w0 = qh * 32 + ch * 4;
          *reinterpret_cast<uint4*>(ds_row + qh * C::SLAB + ((ch ^ sw) << 4)) =
              make_uint4(ds[w0], ds[w0 + 1], ds[w0 + 2], ds[w0 + 3]);
        }
      fence_proxy_async_smem();
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(ds_ready);
    }
    // dK epilogue
    if (ok && mbar_wait(kv_done, 0, abort_flag)) {
      tc_fence_after();
      uint8_t* dst = reinterpret_cast<uint8_t*>(p.dk) +
                     2 * (static_cast<long long>(b) * p.dkv_batch_stride +
                          static_cast<long long>(key) * p.dkv_row_stride + static_cast<long long>(g) * D);
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_off + C::TM_DK + c * 32, v);
        wait_ld_dep32(v);
        uint4 o[4];
        uint32_t* ow = reinterpret_cast<uint32_t*>(o);
#pragma unroll
        for (int e = 0; e < 16; ++e)
          ow[e] = pack2<BF16>(__uint_as_float(v[2 * e]) * p.scale, __uint_as_float(v[2 * e + 1]) * p.scale);
        if (key_ok) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c * 64);
#pragma unroll
          for (int e = 0; e < 4; ++e) d4[e] = o[e];
        }
      }
    }
  } else {
    // ------------------------------------------------------------ dQ warpgroup
    const int qr = threadIdx.x - 128;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tDQ = tmem + lane_off + C::TM_DQ;
    bool ok = true;
    for (int it = 0; it < n_steps; ++it) {
      const int hq = g * G + it / n_i, i = i0 + it % n_i;
      if (!(ok = mbar_wait(dq_full, it & 1, abort_flag))) break;
      tc_fence_after();
      uint32_t v[D];
#pragma unroll
      for (int c = 0; c < D / 32; ++c) tmem_ld32(tDQ + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&v[c * 32]));
#pragma unroll
      for (int c = 0; c < D / 32; ++c) wait_ld_dep32(*reinterpret_cast<uint32_t(*)[32]>(&v[c * 32]));
      tc_fence_before();
      mbar_arrive(dq_empty);
      float* dst = p.dq_acc + ((static_cast<long long>(b) * p.Hq + hq) * p.S_pad + i * 128 + qr) * D;
      const float sc = p.scale;
#pragma unroll
      for (int c = 0; c < D; c += 4)
        red_add_v4(dst + c, __uint_as_float(v[c]) * sc, __uint_as_float(v[c + 1]) * sc,
                   __uint_as_float(v[c + 2]) * sc, __uint_as_float(v[c + 3]) * sc);
    }
    // dV epilogue
    if (ok && mbar_wait(kv_done, 0, abort_flag)) {
      tc_fence_after();
      const int key = jt * 128 + qr;
      uint8_t* dst = reinterpret_cast<uint8_t*>(p.dv) +
                     2 * (static_cast<long long>(b) * p.dkv_batch_stride +
                          static_cast<long long>(key) * p.dkv_row_stride + static_cast<long long>(g) * D);
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_off + C::TM_DV + c * 32, v);
        wait_ld_dep32(v);
        uint4 o[4];
        uint32_t* ow = reinterpret_cast<uint32_t*>(o);
#pragma unroll
        for (int e = 0; e < 16; ++e) ow[e] = pack2<BF16>(__uint_as_float(v[2 * e]), __uint_as_float(v[2 * e + 1]));
        if (key < p.S) {
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

template <int D, bool BF16>
static cudaError_t launch_bwd(const BwdParams& p, cudaStream_t stream) {
  using C = BwdCfg<D>;
  auto kern = attn_bwd_tc_kernel<D, BF16>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  const unsigned grid = static_cast<unsigned>(p.B * p.Hkv * (p.S_pad / 128));
  kern<<<grid, 320, C::SMEM, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t attn_bwd_tc(const BwdParams& p, int D, bool bf16, cudaStream_t stream) {
  if (D == 128) return bf16 ? launch_bwd<128, true>(p, stream) : launch_bwd<128, false>(p, stream);
  if (D == 64) return bf16 ? launch_bwd<64, true>(p, stream) : launch_bwd<64, false>(p, stream);
  return cudaErrorInvalidValue;
}

}  // namespace tkb
