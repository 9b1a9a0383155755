// gemm.cu -- bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM +
// TMA) with fused epilogues.
//
// Replaces the cuBLAS calls of the reference's FC layers (src/tkm_gpu.cu:
// 1207-1236 forward, 1330-1372 backward): C[M][N] (+)= A[M][K] B[K][N] with
// bf16 operands and fp32 accumulation, where each operand is stored either
// K-contiguous or M/N-contiguous, so the forward (X W), the input gradient
// (dY W^T) and the weight gradient (X^T dY) all run without transposes.
//
// Persistent kernel, one CTA per SM walking 128 x 256 output tiles (grouped
// by eight row tiles so the resident CTAs share A and B tiles in L2):
//   warp 0      TMA producer: 64-deep K slices of A (16 KB) and B (32 KB)
//               into a 4-stage shared-memory ring (128-byte swizzle)
//   warp 1      TMEM owner (512 columns = two 128 x 256 fp32 accumulators)
//               and single-thread tcgen05.mma issuer (M=128, N=256, K=16)
//   warps 2-5   epilogue: tcgen05.ld of one accumulator row per thread while
//               the MMA warp fills the other accumulator, then the fused
//               epilogue and 16-byte global stores
// Epilogues: plain (bf16 or fp32, optionally accumulating into C), per-column
// bias, and SwiGLU: the tile's 256 columns are 128 gate and 128 up columns
// of the fused [gate | up] weight (B loaded from both halves), and the
// epilogue writes [gate | up] (the backward replays from it) and
// h = SiLU(gate + b_gate) * (up + b_up) in one pass.
// Every wait is bounded; a timeout sets the device error word and the CTA
// drains its copies and MMAs and frees TMEM before returning.
#include "tkb_common.cuh"
#include "tkb_internal.h"

namespace tkb {

namespace gk {
constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4, THREADS = 192;
constexpr int A_BYTES = BM * BK * 2;   // 16 KB
constexpr int B_BYTES = BN * BK * 2;   // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int OFF_BAR = STAGES * STAGE_BYTES;
constexpr int NBAR = 2 * STAGES + 5;   // full[S], empty[S], acc_full[2], acc_empty[2], drain
constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
constexpr int OFF_BIAS = OFF_MISC + 16;       // the column tile's 256 bias values
constexpr int SMEM = OFF_BIAS + 1024 + 1024;  // + slack for the 1024-byte alignment of the swizzled ring
constexpr int GROUP_M = 8;
enum { EPI_STORE = 0, EPI_BIAS = 1, EPI_SWIGLU = 2, EPI_CE_STATS = 3, EPI_CE_GRAD = 4 };
}  // namespace gk

// Tile t -> (row tile, column tile): groups of GROUP_M row tiles; inside a
// group consecutive tiles walk the group's row tiles for one column tile.
TKB_DEVFN void gemm_tile(int t, int tiles_m, int tiles_n, int& tm, int& tn) {
  const int per_group = gk::GROUP_M * tiles_n;
  const int g = t / per_group;
  const int first = g * gk::GROUP_M;
  const int gm = min(gk::GROUP_M, tiles_m - first);
  const int r = t - g * per_group;
  tm = first + r % gm;
  tn = r / gm;
}

// Column of B where the i-th 64-column box of column tile tn starts.
template <int EPI>
TKB_DEVFN int gemm_b_col(const GemmParams& p, int tn, int i) {
  if constexpr (EPI == gk::EPI_SWIGLU) return (i < 2 ? 0 : p.b_split) + tn * 128 + (i & 1) * 64;
  return tn * gk::BN + i * 64;
}

TKB_DEVFN float silu_f(float x) { return __fdividef(x, 1.0f + ex2(-1.4426950408889634f * x)); }

// Where a plain or bias epilogue writes: C (or a split-K partial), its row
// stride (elements) and mode.
struct EpiOut {
  void* c;
  long long ldc;
  int accumulate, out_f32;
};

// The 128 epilogue threads (warps 2-5) bring the column tile's bias values
// into shared memory once per tile: sb[0..255] for the bias epilogue; the
// gate bias in sb[0..127] and the up bias in sb[128..255] for SwiGLU.
// Named barrier 1 (the epilogue warps only); the caller syncs before reuse.
template <int EPI>
TKB_DEVFN void epi_stage_bias(const GemmParams& p, float* sb, int tn) {
  const int e = static_cast<int>(threadIdx.x) - 64;
  if constexpr (EPI == gk::EPI_SWIGLU) {
    const int n = tn * 128 + e;
    sb[e] = (p.bias && n < p.N) ? p.bias[n] : 0.f;
    sb[128 + e] = (p.bias2 && n < p.N) ? p.bias2[n] : 0.f;
  } else {
#pragma unroll
    for (int j = e; j < 256; j += 128) {
      const int n = tn * 256 + j;
      sb[j] = (p.bias && n < p.N) ? p.bias[n] : 0.f;
    }
  }
  asm volatile("bar.sync 1, 128;" ::: "memory");
}

// Before an epilogue tile: the epilogue warps agree on going on (one of them
// may have given up a wait) and, for the bias epilogues, stage the bias.
// Returns false when the CTA aborts.
template <int EPI>
TKB_DEVFN bool epi_begin(const GemmParams& p, float* sb, int tn, volatile int* abort_flag) {
  if constexpr (EPI == gk::EPI_STORE) {
    // one decision per warp: the epilogue's tcgen05.ld are warp-collective
    // (a lane whose wait gave up has raised the flag before voting)
    return __all_sync(0xffffffffu, !*abort_flag);
  } else {
    // one decision for all 128 epilogue threads (an OR over named barrier 1),
    // taken once every epilogue warp is past the previous tile, so that no
    // warp waits at the next named barrier for a warp that left
    uint32_t any;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, 1, 128, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(any)
        : "r"(static_cast<uint32_t>(*abort_flag))
        : "memory");
    if (any) return false;
    epi_stage_bias<EPI>(p, sb, tn);
    return true;
  }
}

// The epilogue of one accumulator tile for this thread's row: TMEM columns
// 0..255 of the accumulator at `tacc` (this warp's lane quadrant) -> C (and H).
template <int EPI>
TKB_DEVFN void gemm_epilogue(const GemmParams& p, const EpiOut& o, const float* sb, uint32_t tacc, int row, int tn) {
  using namespace gk;
  const bool rv = row < p.M;
  if constexpr (EPI == EPI_SWIGLU) {
    const int f0 = tn * 128;
    const int F = p.N;
#pragma unroll 1
    for (int c = 0; c < 128; c += 32) {
      uint32_t g[32], u[32];
      tmem_ld32(tacc + c, g);
      wait_ld_dep(g);
      tmem_ld32(tacc + 128 + c, u);
      wait_ld_dep(u);
      const int col = f0 + c;
      if (!rv || col >= F) continue;
      uint16_t* gu_row = static_cast<uint16_t*>(p.c) + static_cast<long long>(row) * p.ldc;
      uint16_t* h_row = static_cast<uint16_t*>(p.h) + static_cast<long long>(row) * p.ldh;
#pragma unroll
      for (int v = 0; v < 4; ++v) {  // 8 columns per 16-byte store
        const int c8 = col + v * 8;
        if (c8 >= F) break;
        uint32_t pg[4], pu[4], ph[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          pg[j] = pack2<true>(__uint_as_float(g[v * 8 + 2 * j]), __uint_as_float(g[v * 8 + 2 * j + 1]));
          pu[j] = pack2<true>(__uint_as_float(u[v * 8 + 2 * j]), __uint_as_float(u[v * 8 + 2 * j + 1]));
        }
        // from the stored (bf16) gate and up values, as the unfused twin epilogue reads them
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 g2 = unpack2<true>(pg[j]), u2 = unpack2<true>(pu[j]);
          const int nl = c + v * 8 + 2 * j;  // column within the tile
          ph[j] = pack2<true>(silu_f(g2.x + sb[nl]) * (u2.x + sb[128 + nl]),
                              silu_f(g2.y + sb[nl + 1]) * (u2.y + sb[128 + nl + 1]));
        }
        if (c8 + 8 <= F) {
          *reinterpret_cast<uint4*>(gu_row + c8) = make_uint4(pg[0], pg[1], pg[2], pg[3]);
          *reinterpret_cast<uint4*>(gu_row + p.b_split + c8) = make_uint4(pu[0], pu[1], pu[2], pu[3]);
          *reinterpret_cast<uint4*>(h_row + c8) = make_uint4(ph[0], ph[1], ph[2], ph[3]);
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if (c8 + j >= F) continue;
            const int sh = (j & 1) * 16;
            gu_row[c8 + j] = static_cast<uint16_t>(pg[j >> 1] >> sh);
            gu_row[p.b_split + c8 + j] = static_cast<uint16_t>(pu[j >> 1] >> sh);
            h_row[c8 + j] = static_cast<uint16_t>(ph[j >> 1] >> sh);
          }
        }
      }
    }
  } else if constexpr (EPI == EPI_CE_STATS) {
    // one pass over the row's 256 logits (+ bias): running max with the first
    // index reaching it, sum of exp(x - max) rescaled when the max grows, and
    // the label's logit when the label falls in this tile
    constexpr float kLog2e = 1.4426950408889634f;
    const int n0 = tn * BN;
    const int lab = rv ? p.labels[row] : -1;
    float m = -INFINITY, ssum = 0.f, labv = 0.f;
    int am = -1;
    bool has_lab = false;
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      uint32_t r[32];
      tmem_ld32(tacc + c, r);
      wait_ld_dep(r);
      float v[32], cm = -INFINITY;
      int ci = -1;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int col = n0 + c + j;
        v[j] = col < p.N ? __uint_as_float(r[j]) + sb[c + j] : -INFINITY;
        if (v[j] > cm) {
          cm = v[j];
          ci = col;
        }
        if (col == lab) {
          labv = v[j];
          has_lab = true;
        }
      }
      if (cm > m) {
        ssum *= ex2((m - cm) * kLog2e);
        m = cm;
        am = ci;
      }
      const float mb = m * kLog2e;
#pragma unroll
      for (int j = 0; j < 32; ++j) ssum += ex2(fmaf(v[j], kLog2e, -mb));
    }
    if (rv) {
      p.ce_part[static_cast<long long>(row) * p.tiles_n + tn] = make_float4(m, ssum, __int_as_float(am), 0.f);
      if (has_lab) p.ce_lab[row] = labv;
    }
  } else if constexpr (EPI == EPI_CE_GRAD) {
    // d logits = (softmax - onehot) / rows, from the recomputed tile and the row's LSE
    constexpr float kLog2e = 1.4426950408889634f;
    const int n0 = tn * BN;
    const int lab = rv ? p.labels[row] : -1;
    const float lse2 = rv ? p.ce_lse[row] * kLog2e : 0.f;
    uint16_t* drow = static_cast<uint16_t*>(p.c) + static_cast<long long>(row) * p.ldc;
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      uint32_t r[32];
      tmem_ld32(tacc + c, r);
      wait_ld_dep(r);
      const int col = n0 + c;
      if (!rv || col >= p.N) continue;
      uint32_t w[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        float g2[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int cc = col + 2 * j + e;
          const float x = __uint_as_float(r[2 * j + e]) + sb[c + 2 * j + e];
          g2[e] = (ex2(fmaf(x, kLog2e, -lse2)) - (cc == lab ? 1.f : 0.f)) * p.ce_scale;
        }
        w[j] = pack2<true>(g2[0], g2[1]);
      }
      if (col + 32 <= p.N) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          reinterpret_cast<uint4*>(drow + col)[j] = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (col + j < p.N) drow[col + j] = static_cast<uint16_t>(w[j >> 1] >> ((j & 1) * 16));
      }
    }
  } else {
    const int n0 = tn * BN;
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      uint32_t r[32];
      tmem_ld32(tacc + c, r);
      wait_ld_dep(r);
      const int col = n0 + c;
      if (!rv || col >= p.N) continue;
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
      if constexpr (EPI == EPI_BIAS) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] += sb[c + j];
      }
      const bool whole = col + 32 <= p.N;
      if (o.out_f32) {
        float* dst = static_cast<float*>(o.c) + static_cast<long long>(row) * o.ldc + col;
        if (whole) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float4 w = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            if (o.accumulate) {
              const float4 old = reinterpret_cast<const float4*>(dst)[j];
              w.x += old.x;
              w.y += old.y;
              w.z += old.z;
              w.w += old.w;
            }
            reinterpret_cast<float4*>(dst)[j] = w;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (col + j < p.N) dst[j] = o.accumulate ? dst[j] + v[j] : v[j];
        }
      } else {
        uint16_t* dst = static_cast<uint16_t*>(o.c) + static_cast<long long>(row) * o.ldc + col;
        if (whole) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float w[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) w[e] = v[8 * j + e];
            if (o.accumulate) {
              const uint4 old = reinterpret_cast<const uint4*>(dst)[j];
              const uint32_t ow[4] = {old.x, old.y, old.z, old.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 f = unpack2<true>(ow[e]);
                w[2 * e] += f.x;
                w[2 * e + 1] += f.y;
              }
            }
            reinterpret_cast<uint4*>(dst)[j] = make_uint4(pack2<true>(w[0], w[1]), pack2<true>(w[2], w[3]),
                                                          pack2<true>(w[4], w[5]), pack2<true>(w[6], w[7]));
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (col + j >= p.N) continue;
            float w = v[j];
            if (o.accumulate) w += __uint_as_float(static_cast<uint32_t>(dst[j]) << 16);
            dst[j] = static_cast<uint16_t>(pack2<true>(w, 0.f) & 0xFFFFu);
          }
        }
      }
    }
  }
}

template <bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(gk::THREADS, 1) gemm_tc_kernel(const __grid_constant__ GemmParams p) {
  using namespace gk;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_MISC + 4);

  const int warp = warp_id(), lane = lane_id();
  const int ntiles = p.tiles_m * p.tiles_n;
  const int nk = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&p.tmA);
      prefetch_tmap(&p.tmB);
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x) {
        int tm, tn;
        gemm_tile(t, p.tiles_m, p.tiles_n, tm, tn);
        const int m0 = tm * BM;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!(ok = mbar_wait(&empty[s], ph ^ 1, abort_flag))) break;
          uint8_t* a = smem + s * STAGE_BYTES;
          uint8_t* b = a + A_BYTES;
          const int k0 = kb * BK;
          mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
          if constexpr (A_MN) {
            tma_load_2d(a, &p.tmA, &full[s], m0, k0);
            tma_load_2d(a + 8192, &p.tmA, &full[s], m0 + 64, k0);
          } else {
            tma_load_2d(a, &p.tmA, &full[s], k0, m0);
          }
          if constexpr (B_MN) {
#pragma unroll
            for (int i = 0; i < 4; ++i) tma_load_2d(b + i * 8192, &p.tmB, &full[s], gemm_b_col<EPI>(p, tn, i), k0);
          } else {
            tma_load_2d(b, &p.tmB, &full[s], k0, tn * BN);
          }
        }
      }
      if (!ok) {
        // let every copy this CTA started land before it exits
        volatile int never = 0;
        for (int j = max(0, it - STAGES); j < it; ++j) mbar_wait(&full[j % STAGES], (j / STAGES) & 1, &never);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16kind(BM, BN, true, A_MN, B_MN);
      int it = 0, tc = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x, ++tc) {
        const int ab = tc & 1;
        const uint32_t aph = (tc >> 1) & 1;
        if (!(ok = mbar_wait(&acc_empty[ab], aph ^ 1, abort_flag))) break;
        tc_fence_after();
        const uint32_t d = tmem + ab * BN;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!(ok = mbar_wait(&full[s], ph, abort_flag))) break;
          tc_fence_after();
          const uint32_t a = sbase + s * STAGE_BYTES, b = a + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            // K-major: the 16-wide K step sits 32 bytes into each 128-byte swizzled row;
            // MN-major: it is the next two 8-row swizzle atoms (2 KB), 64-column boxes 8 KB apart
            const uint64_t ad = A_MN ? sdesc_sw128(a + kk * 2048, 8192, 1024) : sdesc_sw128(a + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? sdesc_sw128(b + kk * 2048, 8192, 1024) : sdesc_sw128(b + kk * 32, 16, 1024);
            umma_ss(d, ad, bd, idesc, (kb | kk) ? 1u : 0u);
          }
          umma_commit(&empty[s]);  // the stage is free once these MMAs have read it
        }
        if (ok) umma_commit(&acc_full[ab]);
      }
      if (!ok) {
        // no MMA may still run when TMEM is released
        volatile int never = 0;
        umma_commit(drain);
        mbar_wait(drain, 0, &never);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2-5)
    const int q = warp & 3;  // TMEM lane quadrant this warp may read
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    float* sb = reinterpret_cast<float*>(smem + OFF_BIAS);
    const EpiOut out{p.c, p.ldc, p.accumulate, p.out_f32};
    int tc = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++tc) {
      int tm, tn;
      gemm_tile(t, p.tiles_m, p.tiles_n, tm, tn);
      const int ab = tc & 1;
      const uint32_t aph = (tc >> 1) & 1;
      mbar_wait(&acc_full[ab], aph, abort_flag);
      if (!epi_begin<EPI>(p, sb, tn, abort_flag)) break;
      tc_fence_after();
      const int row = tm * BM + q * 32 + lane;
      gemm_epilogue<EPI>(p, out, sb, tmem + lane_off + ab * BN, row, tn);
      tc_fence_before();
      mbar_arrive(&acc_empty[ab]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ----------------------------------------------------------------------------
// CTA-pair form (tcgen05.mma.cta_group::2): a cluster of two CTAs on the two
// SMs of a TPC computes a 256 x 256 tile.  Each CTA loads its own 128 rows of
// A and its own 128 columns of B (32 KB per 64-deep stage instead of 48 KB),
// so the 6-stage 192 KB ring covers twice the load latency of the one-CTA
// form; the leader's single MMA thread issues M=256 x N=256 MMAs that read
// both CTAs' shared memory, and each CTA's TMEM holds its 128 rows x 256
// columns (two accumulators, 512 columns).  Barriers:
//   full[s]      leader only: armed by the leader with both CTAs' bytes, the
//                peer's copies complete on it remotely;
//   empty[s]     per CTA: the leader's commit arrives on both;
//   acc_full[a]  per CTA: the leader's commit arrives on both;
//   acc_empty[a] leader only: one arrival per epilogue warp of both CTAs.
// No load is multicast.
namespace gk2 {
constexpr int BM = 128, BN = 256, BK = 64, STAGES = 6, THREADS = 192;
constexpr int A_BYTES = BM * BK * 2;         // 16 KB
constexpr int B_BYTES = (BN / 2) * BK * 2;   // 16 KB: this CTA's half of B
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int OFF_BAR = STAGES * STAGE_BYTES;
constexpr int NBAR = 2 * STAGES + 5;
constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
constexpr int OFF_BIAS = OFF_MISC + 16;
constexpr int SMEM = OFF_BIAS + 1024 + 1024;
}  // namespace gk2

template <int EPI>
TKB_DEVFN int gemm_pair_b_col(const GemmParams& p, int tn, uint32_t rank) {
  if constexpr (EPI == gk::EPI_SWIGLU) return (rank ? p.b_split : 0) + tn * 128;
  return tn * gk2::BN + static_cast<int>(rank) * 128;
}

template <bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(gk2::THREADS, 1) gemm_pair_kernel(const __grid_constant__ GemmParams p) {
  using namespace gk2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_MISC + 4);

  const int warp = warp_id(), lane = lane_id();
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster = static_cast<int>(blockIdx.x >> 1), nclusters = static_cast<int>(gridDim.x >> 1);
  const int ntiles_mn = p.tiles_m * p.tiles_n;
  const int ntiles = ntiles_mn * p.splits;  // (tile, K split) work items
  const int nk = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 8);  // 4 epilogue warps x 2 CTAs
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised and TMEM allocated before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      prefetch_tmap(&p.tmA);
      prefetch_tmap(&p.tmB);
      const uint32_t full0_leader = mapa_shared(smem_u32(&full[0]), 0);
      int it = 0;
      bool ok = true;
      for (int t = cluster; ok && t < ntiles; t += nclusters) {
        int tm, tn;
        gemm_tile(t % ntiles_mn, p.tiles_m, p.tiles_n, tm, tn);
        const int kb0 = (t / ntiles_mn) * p.kb_per_split, kb1 = min(nk, kb0 + p.kb_per_split);
        const int m0 = tm * 256 + static_cast<int>(rank) * BM;
        const int nb = gemm_pair_b_col<EPI>(p, tn, rank);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!(ok = mbar_wait(&empty[s], ph ^ 1, abort_flag))) break;
          uint8_t* a = smem + s * STAGE_BYTES;
          uint8_t* b = a + A_BYTES;
          const int k0 = kb * BK;
          const uint32_t bar = full0_leader + static_cast<uint32_t>(s) * 8u;
          if (leader) mbar_arrive_expect_tx(&full[s], 2 * STAGE_BYTES);
          if constexpr (A_MN) {
            tma_load_2d_pair(a, &p.tmA, bar, m0, k0);
            tma_load_2d_pair(a + 8192, &p.tmA, bar, m0 + 64, k0);
          } else {
            tma_load_2d_pair(a, &p.tmA, bar, k0, m0);
          }
          if constexpr (B_MN) {
            tma_load_2d_pair(b, &p.tmB, bar, nb, k0);
            tma_load_2d_pair(b + 8192, &p.tmB, bar, nb + 64, k0);
          } else {
            tma_load_2d_pair(b, &p.tmB, bar, k0, nb);
          }
        }
      }
      if (!ok) {
        // let the copies in flight land before the CTA leaves: the leader
        // waits for the stages it armed (they count both CTAs' bytes), the
        // peer gives its own copies a fixed time
        volatile int never = 0;
        if (leader) {
          for (int j = max(0, it - STAGES); j < it; ++j)
            mbar_wait_cluster(&full[j % STAGES], (j / STAGES) & 1, &never);
        } else {
          const unsigned long long t0 = globaltimer();
          while (globaltimer() - t0 < 200000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader CTA)
    if (leader && lane == 0) {
      constexpr uint32_t idesc = idesc_f16kind(2 * BM, BN, true, A_MN, B_MN);
      int it = 0, tc = 0;
      bool ok = true;
      for (int t = cluster; ok && t < ntiles; t += nclusters, ++tc) {
        const int ab = tc & 1;
        const uint32_t aph = (tc >> 1) & 1;
        if (!(ok = mbar_wait_cluster(&acc_empty[ab], aph ^ 1, abort_flag))) break;
        tc_fence_after();
        const uint32_t d = tmem + ab * BN;
        const int kb0 = (t / ntiles_mn) * p.kb_per_split, kb1 = min(nk, kb0 + p.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!(ok = mbar_wait_cluster(&full[s], ph, abort_flag))) break;
          tc_fence_after();
          const uint32_t a = sbase + s * STAGE_BYTES, b = a + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = A_MN ? sdesc_sw128(a + kk * 2048, 8192, 1024) : sdesc_sw128(a + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? sdesc_sw128(b + kk * 2048, 8192, 1024) : sdesc_sw128(b + kk * 32, 16, 1024);
            umma_pair_ss(d, ad, bd, idesc, (kb != kb0 || kk) ? 1u : 0u);
          }
          umma_pair_commit(&empty[s], 0x3);  // both CTAs' stage s is free once these MMAs read it
        }
        if (ok) umma_pair_commit(&acc_full[ab], 0x3);
      }
      if (!ok) {
        volatile int never = 0;
        umma_pair_commit(drain, 0x1);
        mbar_wait(drain, 0, &never);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2-5, both CTAs)
    const int q = warp & 3;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t acc_empty_leader = mapa_shared(smem_u32(&acc_empty[0]), 0);
    float* sb = reinterpret_cast<float*>(smem + OFF_BIAS);
    int tc = 0;
    for (int t = cluster; t < ntiles; t += nclusters, ++tc) {
      int tm, tn;
      gemm_tile(t % ntiles_mn, p.tiles_m, p.tiles_n, tm, tn);
      const int split = t / ntiles_mn;
      const int ab = tc & 1;
      const uint32_t aph = (tc >> 1) & 1;
      mbar_wait(&acc_full[ab], aph, abort_flag);
      if (!epi_begin<EPI>(p, sb, tn, abort_flag)) break;
      tc_fence_after();
      const int row = tm * 256 + static_cast<int>(rank) * BM + q * 32 + lane;
      // split-K partials go to the workspace, [split][M][N], overwritten
      const EpiOut out = p.splits > 1
                             ? EpiOut{p.ws + static_cast<long long>(split) * p.M * p.N, p.N, 0, 1}
                             : EpiOut{p.c, p.ldc, p.accumulate, p.out_f32};
      gemm_epilogue<EPI>(p, out, sb, tmem + lane_off + ab * BN, row, tn);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(acc_empty_leader + static_cast<uint32_t>(ab) * 8u);
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA leaves while the other may still signal it or read its shared memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

// C[M][N] (+)= sum over s = 0..splits-1 of ws[s][M][N], in that order (fp32).
__global__ void __launch_bounds__(256) gemm_splitk_reduce_kernel(const float* __restrict__ ws, int splits, int M,
                                                                 int N, float* __restrict__ c, long long ldc,
                                                                 int accumulate) {
  const long long MN = static_cast<long long>(M) * N;
  if ((N & 3) == 0 && (ldc & 3) == 0) {
    for (long long i = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 4; i < MN;
         i += static_cast<long long>(gridDim.x) * blockDim.x * 4) {
      float4 acc = reinterpret_cast<const float4*>(ws + i)[0];
      for (int s = 1; s < splits; ++s) {
        const float4 v = reinterpret_cast<const float4*>(ws + s * MN + i)[0];
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      const long long r = i / N, col = i % N;
      float4* dst = reinterpret_cast<float4*>(c + r * ldc + col);
      if (accumulate) {
        const float4 o = *dst;
        acc.x += o.x;
        acc.y += o.y;
        acc.z += o.z;
        acc.w += o.w;
      }
      *dst = acc;
    }
  } else {
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < MN;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
      float acc = ws[i];
      for (int s = 1; s < splits; ++s) acc += ws[s * MN + i];
      float* dst = c + (i / N) * ldc + i % N;
      *dst = accumulate ? *dst + acc : acc;
    }
  }
}

// One warp per row: LSE = M + ln(sum_t s_t exp(m_t - M)) over the row's tile
// partials (M = max_t m_t); the argmax is the first index of the first tile
// reaching M (each tile kept its first maximum).
__global__ void __launch_bounds__(256) ce_combine_kernel(const float4* __restrict__ part, int tiles_n,
                                                         const float* __restrict__ lab_logit,
                                                         const int* __restrict__ labels, float* __restrict__ lse,
                                                         float* __restrict__ row_loss, int* __restrict__ correct,
                                                         int rows, float inv_rows) {
  const int row = static_cast<int>((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float4* pr = part + static_cast<long long>(row) * tiles_n;
  float m = -INFINITY;
  int first = 0x7FFFFFFF;
  for (int t = lane; t < tiles_n; t += 32) {
    const float mt = pr[t].x;
    if (mt > m) {
      m = mt;
      first = t;
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const int f2 = __shfl_xor_sync(0xffffffffu, first, o);
    if (m2 > m || (m2 == m && f2 < first)) {
      m = m2;
      first = f2;
    }
  }
  float s = 0.f;
  for (int t = lane; t < tiles_n; t += 32) {
    const float4 v = pr[t];
    s += v.y * ex2((v.x - m) * 1.4426950408889634f);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) {
    const float l = m + lg2(s) * 0.6931471805599453f;
    lse[row] = l;
    // -ln(max(p_label, 1e-7)) = min(LSE - label logit, -ln(1e-7))
    row_loss[row] = fminf(l - lab_logit[row], 16.11809565095832f) * inv_rows;
    const int am = __float_as_int(pr[first].z);
    if (correct && am == labels[row]) atomicAdd(correct, 1);
  }
}

cudaError_t ce_combine(const float4* part, int tiles_n, const float* lab_logit, const int* labels, float* lse,
                       float* row_loss, int* correct, int rows, float inv_rows, cudaStream_t stream) {
  const unsigned grid = static_cast<unsigned>((static_cast<long long>(rows) * 32 + 255) / 256);
  ce_combine_kernel<<<grid, 256, 0, stream>>>(part, tiles_n, lab_logit, labels, lse, row_loss, correct, rows,
                                              inv_rows);
  return cudaGetLastError();
}

cudaError_t gemm_splitk_reduce(const GemmParams& p, cudaStream_t stream) {
  const long long MN = static_cast<long long>(p.M) * p.N;
  long long blocks = (MN / 4 + 255) / 256 + 1;
  if (blocks > 148LL * 8) blocks = 148LL * 8;
  const unsigned grid = static_cast<unsigned>(blocks);
  gemm_splitk_reduce_kernel<<<grid, 256, 0, stream>>>(p.ws, p.splits, p.M, p.N, static_cast<float*>(p.c), p.ldc,
                                                      p.accumulate);
  return cudaGetLastError();
}

template <bool A_MN, bool B_MN, int EPI>
static cudaError_t launch_gemm_pair(const GemmParams& p, cudaStream_t stream) {
  auto kern = gemm_pair_kernel<A_MN, B_MN, EPI>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, gk2::SMEM);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int ntiles = p.tiles_m * p.tiles_n * p.splits;
  const int nclusters = min(ntiles, sms / 2);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * nclusters));
  cfg.blockDim = dim3(gk2::THREADS);
  cfg.dynamicSmemBytes = gk2::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

template <bool A_MN, bool B_MN, int EPI>
static cudaError_t launch_gemm(const GemmParams& p, cudaStream_t stream) {
  auto kern = gemm_tc_kernel<A_MN, B_MN, EPI>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, gk::SMEM);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int ntiles = p.tiles_m * p.tiles_n;
  const unsigned grid = static_cast<unsigned>(min(ntiles, sms));
  kern<<<grid, gk::THREADS, gk::SMEM, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t gemm_pair_tc(const GemmParams& p, bool a_mn, bool b_mn, int epi, cudaStream_t stream) {
  if (epi == gk::EPI_CE_STATS || epi == gk::EPI_CE_GRAD) {
    if (a_mn || !b_mn) return cudaErrorInvalidValue;
    return epi == gk::EPI_CE_STATS ? launch_gemm_pair<false, true, gk::EPI_CE_STATS>(p, stream)
                                   : launch_gemm_pair<false, true, gk::EPI_CE_GRAD>(p, stream);
  }
  if (epi == gk::EPI_SWIGLU) {
    if (a_mn || !b_mn) return cudaErrorInvalidValue;
    return launch_gemm_pair<false, true, gk::EPI_SWIGLU>(p, stream);
  }
  if (epi == gk::EPI_BIAS) {
    if (!a_mn && b_mn) return launch_gemm_pair<false, true, gk::EPI_BIAS>(p, stream);
    if (!a_mn && !b_mn) return launch_gemm_pair<false, false, gk::EPI_BIAS>(p, stream);
    return cudaErrorInvalidValue;
  }
  if (!a_mn && b_mn) return launch_gemm_pair<false, true, gk::EPI_STORE>(p, stream);
  if (!a_mn && !b_mn) return launch_gemm_pair<false, false, gk::EPI_STORE>(p, stream);
  if (a_mn && b_mn) return launch_gemm_pair<true, true, gk::EPI_STORE>(p, stream);
  return launch_gemm_pair<true, false, gk::EPI_STORE>(p, stream);
}

cudaError_t gemm_tc(const GemmParams& p, bool a_mn, bool b_mn, int epi, cudaStream_t stream) {
  if (epi == gk::EPI_SWIGLU) {
    if (a_mn || !b_mn) return cudaErrorInvalidValue;
    return launch_gemm<false, true, gk::EPI_SWIGLU>(p, stream);
  }
  if (epi == gk::EPI_BIAS) {
    if (!a_mn && b_mn) return launch_gemm<false, true, gk::EPI_BIAS>(p, stream);
    if (!a_mn && !b_mn) return launch_gemm<false, false, gk::EPI_BIAS>(p, stream);
    return cudaErrorInvalidValue;
  }
  if (!a_mn && b_mn) return launch_gemm<false, true, gk::EPI_STORE>(p, stream);
  if (!a_mn && !b_mn) return launch_gemm<false, false, gk::EPI_STORE>(p, stream);
  if (a_mn && b_mn) return launch_gemm<true, true, gk::EPI_STORE>(p, stream);
  return launch_gemm<true, false, gk::EPI_STORE>(p, stream);
}

}  // namespace tkb
