// rows.cu -- HBM-bound fused row kernels of the hot path, for sm_100a.
//
// These replace the NVRTC "plasma group" kernels the reference emits from
// src/tkm_codegen.c (RMSNorm group, twin SwiGLU epilogue, QKV-prep with RoPE)
// and its static softmax / loss kernels (src/tkm_gpu.cu:600-682).  Design:
//   * one 256-thread block per row (grid-stride over rows) for row reductions,
//     the row kept in registers so HBM is read and written exactly once;
//   * 16-byte vector accesses (8 x 16-bit or 2 x float4) when the row length
//     allows, 2-element accesses otherwise (the reference requires even C);
//   * block-wide reductions (warp shuffles + shared memory) over the full row;
//   * column reductions for parameter gradients as per-block fp32 partials
//     reduced by a second kernel (deterministic, no atomics).
#include "tkb_common.cuh"

// Pairs (of the four in each 16-byte vector) whose exponentials the
// bulk-staged softmax loss computes with the FMA-pipe polynomial
// (ex2_poly_f2, relative error 1.02e-4) instead of ex2, to offload the MUFU
// unit the kernel keeps busy.  Same box, 8192 x 32000 bf16: 0.2222 ms with
// none, 0.2181 with one, 0.2245 with two in the register form that preceded
// the bulk-staged kernel; 189.4 us with one and 189.5 with two in the
// bulk-staged kernel.
#ifndef TKB_CE_EMU
#define TKB_CE_EMU 1
#endif

namespace tkb {

// ------------------------------------------------------------------ loads
template <typename T>
struct Elem;
template <>
struct Elem<float> {
  static TKB_DEVFN float ld(const float* p) { return *p; }
  static TKB_DEVFN void st(float* p, float v) { *p = v; }
};
template <>
struct Elem<__nv_bfloat16> {
  static TKB_DEVFN float ld(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  static TKB_DEVFN void st(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
};
template <>
struct Elem<__half> {
  static TKB_DEVFN float ld(const __half* p) { return __half2float(*p); }
  static TKB_DEVFN void st(__half* p, float v) { *p = __float2half_rn(v); }
};

// VEC consecutive elements <-> floats.  VEC = 8 uses 16-byte transactions.
template <typename T, int VEC>
TKB_DEVFN void ldv(const T* p, float (&f)[VEC]) {
  if constexpr (VEC == 8 && sizeof(T) == 2) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 t;
      if constexpr (std::is_same<T, __nv_bfloat16>::value) t = unpack2<true>(w[i]);
      else t = unpack2<false>(w[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  } else if constexpr (VEC == 8 && sizeof(T) == 4) {
    const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) f[i] = Elem<T>::ld(p + i);
  }
}
template <typename T, int VEC>
TKB_DEVFN void stv(T* p, const float (&f)[VEC]) {
  if constexpr (VEC == 8 && sizeof(T) == 2) {
    uint4 u;
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      u.x = pack2<true>(f[0], f[1]); u.y = pack2<true>(f[2], f[3]);
      u.z = pack2<true>(f[4], f[5]); u.w = pack2<true>(f[6], f[7]);
    } else {
      u.x = pack2<false>(f[0], f[1]); u.y = pack2<false>(f[2], f[3]);
      u.z = pack2<false>(f[4], f[5]); u.w = pack2<false>(f[6], f[7]);
    }
    *reinterpret_cast<uint4*>(p) = u;
  } else if constexpr (VEC == 8 && sizeof(T) == 4) {
    reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) Elem<T>::st(p + i, f[i]);
  }
}
// Round a float through T (what a store followed by a load would give).
template <typename T>
TKB_DEVFN float rnd(float v) {
  if constexpr (std::is_same<T, float>::value) return v;
  else if constexpr (std::is_same<T, __nv_bfloat16>::value) return __bfloat162float(__float2bfloat16_rn(v));
  else return __half2float(__float2half_rn(v));
}
template <int VEC>
TKB_DEVFN void ldf(const float* p, float (&f)[VEC]) {
  if constexpr (VEC == 8) {
    const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) f[i] = p[i];
  }
}

constexpr int NT = 256;  // threads per row block

TKB_DEVFN float warp_sum(float v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  return v;
}
TKB_DEVFN float warp_max(float v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, m));
  return v;
}
// Block-wide sum for NT threads; `sh` holds >= 32 floats; safe to call repeatedly.
TKB_DEVFN float block_sum(float v, float* sh) {
  v = warp_sum(v);
  __syncthreads();
  if (lane_id() == 0) sh[warp_id()] = v;
  __syncthreads();
  float t = lane_id() < NT / 32 ? sh[lane_id()] : 0.f;
  return warp_sum(t);
}
TKB_DEVFN float block_max(float v, float* sh) {
  v = warp_max(v);
  __syncthreads();
  if (lane_id() == 0) sh[warp_id()] = v;
  __syncthreads();
  float t = lane_id() < NT / 32 ? sh[lane_id()] : -INFINITY;
  return warp_max(t);
}

// Block-wide reductions for an NTH-thread block (NTH a multiple of 32, <= 1024).
template <int NTH>
TKB_DEVFN float block_sum_n(float v, float* sh) {
  v = warp_sum(v);
  __syncthreads();
  if (lane_id() == 0) sh[warp_id()] = v;
  __syncthreads();
  float t = lane_id() < NTH / 32 ? sh[lane_id()] : 0.f;
  return warp_sum(t);
}

template <int NTH>
TKB_DEVFN float block_max_n(float v, float* sh) {
  v = warp_max(v);
  __syncthreads();
  if (lane_id() == 0) sh[warp_id()] = v;
  __syncthreads();
  float t = lane_id() < NTH / 32 ? sh[lane_id()] : -INFINITY;
  return warp_max(t);
}

static int row_grid(int rows, int per_sm) {
  const int cap = 148 * per_sm;
  return rows < cap ? (rows < 1 ? 1 : rows) : cap;
}

// ============================================================ Add + RMSNorm
// s = x + r, istd = 1/sqrt(mean(s^2) + eps), y = s * istd * gamma
// (RMSNorm spec src/tkm_registry.c:228-238, Add spec 435-439).
template <typename T, int VEC, int MAXV>
__global__ void __launch_bounds__(NT) add_rmsnorm_fwd_kernel(const T* __restrict__ x, const T* __restrict__ r,
                                                             T* __restrict__ s, T* __restrict__ y,
                                                             const float* __restrict__ gamma,
                                                             float* __restrict__ istd, int rows, int C, float eps) {
  __shared__ float sh[32];
  const int nvec = C / VEC;
  const float invC = 1.0f / static_cast<float>(C);
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    const long long base = static_cast<long long>(row) * C;
    float v[MAXV][VEC];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int vi = threadIdx.x + i * NT;
      if (vi < nvec) {
        ldv<T, VEC>(x + base + vi * VEC, v[i]);
        if (r) {
          float rr[VEC];
          ldv<T, VEC>(r + base + vi * VEC, rr);
#pragma unroll
          for (int e = 0; e < VEC; ++e) v[i][e] = rnd<T>(v[i][e] + rr[e]);
          if (s) stv<T, VEC>(s + base + vi * VEC, v[i]);
        }
#pragma unroll
        for (int e = 0; e < VEC; ++e) ss = fmaf(v[i][e], v[i][e], ss);
      }
    }
    ss = block_sum(ss, sh);
    const float is = 1.0f / sqrtf(ss * invC + eps);
    if (threadIdx.x == 0 && istd) istd[row] = is;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int vi = threadIdx.x + i * NT;
      if (vi < nvec) {
        float g[VEC];
        ldf<VEC>(gamma + vi * VEC, g);
#pragma unroll
        for (int e = 0; e < VEC; ++e) v[i][e] = v[i][e] * is * g[e];
        stv<T, VEC>(y + base + vi * VEC, v[i]);
      }
    }
  }
}

// dx = istd*(gamma*dy - xh*mean(gamma*dy*xh)) + ds_skip, xh = s*istd;
// dgamma partial per block = sum over its rows of dy*xh   (src/tkm_registry.c:239-245).
template <typename T, int VEC, int MAXV>
__global__ void __launch_bounds__(NT) add_rmsnorm_bwd_kernel(const T* __restrict__ dy, const T* __restrict__ s,
                                                             const float* __restrict__ gamma,
                                                             const float* __restrict__ istd,
                                                             const T* __restrict__ ds_skip, T* __restrict__ dx,
                                                             float* __restrict__ partial, int rows, int C) {
  __shared__ float sh[32];
  const int nvec = C / VEC;
  const float invC = 1.0f / static_cast<float>(C);
  float g[MAXV][VEC], dg[MAXV][VEC];
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int vi = threadIdx.x + i * NT;
#pragma unroll
    for (int e = 0; e < VEC; ++e) dg[i][e] = 0.f;
    if (vi < nvec) ldf<VEC>(gamma + vi * VEC, g[i]);
  }
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    const long long base = static_cast<long long>(row) * C;
    const float is = istd[row];
    float d[MAXV][VEC], xh[MAXV][VEC];
    float m2 = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int vi = threadIdx.x + i * NT;
      if (vi < nvec) {
        ldv<T, VEC>(dy + base + vi * VEC, d[i]);
        ldv<T, VEC>(s + base + vi * VEC, xh[i]);
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          xh[i][e] *= is;
          m2 = fmaf(d[i][e] * g[i][e], xh[i][e], m2);
          dg[i][e] = fmaf(d[i][e], xh[i][e], dg[i][e]);
        }
      }
    }
    m2 = block_sum(m2, sh) * invC;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int vi = threadIdx.x + i * NT;
      if (vi < nvec) {
        float o[VEC];
        if (ds_skip) ldv<T, VEC>(ds_skip + base + vi * VEC, o);
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          const float v = is * (d[i][e] * g[i][e] - xh[i][e] * m2);
          o[e] = ds_skip ? o[e] + v : v;
        }
        stv<T, VEC>(dx + base + vi * VEC, o);
      }
    }
  }
  if (partial) {
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int vi = threadIdx.x + i * NT;
      if (vi < nvec) {
        float* pp = partial + static_cast<long long>(blockIdx.x) * C + vi * VEC;
#pragma unroll
        for (int e = 0; e < VEC; ++e) pp[e] = dg[i][e];
      }
    }
  }
}

// out[c] += sum_b partial[b][c]  (fixed order: deterministic)
__global__ void __launch_bounds__(256) column_reduce_kernel(const float* __restrict__ partial, int nblk, int C,
                                                            float* __restrict__ out0, float* __restrict__ out1,
                                                            int split) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  float acc = 0.f;
  for (int b = 0; b < nblk; ++b) acc += partial[static_cast<long long>(b) * C + c];
  if (c < split) {
    if (out0) out0[c] += acc;
  } else {
    if (out1) out1[c - split] += acc;
  }
}

// ============================================================ SwiGLU twin epilogue
// gu [rows][2F] (gate | up), h = silu(g + bg) * (u + bu)
// (src/tkm_codegen.c:511-518; SiLU spec src/tkm_registry.c:272-278)
TKB_DEVFN float sigmoidf_(float a) { return 1.0f / (1.0f + expf(-a)); }

// Block (bx, by): columns [bx*NT*VEC, ...), rows by, by+gridDim.y, ...
template <typename T, int VEC>
__global__ void __launch_bounds__(NT) swiglu_fwd_kernel(const T* __restrict__ gu, const float* __restrict__ bg,
                                                        const float* __restrict__ bu, T* __restrict__ h, int rows,
                                                        int F) {
  const int c0 = (blockIdx.x * NT + threadIdx.x) * VEC;
  if (c0 >= F) return;
  float b1[VEC], b2[VEC];
#pragma unroll
  for (int e = 0; e < VEC; ++e) { b1[e] = 0.f; b2[e] = 0.f; }
  if (bg) ldf<VEC>(bg + c0, b1);
  if (bu) ldf<VEC>(bu + c0, b2);
  for (int row = blockIdx.y; row < rows; row += gridDim.y) {
    const long long gb = static_cast<long long>(row) * 2 * F;
    float a[VEC], u[VEC], o[VEC];
    ldv<T, VEC>(gu + gb + c0, a);
    ldv<T, VEC>(gu + gb + F + c0, u);
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const float av = a[e] + b1[e];
      o[e] = av * sigmoidf_(av) * (u[e] + b2[e]);
    }
    stv<T, VEC>(h + static_cast<long long>(row) * F + c0, o);
  }
}

// dg = dh*b*sig(a)*(1 + a*(1 - sig(a))), du = dh*silu(a)  (src/tkm_registry.c:275-277, codegen 592-597)
template <typename T, int VEC>
__global__ void __launch_bounds__(NT) swiglu_bwd_kernel(const T* __restrict__ dh, const T* __restrict__ gu,
                                                        const float* __restrict__ bg, const float* __restrict__ bu,
                                                        T* __restrict__ dgu, float* __restrict__ partial, int rows,
                                                        int F) {
  const int c0 = (blockIdx.x * NT + threadIdx.x) * VEC;
  if (c0 >= F) return;
  float b1[VEC], b2[VEC], sg[VEC], su[VEC];
#pragma unroll
  for (int e = 0; e < VEC; ++e) { b1[e] = 0.f; b2[e] = 0.f; sg[e] = 0.f; su[e] = 0.f; }
  if (bg) ldf<VEC>(bg + c0, b1);
  if (bu) ldf<VEC>(bu + c0, b2);
  for (int row = blockIdx.y; row < rows; row += gridDim.y) {
    const long long gb = static_cast<long long>(row) * 2 * F;
    float a[VEC], u[VEC], d[VEC], og[VEC], ou[VEC];
    ldv<T, VEC>(gu + gb + c0, a);
    ldv<T, VEC>(gu + gb + F + c0, u);
    ldv<T, VEC>(dh + static_cast<long long>(row) * F + c0, d);
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const float av = a[e] + b1[e], bv = u[e] + b2[e];
      const float sgm = sigmoidf_(av);
      og[e] = d[e] * bv * sgm * (1.0f + av * (1.0f - sgm));
      ou[e] = d[e] * av * sgm;
      sg[e] += og[e];
      su[e] += ou[e];
    }
    stv<T, VEC>(dgu + gb + c0, og);
    stv<T, VEC>(dgu + gb + F + c0, ou);
  }
  if (partial) {
    float* pp = partial + static_cast<long long>(blockIdx.y) * 2 * F;
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      pp[c0 + e] = sg[e];
      pp[F + c0 + e] = su[e];
    }
  }
}

// ============================================================ QKV prep (bias + QKNorm + RoPE)
// src/tkm_codegen.c:211-295 with the rotation of 43-70.  One block per row
// (grid-stride), threads over 8-column vectors; a vector never straddles a head.
struct RopeTable {
  double inv_freq[64];  // per pair index within a head (D/2 <= 64)
};

TKB_DEVFN void rope_cs(int pos, double invf, float& sn, float& cs) {
  double a = static_cast<double>(pos) * invf;
  a -= 6.283185307179586 * floor(a * 0.15915494309189535);
  sincosf(static_cast<float>(a), &sn, &cs);
}

template <typename T>
__global__ void __launch_bounds__(NT) qkv_prep_fwd_kernel(const T* __restrict__ in, const float* __restrict__ bias,
                                                          const float* __restrict__ gain, T* __restrict__ out,
                                                          float* __restrict__ save_istd, int rows, int S, int Hq,
                                                          int Hkv, int D, int has_qknorm, int has_rope,
                                                          const RopeTable tab) {
  const int C = (Hq + 2 * Hkv) * D, nqk = Hq + Hkv, nvec = C / 8;
  const int grp = D / 8;  // threads per head
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    const int pos = row % S;
    const long long base = static_cast<long long>(row) * C;
    for (int v0 = 0; v0 < nvec; v0 += NT) {
      const int vi = v0 + threadIdx.x;
      const bool act = vi < nvec;
      const int c = vi * 8, hd = c / D;
      float v[8];
      if (act) {
        ldv<T, 8>(in + base + c, v);
        if (bias) {
          float bb[8];
          ldf<8>(bias + c, bb);
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] += bb[e];
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = 0.f;
      }
      if (has_qknorm) {
        // heads are aligned to groups of `grp` consecutive lanes (D/8 divides 32 or equals 16)
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(v[e], v[e], ss);
        for (int m = grp >> 1; m >= 1; m >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, m);
        if (act && hd < nqk) {
          const float is = 1.0f / sqrtf(ss / static_cast<float>(D) + 1e-5f);
          if (save_istd && (c % D) == 0) save_istd[static_cast<long long>(row) * nqk + hd] = is;
          float gg[8];
          if (gain) ldf<8>(gain + c, gg);
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] = v[e] * is * (gain ? gg[e] : 1.0f);
        }
      }
      if (act && has_rope && hd < nqk) {
        const int pi0 = (c % D) >> 1;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float sn, cs;
          rope_cs(pos, tab.inv_freq[pi0 + e], sn, cs);
          const float x0 = v[2 * e], x1 = v[2 * e + 1];
          v[2 * e] = x0 * cs - x1 * sn;
          v[2 * e + 1] = x0 * sn + x1 * cs;
        }
      }
      if (act) stv<T, 8>(out + base + c, v);
    }
  }
}

// din += J^T dout; dbias partial, dgain partial per block.
template <typename T>
__global__ void __launch_bounds__(NT) qkv_prep_bwd_kernel(const T* __restrict__ dout, const T* __restrict__ in,
                                                          const float* __restrict__ bias,
                                                          const float* __restrict__ gain,
                                                          const float* __restrict__ save_istd, T* __restrict__ din,
                                                          float* __restrict__ partial, int rows, int S, int Hq,
                                                          int Hkv, int D, int has_qknorm, int has_rope,
                                                          const RopeTable tab) {
  const int C = (Hq + 2 * Hkv) * D, nqk = Hq + Hkv, nvec = C / 8;
  const int grp = D / 8;
  // partial layout per block: [dbias C][dgain nqk*D]
  const long long pstride = static_cast<long long>(C) + static_cast<long long>(nqk) * D;
  for (int v0 = 0; v0 < nvec; v0 += NT) {
    const int vi = v0 + threadIdx.x;
    const bool act = vi < nvec;
    const int c = vi * 8, hd = c / D;
    float accb[8], accg[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) { accb[e] = 0.f; accg[e] = 0.f; }
    for (int row = blockIdx.x; row < rows; row += gridDim.x) {
      const int pos = row % S;
      const long long base = static_cast<long long>(row) * C;
      float dy[8];
      if (act) ldv<T, 8>(dout + base + c, dy);
      else {
#pragma unroll
        for (int e = 0; e < 8; ++e) dy[e] = 0.f;
      }
      if (act && has_rope && hd < nqk) {
        const int pi0 = (c % D) >> 1;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float sn, cs;
          rope_cs(pos, tab.inv_freq[pi0 + e], sn, cs);
          const float y0 = dy[2 * e], y1 = dy[2 * e + 1];
          dy[2 * e] = y0 * cs + y1 * sn;
          dy[2 * e + 1] = -y0 * sn + y1 * cs;
        }
      }
      if (has_qknorm) {
        float xh[8], gg[8], m2 = 0.f;
        float is = 0.f;
        if (act && hd < nqk) {
          is = save_istd[static_cast<long long>(row) * nqk + hd];
          ldv<T, 8>(in + base + c, xh);
          float bb[8];
          if (bias) ldf<8>(bias + c, bb);
          if (gain) ldf<8>(gain + c, gg);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            xh[e] = (xh[e] + (bias ? bb[e] : 0.f)) * is;
            if (!gain) gg[e] = 1.f;
            accg[e] = fmaf(dy[e], xh[e], accg[e]);
            m2 = fmaf(dy[e] * gg[e], xh[e], m2);
          }
        }
        for (int m = grp >> 1; m >= 1; m >>= 1) m2 += __shfl_xor_sync(0xffffffffu, m2, m);
        if (act && hd < nqk) {
          m2 /= static_cast<float>(D);
#pragma unroll
          for (int e = 0; e < 8; ++e) dy[e] = is * (dy[e] * gg[e] - xh[e] * m2);
        }
      }
      if (act) {
        float prev[8];
        ldv<T, 8>(din + base + c, prev);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          accb[e] += dy[e];
          prev[e] += dy[e];
        }
        stv<T, 8>(din + base + c, prev);
      }
    }
    if (act && partial) {
      float* pp = partial + static_cast<long long>(blockIdx.x) * pstride;
#pragma unroll
      for (int e = 0; e < 8; ++e) pp[c + e] = accb[e];
      if (hd < nqk) {
#pragma unroll
        for (int e = 0; e < 8; ++e) pp[C + c + e] = accg[e];
      }
    }
  }
}

// ============================================================ softmax and softmax losses
// Row kept in registers: MAXV vectors of VEC per thread (C <= NT*VEC*MAXV).
template <typename T, int VEC, int MAXV, int NTH>
__global__ void __launch_bounds__(NTH) softmax_fwd_kernel(const T* __restrict__ x, T* __restrict__ p, int rows, int C) {
  __shared__ float sh[32];
  const int nvec = C / VEC;
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    const long long base = static_cast<long long>(row) * C;
    float v[MAXV][VEC];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int vi = threadIdx.x + i * NTH;
      if (vi < nvec) {
        ldv<T, VEC>(x + base + vi * VEC, v[i]);
#pragma unroll
        for (int e = 0; e < VEC; ++e) mx = fmaxf(mx, v[i][e]);
      }
    }
    mx = block_max_n<NTH>(mx, sh);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int vi = threadIdx.x + i * NTH;
      if (vi < nvec) {
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          v[i][e] = expf(v[i][e] - mx);
          sum += v[i][e];
        }
      }
    }
    const float inv = 1.0f / block_sum_n<NTH>(sum, sh);
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int vi = threadIdx.x + i * NTH;
      if (vi < nvec) {
#pragma unroll
        for (int e = 0; e < VEC; ++e) v[i][e] *= inv;
        stv<T, VEC>(p + base + vi * VEC, v[i]);
      }
    }
  }
}

// dx += p * (dp - <p, dp>)   (src/tkm_gpu.cu:615-630)
template <typename T, int VEC, int MAXV, int NTH>
__global__ void __launch_bounds__(NTH) softmax_bwd_kernel(const T* __restrict__ p, const T* __restrict__ dp,
                                                         T* __restrict__ dx, int rows, int C) {
  __shared__ float sh[32];
  const int nvec = C / VEC;
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    const long long base = static_cast<long long>(row) * C;
    float pv[MAXV][VEC], dv[MAXV][VEC];
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int vi = threadIdx.x + i * NTH;
      if (vi < nvec) {
        ldv<T, VEC>(p + base + vi * VEC, pv[i]);
        ldv<T, VEC>(dp + base + vi * VEC, dv[i]);
#pragma unroll
        for (int e = 0; e < VEC; ++e) dot = fmaf(pv[i][e], dv[i][e], dot);
      }
    }
    dot = block_sum_n<NTH>(dot, sh);
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int vi = threadIdx.x + i * NTH;
      if (vi < nvec) {
        float o[VEC];
        ldv<T, VEC>(dx + base + vi * VEC, o);
#pragma unroll
        for (int e = 0; e < VEC; ++e) o[e] += pv[i][e] * (dv[i][e] - dot);
        stv<T, VEC>(dx + base + vi * VEC, o);
      }
    }
  }
}

// Fused softmax loss forward + backward for one row per block
// (src/tkm_gpu.cu:632-682): kind 0 CE, 1 focal(gamma), 2 Brier.
// row_loss[row] receives the row's loss contribution already divided by rows.
template <typename T, int VEC, int MAXV, int NTH>
__global__ void __launch_bounds__(NTH) softmax_loss_kernel(const T* __restrict__ logits,
                                                          const int32_t* __restrict__ labels, T* __restrict__ dlogits,
                                                          float* __restrict__ row_loss, int* __restrict__ correct,
                                                          int rows, int C, int kind, float gamma) {
  __shared__ float sh[32];
  __shared__ int shi[32];
  const int nvec = C / VEC;
  const float inv_rows = 1.0f / static_cast<float>(rows);
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    const long long base = static_cast<long long>(row) * C;
    const int y = labels ? labels[row] : 0;
    float v[MAXV][VEC];
    float mx = -INFINITY;
    int arg = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int vi = threadIdx.x + i * NTH;
      if (vi < nvec) {
        ldv<T, VEC>(logits + base + vi * VEC, v[i]);
#pragma unroll
        for (int e = 0; e < VEC; ++e)
          if (v[i][e] > mx) { mx = v[i][e]; arg = vi * VEC + e; }
      }
    }
    // (max, first index) reduction
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, mx, m);
      const int oa = __shfl_xor_sync(0xffffffffu, arg, m);
      if (om > mx || (om == mx && oa < arg)) { mx = om; arg = oa; }
    }
    __syncthreads();
    if (lane_id() == 0) { sh[warp_id()] = mx; shi[warp_id()] = arg; }
    __syncthreads();
    mx = lane_id() < NTH / 32 ? sh[lane_id()] : -INFINITY;
    arg = lane_id() < NTH / 32 ? shi[lane_id()] : 0x7fffffff;
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, mx, m);
      const int oa = __shfl_xor_sync(0xffffffffu, arg, m);
      if (om > mx || (om == mx && oa < arg)) { mx = om; arg = oa; }
    }
    float sum = 0.f, xy = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int vi = threadIdx.x + i * NTH;
      if (vi < nvec) {
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          if (vi * VEC + e == y) xy = v[i][e];
          v[i][e] = expf(v[i][e] - mx);
          sum += v[i][e];
        }
      }
    }
    sum = block_sum_n<NTH>(sum, sh);
    xy = block_sum_n<NTH>(xy, sh);  // exactly one thread holds the label logit
    const float inv_sum = 1.0f / sum;
    float pt = expf(xy - mx) * inv_sum;
    pt = fmaxf(pt, 1e-7f);
    const float fw = powf(1.0f - pt, gamma);
    const float fgs = kind == 1 ? fw - gamma * pt * powf(1.0f - pt, gamma - 1.0f) * logf(pt) : 1.0f;
    float bdot = 0.f, brier = 0.f;
    if (kind == 2) {
#pragma unroll
      for (int i = 0; i < MAXV; ++i) {
        const int vi = threadIdx.x + i * NTH;
        if (vi < nvec) {
#pragma unroll
          for (int e = 0; e < VEC; ++e) {
            const float pc = v[i][e] * inv_sum, t = (vi * VEC + e == y) ? 1.f : 0.f;
            bdot += pc * (pc - t);
            brier += (pc - t) * (pc - t);
          }
        }
      }
      bdot = block_sum_n<NTH>(bdot, sh);
      brier = block_sum_n<NTH>(brier, sh);
    }
    if (threadIdx.x == 0) {
      float lr;
      if (kind == 0) lr = -logf(pt) * inv_rows;
      else if (kind == 1) lr = -fw * logf(pt) * inv_rows;
      else lr = brier / static_cast<float>(C) * inv_rows;
      if (row_loss) row_loss[row] = lr;
      if (correct && arg == y) atomicAdd(correct, 1);
    }
    if (dlogits) {
      const float k2 = 2.0f / static_cast<float>(C);
#pragma unroll
      for (int i = 0; i < MAXV; ++i) {
        const int vi = threadIdx.x + i * NTH;
        if (vi < nvec) {
          float o[VEC];
#pragma unroll
          for (int e = 0; e < VEC; ++e) {
            const float pc = v[i][e] * inv_sum, t = (vi * VEC + e == y) ? 1.f : 0.f;
            float gr;
            if (kind == 0) gr = pc - t;
            else if (kind == 1) gr = fgs * (pc - t);
            else gr = k2 * pc * ((pc - t) - bdot);
            o[e] = gr * inv_rows;
          }
          stv<T, VEC>(dlogits + base + vi * VEC, o);
        }
      }
    }
  }
}

// Streaming variant for wide rows (vocabularies): two passes over the row
// instead of holding it in registers, so a 256-thread block per row keeps
// its registers low.  Pass 1 keeps per-thread online statistics (running max
// m, s1 = sum e^(x-m), s2 = sum e^(2(x-m)) for the Brier score, first-index
// argmax, the label logit); pass 2 reads the row again and writes the
// gradient, re-reading global memory (mostly L2) with eight rows in flight
// per SM.  Used for rows wider than 72 KB; narrower wide rows take
// softmax_loss_bulk_kernel (16-bit, 8192-32768 wide) or
// softmax_loss_staged_kernel.  Same results as softmax_loss_kernel
// (src/tkm_gpu.cu:632-682).
template <typename T, int VEC>
__global__ void __launch_bounds__(256) softmax_loss_stream_kernel(const T* __restrict__ logits,
                                                                  const int32_t* __restrict__ labels,
                                                                  T* __restrict__ dlogits, float* __restrict__ row_loss,
                                                                  int* __restrict__ correct, int rows, int C, int kind,
                                                                  float gamma) {
  constexpr int NTH = 256;
  __shared__ float shm[NTH / 32], sh1[NTH / 32], sh2[NTH / 32], shx[NTH / 32];
  __shared__ int sha[NTH / 32];
  const int nvec = C / VEC;
  const float inv_rows = 1.0f / static_cast<float>(rows);
  const bool brier = kind == 2;
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    const long long base = static_cast<long long>(row) * C;
    const int y = labels ? labels[row] : 0;
    const T* src = logits + base;
    float m = -INFINITY, s1 = 0.f, s2 = 0.f, xy = 0.f, best = -INFINITY;
    int arg = 0x7fffffff;
    for (int vi = threadIdx.x; vi < nvec; vi += NTH) {
      float v[VEC];
      ldv<T, VEC>(src + static_cast<long long>(vi) * VEC, v);
      float vm = v[0];
      int va = 0;
#pragma unroll
      for (int e = 1; e < VEC; ++e)
        if (v[e] > vm) { vm = v[e]; va = e; }
      if (vm > best) { best = vm; arg = vi * VEC + va; }
      if (y >= vi * VEC && y < vi * VEC + VEC) {
#pragma unroll
        for (int e = 0; e < VEC; ++e)
          if (vi * VEC + e == y) xy = v[e];
      }
      if (vm > m) {
        const float r = ex2((m - vm) * 1.4426950408889634f);
        s1 *= r;
        s2 *= r * r;
        m = vm;
      }
      // e^(x - m) = 2^(x log2 e - m log2 e): one FMA and one MUFU ex2 each
      const float nml = -m * 1.4426950408889634f;
      if (brier) {
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          const float ex = ex2(fmaf(v[e], 1.4426950408889634f, nml));
          s1 += ex;
          s2 = fmaf(ex, ex, s2);
        }
      } else {
        float a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int e = 0; e < VEC; e += 2) {
          a0 += ex2(fmaf(v[e], 1.4426950408889634f, nml));
          a1 += ex2(fmaf(v[e + 1], 1.4426950408889634f, nml));
        }
        s1 += a0 + a1;
      }
    }
    // combine the threads' (m, s1, s2), argmax (first index on ties) and label logit
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, m, o), o1 = __shfl_xor_sync(0xffffffffu, s1, o);
      const float o2 = __shfl_xor_sync(0xffffffffu, s2, o);
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oa = __shfl_xor_sync(0xffffffffu, arg, o);
      xy += __shfl_xor_sync(0xffffffffu, xy, o);
      const float nm = fmaxf(m, om);
      const float ra = m == -INFINITY ? 0.f : exp2f((m - nm) * 1.4426950408889634f);
      const float rb = om == -INFINITY ? 0.f : exp2f((om - nm) * 1.4426950408889634f);
      s1 = s1 * ra + o1 * rb;
      s2 = s2 * ra * ra + o2 * rb * rb;
      m = nm;
      if (ob > best || (ob == best && oa < arg)) { best = ob; arg = oa; }
    }
    __syncthreads();
    if (lane_id() == 0) {
      shm[warp_id()] = m;
      sh1[warp_id()] = s1;
      sh2[warp_id()] = s2;
      shx[warp_id()] = xy;
      sha[warp_id()] = arg;
      // best is recovered from the argmax's logit below, not stored
    }
    __syncthreads();
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NTH / 32; ++w) M = fmaxf(M, shm[w]);
    float S1 = 0.f, S2 = 0.f, XY = 0.f;
    int A = 0x7fffffff;
    float AB = -INFINITY;
#pragma unroll
    for (int w = 0; w < NTH / 32; ++w) {
      if (shm[w] != -INFINITY) {
        const float r = exp2f((shm[w] - M) * 1.4426950408889634f);
        S1 = fmaf(sh1[w], r, S1);
        S2 = fmaf(sh2[w], r * r, S2);
      }
      XY += shx[w];
      // the warp maxima are the warp arguments' logits: compare by value, then index
      const float wb = shm[w];
      if (wb > AB || (wb == AB && sha[w] < A)) { AB = wb; A = sha[w]; }
    }
    const float inv_s = 1.0f / S1;
    const float py_raw = exp2f((XY - M) * 1.4426950408889634f) * inv_s;
    const float pt = fmaxf(py_raw, 1e-7f);
    const float fw = powf(1.0f - pt, gamma);
    const float fgs = kind == 1 ? fw - gamma * pt * powf(1.0f - pt, gamma - 1.0f) * logf(pt) : 1.0f;
    const float sum_p2 = S2 * inv_s * inv_s;
    const float bdot = sum_p2 - py_raw;                 // sum_c p_c (p_c - t_c)
    const float brier_sum = sum_p2 - 2.0f * py_raw + 1.0f;  // sum_c (p_c - t_c)^2
    if (threadIdx.x == 0) {
      float lr;
      if (kind == 0) lr = -logf(pt) * inv_rows;
      else if (kind == 1) lr = -fw * logf(pt) * inv_rows;
      else lr = brier_sum / static_cast<float>(C) * inv_rows;
      if (row_loss) row_loss[row] = lr;
      if (correct && A == y) atomicAdd(correct, 1);
    }
    if (dlogits) {
      // gradient / rows = pc * (ga + gb * pc), minus gsub at the label:
      //   CE    pc - t                 -> ga = 1,          gb = 0,  gsub = 1
      //   focal fgs (pc - t)           -> ga = fgs,        gb = 0,  gsub = fgs
      //   Brier k2 pc ((pc - t) - bdot) -> ga = -k2 bdot,  gb = k2, gsub = k2 pc
      const float k2 = 2.0f / static_cast<float>(C);
      const float ga = (kind == 0 ? 1.f : kind == 1 ? fgs : -k2 * bdot) * inv_rows;
      const float gb = (kind == 2 ? k2 : 0.f) * inv_rows;
      const float nml = -M * 1.4426950408889634f, es = inv_s;
      for (int vi = threadIdx.x; vi < nvec; vi += NTH) {
        float v[VEC], o[VEC];
        ldv<T, VEC>(src + static_cast<long long>(vi) * VEC, v);
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          const float pc = ex2(fmaf(v[e], 1.4426950408889634f, nml)) * es;
          o[e] = pc * fmaf(gb, pc, ga);
        }
        if (y >= vi * VEC && y < vi * VEC + VEC) {
#pragma unroll
          for (int e = 0; e < VEC; ++e)
            if (vi * VEC + e == y) {
              const float pc = ex2(fmaf(v[e], 1.4426950408889634f, nml)) * es;
              o[e] -= (kind == 0 ? 1.f : kind == 1 ? fgs : k2 * pc) * inv_rows;
            }
        }
        stv<T, VEC>(dlogits + base + static_cast<long long>(vi) * VEC, o);
      }
    }
  }
}

// Staged form for rows of at most 72 KB: the row comes into shared memory by
// one bulk copy (one HBM read), then three passes over shared memory:
//   1. row max, first-index argmax and the label logit (no exponentials);
//   2. e = e^(x - max) written back over the row in place, with sum e and
//      sum e^2 (Brier);
//   3. the gradient from the stored e.
// One exponential per element instead of the streaming kernel's two (online
// statistics, then the gradient): at 32000-wide rows the exponentials were
// as long as the HBM traffic and did not overlap it.  The stored e is rounded
// to T (exact for fp32); the loss uses the fp32 sums, not the stored values.
// Same results as softmax_loss_kernel (src/tkm_gpu.cu:632-682).
template <typename T, int VEC>
__global__ void __launch_bounds__(256) softmax_loss_staged_kernel(const T* __restrict__ logits,
                                                                  const int32_t* __restrict__ labels,
                                                                  T* __restrict__ dlogits, float* __restrict__ row_loss,
                                                                  int* __restrict__ correct, int rows, int C, int kind,
                                                                  float gamma) {
  constexpr int NTH = 256, NW = NTH / 32;
  constexpr float LOG2E = 1.4426950408889634f;
  __shared__ float shm[NW], sh1[NW], sh2[NW], shx[NW];
  __shared__ int sha[NW];
  __shared__ uint64_t row_full;
  __shared__ int abort_flag;
  extern __shared__ __align__(16) uint8_t stage_raw[];
  T* stage = reinterpret_cast<T*>(stage_raw);
  const uint32_t row_bytes = static_cast<uint32_t>(C) * sizeof(T);
  const int nvec = C / VEC;
  const float inv_rows = 1.0f / static_cast<float>(rows);
  const bool brier = kind == 2;
  const int warp = warp_id(), lane = lane_id();
  if (threadIdx.x == 0) {
    mbar_init(&row_full, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  int it = 0;
  for (int row = blockIdx.x; row < rows; row += gridDim.x, ++it) {
    const long long base = static_cast<long long>(row) * C;
    const int y = labels ? labels[row] : 0;
    if (threadIdx.x == 0) {
      // the previous row's accesses of the buffer (generic proxy) come first
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(&row_full, row_bytes);
      bulk_load(stage, logits + base, row_bytes, &row_full);
    }
    if (!mbar_wait(&row_full, it & 1, &abort_flag)) return;  // bounded; error word set
    // ---- pass 1: max, first-index argmax, label logit
    float m = -INFINITY, xy = 0.f;
    int arg = 0x7fffffff;
    for (int vi = threadIdx.x; vi < nvec; vi += NTH) {
      float v[VEC];
      ldv<T, VEC>(stage + vi * VEC, v);
      float vm = v[0];
      int va = 0;
#pragma unroll
      for (int e = 1; e < VEC; ++e)
        if (v[e] > vm) { vm = v[e]; va = e; }
      if (vm > m) { m = vm; arg = vi * VEC + va; }
      if (y >= vi * VEC && y < vi * VEC + VEC) {
#pragma unroll
        for (int e = 0; e < VEC; ++e)
          if (vi * VEC + e == y) xy = v[e];
      }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, m, o);
      const int oa = __shfl_xor_sync(0xffffffffu, arg, o);
      xy += __shfl_xor_sync(0xffffffffu, xy, o);
      if (om > m || (om == m && oa < arg)) { m = om; arg = oa; }
    }
    if (lane == 0) {
      shm[warp] = m;
      sha[warp] = arg;
      shx[warp] = xy;
    }
    __syncthreads();
    float M = -INFINITY, XY = 0.f;
    int A = 0x7fffffff;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      if (shm[w] > M || (shm[w] == M && sha[w] < A)) { M = shm[w]; A = sha[w]; }
      XY += shx[w];
    }
    // ---- pass 2: e = 2^(x log2e - M log2e) in place; sum e, sum e^2
    const float nml = -M * LOG2E;
    float s1 = 0.f, s2 = 0.f;
    for (int vi = threadIdx.x; vi < nvec; vi += NTH) {
      float v[VEC];
      ldv<T, VEC>(stage + vi * VEC, v);
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        v[e] = ex2(fmaf(v[e], LOG2E, nml));
        s1 += v[e];
        if (brier) s2 = fmaf(v[e], v[e], s2);
      }
      stv<T, VEC>(stage + vi * VEC, v);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
      s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    }
    if (lane == 0) {
      sh1[warp] = s1;
      sh2[warp] = s2;
    }
    __syncthreads();
    float S1 = 0.f, S2 = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      S1 += sh1[w];
      S2 += sh2[w];
    }
    const float inv_s = 1.0f / S1;
    const float py_raw = exp2f((XY - M) * LOG2E) * inv_s;
    const float pt = fmaxf(py_raw, 1e-7f);
    const float fw = powf(1.0f - pt, gamma);
    const float fgs = kind == 1 ? fw - gamma * pt * powf(1.0f - pt, gamma - 1.0f) * logf(pt) : 1.0f;
    const float sum_p2 = S2 * inv_s * inv_s;
    const float bdot = sum_p2 - py_raw;                     // sum_c p_c (p_c - t_c)
    const float brier_sum = sum_p2 - 2.0f * py_raw + 1.0f;  // sum_c (p_c - t_c)^2
    if (threadIdx.x == 0) {
      float lr;
      if (kind == 0) lr = -logf(pt) * inv_rows;
      else if (kind == 1) lr = -fw * logf(pt) * inv_rows;
      else lr = brier_sum / static_cast<float>(C) * inv_rows;
      if (row_loss) row_loss[row] = lr;
      if (correct && A == y) atomicAdd(correct, 1);
    }
    // ---- pass 3: gradient / rows = pc * (ga + gb * pc), minus gsub at the label
    //   CE    pc - t                 -> ga = 1,          gb = 0,  gsub = 1
    //   focal fgs (pc - t)           -> ga = fgs,        gb = 0,  gsub = fgs
    //   Brier k2 pc ((pc - t) - bdot) -> ga = -k2 bdot,  gb = k2, gsub = k2 pc
    if (dlogits) {
      const float k2 = 2.0f / static_cast<float>(C);
      const float ga = (kind == 0 ? 1.f : kind == 1 ? fgs : -k2 * bdot) * inv_rows;
      const float gb = (kind == 2 ? k2 : 0.f) * inv_rows;
      for (int vi = threadIdx.x; vi < nvec; vi += NTH) {
        float v[VEC], o[VEC];
        ldv<T, VEC>(stage + vi * VEC, v);  // this thread's own pass-2 values
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          const float pc = v[e] * inv_s;
          o[e] = pc * fmaf(gb, pc, ga);
        }
        if (y >= vi * VEC && y < vi * VEC + VEC) {
#pragma unroll
          for (int e = 0; e < VEC; ++e)
            if (vi * VEC + e == y) o[e] -= (kind == 0 ? 1.f : kind == 1 ? fgs : k2 * v[e] * inv_s) * inv_rows;
        }
        stv<T, VEC>(dlogits + base + static_cast<long long>(vi) * VEC, o);
      }
    }
    __syncthreads();  // every access of the buffer and of the reduction slots is done before the next row
  }
}

// loss += sum(row_loss) in a fixed order (one block).
__global__ void __launch_bounds__(256) sum_rows_kernel(const float* __restrict__ row_loss, int rows,
                                                       float* __restrict__ loss) {
  __shared__ float sh[32];
  float acc = 0.f;
  for (int r = threadIdx.x; r < rows; r += 256) acc += row_loss[r];
  acc = block_sum(acc, sh);
  if (threadIdx.x == 0) *loss += acc;
}

// ============================================================ multi-tensor SGD
// src/tkm_gpu.cu:684-720: g += wd*p (tensors flagged for decay), v = m*v + g,
// p -= lr*(m*v + g), refresh the 16-bit copy, bump the step seed.
struct SgdTensor {
  float* master;
  float* vel;
  const float* grad;
  void* lowp;        // optional 16-bit copy (bf16 or f16 by lowp_dtype)
  long long n;
  int apply_wd;
  int lowp_dtype;    // 1 = bf16, 2 = f16
};

// One SGD update of element i (the reference's order of operations).
TKB_DEVFN void sgd_one(float& p, float& v, float g, float lr, float momentum, float wd, int apply_wd) {
  if (apply_wd) g = fmaf(wd, p, g);
  v = fmaf(momentum, v, g);
  p = fmaf(-lr, fmaf(momentum, v, g), p);
}

TKB_DEVFN void sgd_store_lowp(void* lowp, int dtype, long long i, float p) {
  if (dtype == 1) reinterpret_cast<__nv_bfloat16*>(lowp)[i] = __float2bfloat16_rn(p);
  else reinterpret_cast<__half*>(lowp)[i] = __float2half_rn(p);
}

// The work is cut into chunks of SGD_CHUNK elements over all tensors; blocks
// take chunks in turn (balanced whatever the tensor sizes) and move 16 bytes
// per access when the tensor's arrays are 16-byte aligned.
constexpr int SGD_CHUNK = 4096;
constexpr int SGD_MAXT = 1024;

__global__ void __launch_bounds__(256) sgd_kernel(const SgdTensor* __restrict__ tensors, int ntensors,
                                                  const float* __restrict__ d_lr, float momentum, float wd,
                                                  uint32_t* __restrict__ d_seed) {
  __shared__ long long start[SGD_MAXT + 1];
  const float lr = *d_lr;
  // chunk prefix over the tensors: warp 0, each lane owns a contiguous segment
  if (threadIdx.x < 32) {
    const int seg = (ntensors + 31) / 32, t0 = threadIdx.x * seg;
    long long run = 0;
    for (int t = t0; t < t0 + seg && t < ntensors; ++t) run += (tensors[t].n + SGD_CHUNK - 1) / SGD_CHUNK;
    long long incl = run;
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
      const long long o = __shfl_up_sync(0xffffffffu, incl, m);
      if (static_cast<int>(threadIdx.x) >= m) incl += o;
    }
    long long c = incl - run;
    for (int t = t0; t < t0 + seg && t < ntensors; ++t) {
      start[t] = c;
      c += (tensors[t].n + SGD_CHUNK - 1) / SGD_CHUNK;
    }
    if (threadIdx.x == 31) start[ntensors] = incl;
  }
  __syncthreads();
  const long long total = start[ntensors];
  for (long long ch = blockIdx.x; ch < total; ch += gridDim.x) {
    int lo = 0, hi = ntensors - 1;  // last tensor whose first chunk is <= ch
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (start[mid] <= ch) lo = mid;
      else hi = mid - 1;
    }
    const SgdTensor T = tensors[lo];
    const long long base = (ch - start[lo]) * SGD_CHUNK;
    const long long end = base + SGD_CHUNK < T.n ? base + SGD_CHUNK : T.n;
    const bool vec = ((reinterpret_cast<uintptr_t>(T.master) | reinterpret_cast<uintptr_t>(T.vel) |
                       reinterpret_cast<uintptr_t>(T.grad)) & 15) == 0 &&
                     (!T.lowp || (reinterpret_cast<uintptr_t>(T.lowp) & 7) == 0) && (base & 3) == 0;
    if (vec) {
      for (long long i = base + threadIdx.x * 4; i < end; i += 256 * 4) {
        if (i + 3 < end) {
          float4 p = *reinterpret_cast<const float4*>(T.master + i);
          float4 v = *reinterpret_cast<const float4*>(T.vel + i);
          const float4 g = *reinterpret_cast<const float4*>(T.grad + i);
          sgd_one(p.x, v.x, g.x, lr, momentum, wd, T.apply_wd);
          sgd_one(p.y, v.y, g.y, lr, momentum, wd, T.apply_wd);
          sgd_one(p.z, v.z, g.z, lr, momentum, wd, T.apply_wd);
          sgd_one(p.w, v.w, g.w, lr, momentum, wd, T.apply_wd);
          *reinterpret_cast<float4*>(T.master + i) = p;
          *reinterpret_cast<float4*>(T.vel + i) = v;
          if (T.lowp) {
            if (T.lowp_dtype == 1) {
              const uint2 u = make_uint2(pack2<true>(p.x, p.y), pack2<true>(p.z, p.w));
              *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(T.lowp) + i) = u;
            } else {
              const uint2 u = make_uint2(pack2<false>(p.x, p.y), pack2<false>(p.z, p.w));
              *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(T.lowp) + i) = u;
            }
          }
        } else {
          for (long long k = i; k < end; ++k) {
            float p = T.master[k], v = T.vel[k];
            sgd_one(p, v, T.grad[k], lr, momentum, wd, T.apply_wd);
            T.master[k] = p;
            T.vel[k] = v;
            if (T.lowp) sgd_store_lowp(T.lowp, T.lowp_dtype, k, p);
          }
        }
      }
    } else {
      for (long long k = base + threadIdx.x; k < end; k += 256) {
        float p = T.master[k], v = T.vel[k];
        sgd_one(p, v, T.grad[k], lr, momentum, wd, T.apply_wd);
        T.master[k] = p;
        T.vel[k] = v;
        if (T.lowp) sgd_store_lowp(T.lowp, T.lowp_dtype, k, p);
      }
    }
  }
  if (blockIdx.x == 0 && threadIdx.x == 0 && d_seed) *d_seed += 0x9E3779B9u;
}

// Tables longer than SGD_MAXT: one grid row per tensor, grid-stride within it.
__global__ void __launch_bounds__(256) sgd_kernel_many(const SgdTensor* __restrict__ tensors, int ntensors,
                                                       const float* __restrict__ d_lr, float momentum, float wd,
                                                       uint32_t* __restrict__ d_seed) {
  const float lr = *d_lr;
  for (int t = blockIdx.y; t < ntensors; t += gridDim.y) {
    const SgdTensor T = tensors[t];
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < T.n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
      float p = T.master[i], v = T.vel[i];
      sgd_one(p, v, T.grad[i], lr, momentum, wd, T.apply_wd);
      T.vel[i] = v;
      T.master[i] = p;
      if (T.lowp) sgd_store_lowp(T.lowp, T.lowp_dtype, i, p);
    }
  }
  if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0 && d_seed) *d_seed += 0x9E3779B9u;
}

// ============================================================ dispatch
#define TKB_ROW_DISPATCH(KERNEL, T, VEC, C, GRID, ST, ...)                                    \
  do {                                                                                        \
    const int _nv = ((C) / (VEC) + NT - 1) / NT;                                              \
    if (_nv <= 1) KERNEL<T, VEC, 1><<<GRID, NT, 0, ST>>>(__VA_ARGS__);                        \
    else if (_nv <= 2) KERNEL<T, VEC, 2><<<GRID, NT, 0, ST>>>(__VA_ARGS__);                   \
    else if (_nv <= 4) KERNEL<T, VEC, 4><<<GRID, NT, 0, ST>>>(__VA_ARGS__);                   \
    else if (_nv <= 8) KERNEL<T, VEC, 8><<<GRID, NT, 0, ST>>>(__VA_ARGS__);                   \
    else if (_nv <= 16) KERNEL<T, VEC, 16><<<GRID, NT, 0, ST>>>(__VA_ARGS__);                 \
    else return cudaErrorInvalidValue;                                                        \
  } while (0)

// Softmax-style kernels: 256 threads per row up to 1024 vectors per row,
// 1024 threads above (each thread keeps at most 16 vectors of the row).
#define TKB_NV_DISPATCH(KERNEL, T, VEC, NTH, NVEC, GRID, ST, ...)                             \
  do {                                                                                        \
    const int _nv = ((NVEC) + (NTH)-1) / (NTH);                                               \
    if (_nv <= 1) KERNEL<T, VEC, 1, NTH><<<GRID, NTH, 0, ST>>>(__VA_ARGS__);                  \
    else if (_nv <= 2) KERNEL<T, VEC, 2, NTH><<<GRID, NTH, 0, ST>>>(__VA_ARGS__);             \
    else if (_nv <= 4) KERNEL<T, VEC, 4, NTH><<<GRID, NTH, 0, ST>>>(__VA_ARGS__);             \
    else if (_nv <= 8) KERNEL<T, VEC, 8, NTH><<<GRID, NTH, 0, ST>>>(__VA_ARGS__);             \
    else if (_nv <= 16) KERNEL<T, VEC, 16, NTH><<<GRID, NTH, 0, ST>>>(__VA_ARGS__);           \
    else return cudaErrorInvalidValue;                                                        \
  } while (0)

#define TKB_WIDE_DISPATCH(KERNEL, T, VEC, C, ROWS, ST, ...)                                   \
  do {                                                                                        \
    const int _nvec = (C) / (VEC);                                                            \
    if (_nvec <= 1024) TKB_NV_DISPATCH(KERNEL, T, VEC, 256, _nvec, row_grid(ROWS, 8), ST, __VA_ARGS__); \
    else TKB_NV_DISPATCH(KERNEL, T, VEC, 1024, _nvec, row_grid(ROWS, 2), ST, __VA_ARGS__);     \
  } while (0)

template <typename T>
static cudaError_t add_rmsnorm_fwd_t(const void* x, const void* r, void* s, void* y, const float* gamma, float* istd,
                                     int rows, int C, float eps, cudaStream_t st) {
  const int grid = row_grid(rows, 8);
  if (C % 8 == 0)
    TKB_ROW_DISPATCH(add_rmsnorm_fwd_kernel, T, 8, C, grid, st, (const T*)x, (const T*)r, (T*)s, (T*)y, gamma, istd,
                     rows, C, eps);
  else
    TKB_ROW_DISPATCH(add_rmsnorm_fwd_kernel, T, 2, C, grid, st, (const T*)x, (const T*)r, (T*)s, (T*)y, gamma, istd,
                     rows, C, eps);
  return cudaGetLastError();
}

int add_rmsnorm_bwd_grid(int rows) { return row_grid(rows, 4); }

template <typename T>
static cudaError_t add_rmsnorm_bwd_t(const void* dy, const void* s, const float* gamma, const float* istd,
                                     const void* ds_skip, void* dx, float* dgamma, float* partial, int rows, int C,
                                     cudaStream_t st) {
  const int grid = add_rmsnorm_bwd_grid(rows);
  float* part = dgamma ? partial : nullptr;
  if (C % 8 == 0)
    TKB_ROW_DISPATCH(add_rmsnorm_bwd_kernel, T, 8, C, grid, st, (const T*)dy, (const T*)s, gamma, istd,
                     (const T*)ds_skip, (T*)dx, part, rows, C);
  else
    TKB_ROW_DISPATCH(add_rmsnorm_bwd_kernel, T, 2, C, grid, st, (const T*)dy, (const T*)s, gamma, istd,
                     (const T*)ds_skip, (T*)dx, part, rows, C);
  if (dgamma) column_reduce_kernel<<<(C + 255) / 256, 256, 0, st>>>(partial, grid, C, dgamma, nullptr, C);
  return cudaGetLastError();
}

// SwiGLU grid: x covers columns, y covers row slices.
void swiglu_grid(int rows, int F, int vec, int& gx, int& gy) {
  gx = (F / vec + NT - 1) / NT;
  int want = (148 * 8 + gx - 1) / gx;
  gy = rows < want ? rows : want;
  if (gy < 1) gy = 1;
}

template <typename T>
static cudaError_t swiglu_fwd_t(const void* gu, const float* bg, const float* bu, void* h, int rows, int F,
                                cudaStream_t st) {
  const int vec = (F % 8 == 0) ? 8 : 2;
  int gx, gy;
  swiglu_grid(rows, F, vec, gx, gy);
  if (vec == 8) swiglu_fwd_kernel<T, 8><<<dim3(gx, gy), NT, 0, st>>>((const T*)gu, bg, bu, (T*)h, rows, F);
  else swiglu_fwd_kernel<T, 2><<<dim3(gx, gy), NT, 0, st>>>((const T*)gu, bg, bu, (T*)h, rows, F);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t swiglu_bwd_t(const void* dh, const void* gu, const float* bg, const float* bu, void* dgu,
                                float* dbg, float* dbu, float* partial, int rows, int F, cudaStream_t st) {
  const int vec = (F % 8 == 0) ? 8 : 2;
  int gx, gy;
  swiglu_grid(rows, F, vec, gx, gy);
  float* part = (dbg || dbu) ? partial : nullptr;
  if (vec == 8)
    swiglu_bwd_kernel<T, 8><<<dim3(gx, gy), NT, 0, st>>>((const T*)dh, (const T*)gu, bg, bu, (T*)dgu, part, rows, F);
  else
    swiglu_bwd_kernel<T, 2><<<dim3(gx, gy), NT, 0, st>>>((const T*)dh, (const T*)gu, bg, bu, (T*)dgu, part, rows, F);
  if (part) column_reduce_kernel<<<(2 * F + 255) / 256, 256, 0, st>>>(part, gy, 2 * F, dbg, dbu, F);
  return cudaGetLastError();
}

int qkv_prep_bwd_grid(int rows) { return row_grid(rows, 4); }

template <typename T>
static cudaError_t qkv_prep_fwd_t(const void* in, const float* bias, const float* gain, void* out, float* save_istd,
                                  int rows, int S, int Hq, int Hkv, int D, int qkn, int rope, const RopeTable& tab,
                                  cudaStream_t st) {
  qkv_prep_fwd_kernel<T><<<row_grid(rows, 8), NT, 0, st>>>((const T*)in, bias, gain, (T*)out, save_istd, rows, S, Hq,
                                                          Hkv, D, qkn, rope, tab);
  return cudaGetLastError();
}

// Softmax loss for 16-bit rows of 8192 to 32768 elements (the vocabulary
// losses): one persistent 512-thread block per SM walks the rows.  The rows
// come into shared memory by cp.async.bulk (one elected thread, an mbarrier
// per row buffer), NS buffers per SM (three of 64 KB at 32000 columns), so
// two to three rows are in flight from HBM while one is reduced; each thread
// then holds NV of the row's 16-byte vectors (64 values at NV = 8) in
// registers.  Per row:
//   1. max on the packed 16-bit pairs (one max.bf16x2 / f16x2 per pair);
//      the first-index argmax (only when `correct` is asked for) scanned by
//      the threads whose own maximum equals the row's; the label logit is
//      read from the staged row;
//   2. e = 2^(x log2e - M log2e) into fp32 registers, sum e and sum e^2;
//   3. the gradient from the fp32 e (one rounding, at the store); the
//      thread that stored the label's vector then rewrites that element with
//      its target term.
// Two block reductions per row, their shared slots alternating between rows;
// a thread holds 2, 4 or 8 vectors (NV), the fewest that cover the row.  A
// buffer is refilled once every thread has passed the first block reduction
// of its row (all its reads are done).  Every wait is bounded; on a timeout the block stops together and the
// elected thread waits for the copies it still has in flight before exiting.
// Against the register form it replaced (each thread loading its vectors of
// the next row into registers, one row in flight), same box, bit-identical
// results: 8192 x 32000 bf16 214 -> 189.5 us (4.90 -> 5.54 TB/s), 16384
// rows 407 -> 360 us (5.83 TB/s); before that a shared-memory staged form
// took 240.6 us.
// Same results as softmax_loss_kernel (src/tkm_gpu.cu:632-682).
template <typename T, bool BRIER, int NV>
__global__ void __launch_bounds__(512, 1) softmax_loss_bulk_kernel(const T* __restrict__ logits,
                                                                   const int32_t* __restrict__ labels,
                                                                   T* __restrict__ dlogits, float* __restrict__ row_loss,
                                                                   int* __restrict__ correct, int rows, int C, int kind,
                                                                   float gamma, int ns, int pitch) {
  constexpr int NT = 512, NW = NT / 32;
  constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
  constexpr float LOG2E = 1.4426950408889634f;
  constexpr uint32_t NEG_INF2 = BF ? 0xff80ff80u : 0xfc00fc00u;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __shared__ float sh_m[2][NW], sh_s1[2][NW], sh_s2[2][NW];
  __shared__ int sh_a[2][NW];
  __shared__ uint64_t full[8];
  __shared__ int abort_flag;
  const int nvec = C >> 3;
  const uint32_t row_bytes = static_cast<uint32_t>(C) * 2u;
  const float inv_rows = 1.0f / static_cast<float>(rows);
  const int warp = warp_id(), lane = lane_id();
  auto hmax2 = [](uint32_t a, uint32_t b) {
    uint32_t d;
    if constexpr (BF) asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    else asm("max.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  };
  auto issue = [&](int j, int r) {  // row r into buffer j % ns (elected thread)
    uint64_t* bar = &full[j % ns];
    mbar_arrive_expect_tx(bar, row_bytes);
    bulk_load(smem_raw + (j % ns) * pitch, logits + static_cast<long long>(r) * C, row_bytes, bar);
  };
  if (ns < 1 || ns > 8 || pitch < static_cast<int>(row_bytes) || (pitch & 15)) {  // launch contract of the host side
    if (threadIdx.x == 0) atomicOr(&g_device_error, ERR_BAD_LAUNCH);
    return;
  }
  if (threadIdx.x == 0) {
    for (int j = 0; j < ns; ++j) mbar_init(&full[j], 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0)
    for (int j = 0; j < ns && blockIdx.x + j * gridDim.x < rows; ++j) issue(j, blockIdx.x + j * gridDim.x);
  auto label_of = [&](int r) { return labels ? labels[r] : 0; };
  int row = blockIdx.x, it = 0;
  int y_next = row < rows ? label_of(row) : 0;
  bool stopped = false;
  for (; row < rows; row += gridDim.x, ++it) {
    const int par = it & 1;
    const int nrow = row + gridDim.x;
    const int y = y_next;
    const bool y_ok = y >= 0 && y < C;
    if (nrow < rows) y_next = label_of(nrow);
    const bool ok = mbar_wait(&full[it % ns], (it / ns) & 1, &abort_flag);
    const uint8_t* buf = smem_raw + (it % ns) * pitch;
    uint4 v[NV];
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int vi = threadIdx.x + k * NT;
      v[k] = (ok && vi < nvec) ? reinterpret_cast<const uint4*>(buf)[vi]
                               : make_uint4(NEG_INF2, NEG_INF2, NEG_INF2, NEG_INF2);
    }
    const float XY = (ok && y_ok) ? Elem<T>::ld(reinterpret_cast<const T*>(buf) + y) : 0.f;
    // ---- pass 1: max, first-index argmax
    uint32_t m2 = NEG_INF2;
#pragma unroll
    for (int k = 0; k < NV; ++k) m2 = hmax2(m2, hmax2(hmax2(v[k].x, v[k].y), hmax2(v[k].z, v[k].w)));
    const float2 mf = unpack2<BF>(m2);
    const float mt = fmaxf(mf.x, mf.y);
    float M = warp_max(mt);
    if (lane == 0) sh_m[par][warp] = M;
    if (__syncthreads_or(!ok)) {
      stopped = true;
      break;
    }
    // every thread's reads of this buffer are done: refill it
    if (threadIdx.x == 0 && row + ns * gridDim.x < rows) {
      fence_proxy_async_smem();
      issue(it + ns, row + ns * gridDim.x);
    }
    M = sh_m[par][0];
#pragma unroll
    for (int w = 1; w < NW; ++w) M = fmaxf(M, sh_m[par][w]);
    int arg = 0x7fffffff;
    if (correct && mt == M) {
#pragma unroll
      for (int k = NV - 1; k >= 0; --k) {
        const uint32_t wv[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
        for (int e = 7; e >= 0; --e) {
          const float2 f = unpack2<BF>(wv[e >> 1]);
          if (((e & 1) ? f.y : f.x) == M) arg = (threadIdx.x + k * NT) * 8 + e;
        }
      }
    }
    // ---- pass 2: e = 2^((x - M) log2e) in fp32 registers, sum e, sum e^2
    const uint64_t l2e2 = f2(LOG2E, LOG2E), nml2 = f2(-M * LOG2E, -M * LOG2E);
    float ev[NV][8];
    uint64_t s1 = f2(0.f, 0.f), s2 = f2(0.f, 0.f);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const uint32_t wv[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = unpack2<BF>(wv[i]);
        float a, b;
        f2_split(fma_f2(f2(f.x, f.y), l2e2, nml2), a, b);
        if (i < TKB_CE_EMU) {
          ex2_poly_f2(a, b, a, b);
        } else {
          a = ex2(a);
          b = ex2(b);
        }
        ev[k][2 * i] = a;
        ev[k][2 * i + 1] = b;
        const uint64_t ab = f2(a, b);
        s1 = add_f2(s1, ab);
        if (BRIER) s2 = fma_f2(ab, ab, s2);
      }
    }
    float S1, S2;
    {
      float a, b;
      f2_split(s1, a, b);
      S1 = a + b;
      f2_split(s2, a, b);
      S2 = a + b;
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      S1 += __shfl_xor_sync(0xffffffffu, S1, o);
      if (BRIER) S2 += __shfl_xor_sync(0xffffffffu, S2, o);
      arg = min(arg, __shfl_xor_sync(0xffffffffu, arg, o));
    }
    if (lane == 0) {
      sh_s1[par][warp] = S1;
      sh_s2[par][warp] = S2;
      sh_a[par][warp] = arg;
    }
    __syncthreads();
    S1 = 0.f;
    S2 = 0.f;
    int A = 0x7fffffff;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      S1 += sh_s1[par][w];
      if (BRIER) S2 += sh_s2[par][w];
      A = min(A, sh_a[par][w]);
    }
    const float inv_s = 1.0f / S1;
    const float py_raw = exp2f((XY - M) * LOG2E) * inv_s;
    const float pt = fmaxf(py_raw, 1e-7f);
    const float fw = kind == 1 ? powf(1.0f - pt, gamma) : 1.0f;
    const float fgs = kind == 1 ? fw - gamma * pt * powf(1.0f - pt, gamma - 1.0f) * logf(pt) : 1.0f;
    const float sum_p2 = S2 * inv_s * inv_s;
    const float bdot = sum_p2 - py_raw;
    const float brier_sum = sum_p2 - 2.0f * py_raw + 1.0f;
    if (threadIdx.x == 0) {
      float lr;
      if (kind == 0) lr = -logf(pt) * inv_rows;
      else if (kind == 1) lr = -fw * logf(pt) * inv_rows;
      else lr = brier_sum / static_cast<float>(C) * inv_rows;
      if (row_loss) row_loss[row] = lr;
      if (correct && A == y) atomicAdd(correct, 1);
    }
    // ---- pass 3: gradient / rows = pc * (ga + gb * pc), minus gsub at the label
    if (dlogits) {
      const float k2 = 2.0f / static_cast<float>(C);
      const float ga = (kind == 0 ? 1.f : kind == 1 ? fgs : -k2 * bdot) * inv_rows;
      const float gb = (kind == 2 ? k2 : 0.f) * inv_rows;
      const uint64_t is2 = f2(inv_s, inv_s), ga2 = f2(ga, ga), gb2 = f2(gb, gb);
      uint4* dst = reinterpret_cast<uint4*>(dlogits) + static_cast<long long>(row) * nvec;
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const int vi = threadIdx.x + k * NT;
        if (vi < nvec) {
          float o[8];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint64_t pc = mul_f2(f2(ev[k][2 * i], ev[k][2 * i + 1]), is2);
            f2_split(mul_f2(pc, BRIER ? fma_f2(gb2, pc, ga2) : ga2), o[2 * i], o[2 * i + 1]);
          }
          st_stream_v4(dst + vi, make_uint4(pack2<BF>(o[0], o[1]), pack2<BF>(o[2], o[3]), pack2<BF>(o[4], o[5]),
                                            pack2<BF>(o[6], o[7])));
        }
      }
      if (y_ok && ((y >> 3) & (NT - 1)) == threadIdx.x) {
        const float ey = ex2(fmaf(XY, LOG2E, -M * LOG2E));
        const float pc = ey * inv_s;
        float oy = pc * (BRIER ? fmaf(gb, pc, ga) : ga);
        oy -= (kind == 0 ? 1.f : kind == 1 ? fgs : k2 * pc) * inv_rows;
        Elem<T>::st(dlogits + static_cast<long long>(row) * C + y, oy);
      }
    }
  }
  if (stopped && threadIdx.x == 0) {
    // copies issued for iterations it .. it + ns - 1 may still be landing
    volatile int never = 0;
    for (int j = it; j < it + ns && blockIdx.x + j * gridDim.x < rows; ++j)
      mbar_wait(&full[j % ns], (j / ns) & 1, &never);
  }
}

template <typename T>
static cudaError_t qkv_prep_bwd_t(const void* dout, const void* in, const float* bias, const float* gain,
                                  const float* save_istd, void* din, float* dbias, float* dgain, float* partial,
                                  int rows, int S, int Hq, int Hkv, int D, int qkn, int rope, const RopeTable& tab,
                                  cudaStream_t st) {
  const int grid = qkv_prep_bwd_grid(rows);
  const bool want = dbias || (qkn && dgain);
  qkv_prep_bwd_kernel<T><<<grid, NT, 0, st>>>((const T*)dout, (const T*)in, bias, gain, save_istd, (T*)din,
                                             want ? partial : nullptr, rows, S, Hq, Hkv, D, qkn, rope, tab);
  if (want) {
    const int C = (Hq + 2 * Hkv) * D, G = (Hq + Hkv) * D;
    const int tot = C + G;
    column_reduce_kernel<<<(tot + 255) / 256, 256, 0, st>>>(partial, grid, tot, dbias, qkn ? dgain : nullptr, C);
  }
  return cudaGetLastError();
}

template <typename T>
static cudaError_t softmax_fwd_t(const void* x, void* p, int rows, int C, cudaStream_t st) {
  const int grid = row_grid(rows, 8);
  (void)grid;
  if (C % 8 == 0) TKB_WIDE_DISPATCH(softmax_fwd_kernel, T, 8, C, rows, st, (const T*)x, (T*)p, rows, C);
  else TKB_WIDE_DISPATCH(softmax_fwd_kernel, T, 2, C, rows, st, (const T*)x, (T*)p, rows, C);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t softmax_bwd_t(const void* p, const void* dp, void* dx, int rows, int C, cudaStream_t st) {
  const int grid = row_grid(rows, 8);
  (void)grid;
  if (C % 8 == 0) TKB_WIDE_DISPATCH(softmax_bwd_kernel, T, 8, C, rows, st, (const T*)p, (const T*)dp, (T*)dx, rows, C);
  else TKB_WIDE_DISPATCH(softmax_bwd_kernel, T, 2, C, rows, st, (const T*)p, (const T*)dp, (T*)dx, rows, C);
  return cudaGetLastError();
}

// loss += sum(row_loss) in the fixed order of sum_rows_kernel (used by the fused LM-head loss)
cudaError_t sum_rows(const float* row_loss, int rows, float* loss, cudaStream_t st) {
  sum_rows_kernel<<<1, 256, 0, st>>>(row_loss, rows, loss);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t softmax_loss_t(const void* logits, const int32_t* labels, void* dlogits, float* loss, int* correct,
                                  float* row_loss, int rows, int C, int kind, float gamma, cudaStream_t st) {
  const size_t row_bytes = static_cast<size_t>(C) * sizeof(T);
  const int pitch = static_cast<int>((row_bytes + 127) / 128 * 128);
  const int ns = 200 * 1024 / pitch < 8 ? 200 * 1024 / pitch : 8;  // row buffers: ~200 KB in flight
  if (sizeof(T) == 2 && C % 8 == 0 && C >= 8192 && C <= 512 * 8 * 8 && reinterpret_cast<uintptr_t>(logits) % 16 == 0) {
    const int grid = row_grid(rows, 1);
    // vectors per thread: 2, 4 or 8 (a runtime bound on one kernel measured
    // 218 against 189 us at 32000 columns)
    const int per = (C / 8 + 511) / 512;
    auto kern = per <= 2 ? (kind == 2 ? softmax_loss_bulk_kernel<T, true, 2> : softmax_loss_bulk_kernel<T, false, 2>)
                : per <= 4 ? (kind == 2 ? softmax_loss_bulk_kernel<T, true, 4> : softmax_loss_bulk_kernel<T, false, 4>)
                           : (kind == 2 ? softmax_loss_bulk_kernel<T, true, 8> : softmax_loss_bulk_kernel<T, false, 8>);
    const int dyn = ns * pitch;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn);
    if (e != cudaSuccess) return e;
    kern<<<grid, 512, dyn, st>>>((const T*)logits, labels, (T*)dlogits, row_loss, correct, rows, C, kind, gamma, ns,
                                 pitch);
  } else if (C % 8 == 0 && C >= 8192 && row_bytes <= 72 * 1024) {
    auto kern = softmax_loss_staged_kernel<T, 8>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(row_bytes));
    if (e != cudaSuccess) return e;
    kern<<<row_grid(rows, 3), 256, row_bytes, st>>>((const T*)logits, labels, (T*)dlogits, row_loss, correct, rows, C,
                                                    kind, gamma);
  } else if (C % 8 == 0 && C >= 8192)
    softmax_loss_stream_kernel<T, 8><<<row_grid(rows, 8), 256, 0, st>>>((const T*)logits, labels, (T*)dlogits,
                                                                               row_loss, correct, rows, C, kind, gamma);
  else if (C % 8 == 0)
    TKB_WIDE_DISPATCH(softmax_loss_kernel, T, 8, C, rows, st, (const T*)logits, labels, (T*)dlogits, row_loss, correct,
                      rows, C, kind, gamma);
  else
    TKB_WIDE_DISPATCH(softmax_loss_kernel, T, 2, C, rows, st, (const T*)logits, labels, (T*)dlogits, row_loss, correct,
                      rows, C, kind, gamma);
  if (loss) sum_rows_kernel<<<1, 256, 0, st>>>(row_loss, rows, loss);
  return cudaGetLastError();
}

}  // namespace tkb
