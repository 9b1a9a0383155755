// attn_f32.cu -- fp32 attention (the fp32 mode of the hot path).
//
// The tensor-core path computes in 16-bit inputs with fp32 accumulation; the
// fp32 mode must match the fp64 oracle to 1e-4 relative L2, which rules out
// tf32.  These kernels use fp32 FMA throughout.  Same packed layouts and
// semantics as the 16-bit kernels (src/tkm_gpu.cu:302-598 of the reference,
// with the true dK/dV).
//
// Thread layout: 4 threads own one row (query or key), each holding D/4
// contiguous features; 32 rows per 128-thread block; the other side is
// streamed through shared memory in 32-row tiles.
#include "tkb_common.cuh"

namespace tkb {

template <int D>
struct F32Tile {
  static constexpr int R = 32;       // rows per block and per streamed tile
  static constexpr int DP = D / 4;   // features per thread
};

TKB_DEVFN float quad_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  return v;
}

template <int D>
__global__ void __launch_bounds__(128) attn_f32_fwd_kernel(const float* __restrict__ qkv, float* __restrict__ out,
                                                           float* __restrict__ lse, int B, int S, int Hq, int Hkv,
                                                           float scale, int causal) {
  using T = F32Tile<D>;
  __shared__ float sk[T::R][D];
  __shared__ float sv[T::R][D];
  const int bh = blockIdx.x, b = bh / Hq, h = bh % Hq, g = h / (Hq / Hkv);
  const long long ld = static_cast<long long>(Hq + 2 * Hkv) * D;
  const int row = blockIdx.y * T::R + (threadIdx.x >> 2);
  const int part = threadIdx.x & 3;
  const bool valid = row < S;
  float q[T::DP], o[T::DP];
  const float* qp = qkv + (static_cast<long long>(b) * S + (valid ? row : 0)) * ld + static_cast<long long>(h) * D + part * T::DP;
#pragma unroll
  for (int d = 0; d < T::DP; ++d) {
    q[d] = qp[d] * scale;
    o[d] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  const int kend = causal ? min(S, (blockIdx.y + 1) * T::R) : S;
  for (int k0 = 0; k0 < kend; k0 += T::R) {
    __syncthreads();
    for (int e = threadIdx.x; e < T::R * D; e += 128) {
      const int r = e / D, c = e % D, key = k0 + r;
      const float* base = qkv + (static_cast<long long>(b) * S + (key < S ? key : 0)) * ld;
      sk[r][c] = key < S ? base[static_cast<long long>(Hq + g) * D + c] : 0.f;
      sv[r][c] = key < S ? base[static_cast<long long>(Hq + Hkv + g) * D + c] : 0.f;
    }
    __syncthreads();
    for (int r = 0; r < T::R; ++r) {
      const int key = k0 + r;
      float s = 0.f;
#pragma unroll
      for (int d = 0; d < T::DP; ++d) s = fmaf(q[d], sk[r][part * T::DP + d], s);
      s = quad_sum(s);
      if (key >= S || (causal && key > row)) continue;
      const float mn = fmaxf(m, s);
      const float corr = expf(m - mn);
      const float pr = expf(s - mn);
      l = l * corr + pr;
#pragma unroll
      for (int d = 0; d < T::DP; ++d) o[d] = fmaf(pr, sv[r][part * T::DP + d], o[d] * corr);
      m = mn;
    }
  }
  if (valid) {
    float* op = out + (static_cast<long long>(b) * S + row) * Hq * D + static_cast<long long>(h) * D + part * T::DP;
    const float inv = 1.0f / (l + 1e-8f);
#pragma unroll
    for (int d = 0; d < T::DP; ++d) op[d] = o[d] * inv;
    if (part == 0 && lse) lse[static_cast<long long>(bh) * S + row] = m + logf(l + 1e-8f);
  }
}

// dQ: one query row per 4 threads, keys streamed.  delta = rowsum(O*dO) computed in place.
template <int D>
__global__ void __launch_bounds__(128) attn_f32_bwd_dq_kernel(const float* __restrict__ qkv, const float* __restrict__ out,
                                                              const float* __restrict__ dout, const float* __restrict__ lse,
                                                              float* __restrict__ dqkv, int B, int S, int Hq, int Hkv,
                                                              float scale, int causal) {
  using T = F32Tile<D>;
  __shared__ float sk[T::R][D];
  __shared__ float sv[T::R][D];
  const int bh = blockIdx.x, b = bh / Hq, h = bh % Hq, g = h / (Hq / Hkv);
  const long long ld = static_cast<long long>(Hq + 2 * Hkv) * D, ldo = static_cast<long long>(Hq) * D;
  const int row = blockIdx.y * T::R + (threadIdx.x >> 2);
  const int part = threadIdx.x & 3;
  const bool valid = row < S;
  const int rr = valid ? row : 0;
  float q[T::DP], dO[T::DP], dq[T::DP];
  const float* qp = qkv + (static_cast<long long>(b) * S + rr) * ld + static_cast<long long>(h) * D + part * T::DP;
  const float* op = out + (static_cast<long long>(b) * S + rr) * ldo + static_cast<long long>(h) * D + part * T::DP;
  const float* dp = dout + (static_cast<long long>(b) * S + rr) * ldo + static_cast<long long>(h) * D + part * T::DP;
  float del = 0.f;
#pragma unroll
  for (int d = 0; d < T::DP; ++d) {
    q[d] = qp[d];
    dO[d] = dp[d];
    dq[d] = 0.f;
    del = fmaf(op[d], dO[d], del);
  }
  del = quad_sum(del);
  const float L = lse[static_cast<long long>(bh) * S + rr];
  const int kend = causal ? min(S, (blockIdx.y + 1) * T::R) : S;
  for (int k0 = 0; k0 < kend; k0 += T::R) {
    __syncthreads();
    for (int e = threadIdx.x; e < T::R * D; e += 128) {
      const int r = e / D, c = e % D, key = k0 + r;
      const float* base = qkv + (static_cast<long long>(b) * S + (key < S ? key : 0)) * ld;
      sk[r][c] = key < S ? base[static_cast<long long>(Hq + g) * D + c] : 0.f;
      sv[r][c] = key < S ? base[static_cast<long long>(Hq + Hkv + g) * D + c] : 0.f;
    }
    __syncthreads();
    for (int r = 0; r < T::R; ++r) {
      const int key = k0 + r;
      float s = 0.f, pd = 0.f;
#pragma unroll
      for (int d = 0; d < T::DP; ++d) {
        s = fmaf(q[d], sk[r][part * T::DP + d], s);
        pd = fmaf(dO[d], sv[r][part * T::DP + d], pd);
      }
      s = quad_sum(s);
      pd = quad_sum(pd);
      if (key >= S || (causal && key > row)) continue;
      const float pr = expf(s * scale - L);
      const float ds = pr * (pd - del) * scale;
#pragma unroll
      for (int d = 0; d < T::DP; ++d) dq[d] = fmaf(ds, sk[r][part * T::DP + d], dq[d]);
    }
  }
  if (valid) {
    float* dst = dqkv + (static_cast<long long>(b) * S + row) * ld + static_cast<long long>(h) * D + part * T::DP;
#pragma unroll
    for (int d = 0; d < T::DP; ++d) dst[d] = dq[d];
  }
}

// dK, dV: one key row per 4 threads, (query head, query) pairs of the group streamed.
template <int D>
__global__ void __launch_bounds__(128) attn_f32_bwd_dkv_kernel(const float* __restrict__ qkv, const float* __restrict__ out,
                                                               const float* __restrict__ dout, const float* __restrict__ lse,
                                                               float* __restrict__ dqkv, int B, int S, int Hq, int Hkv,
                                                               float scale, int causal) {
  using T = F32Tile<D>;
  __shared__ float sq[T::R][D];
  __shared__ float sdo[T::R][D];
  __shared__ float sl[T::R], sdel[T::R];
  const int bg = blockIdx.x, b = bg / Hkv, g = bg % Hkv, G = Hq / Hkv;
  const long long ld = static_cast<long long>(Hq + 2 * Hkv) * D, ldo = static_cast<long long>(Hq) * D;
  const int key = blockIdx.y * T::R + (threadIdx.x >> 2);
  const int part = threadIdx.x & 3;
  const bool valid = key < S;
  const int kk = valid ? key : 0;
  float k[T::DP], v[T::DP], dk[T::DP], dv[T::DP];
  const float* kp = qkv + (static_cast<long long>(b) * S + kk) * ld + static_cast<long long>(Hq + g) * D + part * T::DP;
  const float* vp = qkv + (static_cast<long long>(b) * S + kk) * ld + static_cast<long long>(Hq + Hkv + g) * D + part * T::DP;
#pragma unroll
  for (int d = 0; d < T::DP; ++d) {
    k[d] = kp[d];
    v[d] = vp[d];
    dk[d] = 0.f;
    dv[d] = 0.f;
  }
  const int q_start = causal ? blockIdx.y * T::R : 0;
  for (int hh = 0; hh < G; ++hh) {
    const int h = g * G + hh;
    for (int q0 = q_start; q0 < S; q0 += T::R) {
      __syncthreads();
      for (int e = threadIdx.x; e < T::R * D; e += 128) {
        const int r = e / D, c = e % D, qi = q0 + r;
        const long long ro = static_cast<long long>(b) * S + (qi < S ? qi : 0);
        sq[r][c] = qi < S ? qkv[ro * ld + static_cast<long long>(h) * D + c] : 0.f;
        sdo[r][c] = qi < S ? dout[ro * ldo + static_cast<long long>(h) * D + c] : 0.f;
      }
      if (threadIdx.x < T::R) {
        const int qi = q0 + threadIdx.x;
        float dsum = 0.f;
        if (qi < S) {
          const long long ro = static_cast<long long>(b) * S + qi;
          for (int c = 0; c < D; ++c) dsum = fmaf(out[ro * ldo + static_cast<long long>(h) * D + c],
                                                   dout[ro * ldo + static_cast<long long>(h) * D + c], dsum);
        }
        sdel[threadIdx.x] = dsum;
        sl[threadIdx.x] = qi < S ? lse[(static_cast<long long>(b) * Hq + h) * S + qi] : 0.f;
      }
      __syncthreads();
      for (int r = 0; r < T::R; ++r) {
        const int qi = q0 + r;
        float s = 0.f, pd = 0.f;
#pragma unroll
        for (int d = 0; d < T::DP; ++d) {
          s = fmaf(k[d], sq[r][part * T::DP + d], s);
          pd = fmaf(v[d], sdo[r][part * T::DP + d], pd);
        }
        s = quad_sum(s);
        pd = quad_sum(pd);
        if (qi >= S || (causal && key > qi)) continue;
        const float pr = expf(s * scale - sl[r]);
        const float ds = pr * (pd - sdel[r]) * scale;
#pragma unroll
        for (int d = 0; d < T::DP; ++d) {
          dk[d] = fmaf(ds, sq[r][part * T::DP + d], dk[d]);
          dv[d] = fmaf(pr, sdo[r][part * T::DP + d], dv[d]);
        }
      }
    }
  }
  if (valid) {
    float* dkp = dqkv + (static_cast<long long>(b) * S + key) * ld + static_cast<long long>(Hq + g) * D + part * T::DP;
    float* dvp = dqkv + (static_cast<long long>(b) * S + key) * ld + static_cast<long long>(Hq + Hkv + g) * D + part * T::DP;
#pragma unroll
    for (int d = 0; d < T::DP; ++d) {
      dkp[d] = dk[d];
      dvp[d] = dv[d];
    }
  }
}

cudaError_t attn_f32_fwd(const float* qkv, float* out, float* lse, int B, int S, int Hq, int Hkv, int D, float scale,
                         int causal, cudaStream_t st) {
  dim3 grid(B * Hq, (S + 31) / 32);
  if (D == 64) attn_f32_fwd_kernel<64><<<grid, 128, 0, st>>>(qkv, out, lse, B, S, Hq, Hkv, scale, causal);
  else if (D == 128) attn_f32_fwd_kernel<128><<<grid, 128, 0, st>>>(qkv, out, lse, B, S, Hq, Hkv, scale, causal);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

cudaError_t attn_f32_bwd(const float* qkv, const float* out, const float* dout, const float* lse, float* dqkv, int B,
                         int S, int Hq, int Hkv, int D, float scale, int causal, cudaStream_t st) {
  dim3 gq(B * Hq, (S + 31) / 32), gk(B * Hkv, (S + 31) / 32);
  if (D == 64) {
    attn_f32_bwd_dq_kernel<64><<<gq, 128, 0, st>>>(qkv, out, dout, lse, dqkv, B, S, Hq, Hkv, scale, causal);
    attn_f32_bwd_dkv_kernel<64><<<gk, 128, 0, st>>>(qkv, out, dout, lse, dqkv, B, S, Hq, Hkv, scale, causal);
  } else if (D == 128) {
    attn_f32_bwd_dq_kernel<128><<<gq, 128, 0, st>>>(qkv, out, dout, lse, dqkv, B, S, Hq, Hkv, scale, causal);
    attn_f32_bwd_dkv_kernel<128><<<gk, 128, 0, st>>>(qkv, out, dout, lse, dqkv, B, S, Hq, Hkv, scale, causal);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace tkb
