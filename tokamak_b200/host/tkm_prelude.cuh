// tkm_prelude.cuh -- device helpers compiled by NVRTC in front of the code
// that tkm_codegen_cuda_string() generates (sm_100a, no system headers).
//
// TKM_ACT_BYTES selects the activation storage: 2 = bf16 (default), 4 = fp32.
// Plasma kernels move a row in 16-byte chunks of TKG_VP channel pairs and
// compute in fp32.
#ifndef TKM_ACT_BYTES
#define TKM_ACT_BYTES 2
#endif

typedef unsigned char uint8_t;
typedef unsigned short uint16_t;
typedef unsigned int uint32_t;
typedef unsigned long long uint64_t;

#if TKM_ACT_BYTES == 2
typedef unsigned short tkm_act_t;  // bf16 bit pattern
#else
typedef float tkm_act_t;
#endif

// ------------------------------------------------------------ conversions

__device__ __forceinline__ float2 tkm_bf16x2_to_f2(uint32_t u) {
  return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xFFFF0000u));
}

// round-to-nearest-even to two bf16 in one word (x in the low half)
__device__ __forceinline__ uint32_t tkm_f2_to_bf16x2(float2 v) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(v.y), "f"(v.x));
  return r;
}

// ---------------------------------------------------- chunk loads / stores
// p is the pair offset from `base` (element offset 2 * p); VP pairs move.

template <int VP>
__device__ __forceinline__ void tkm_zero(float2 (&v)[VP]) {
#pragma unroll
  for (int i = 0; i < VP; ++i) v[i] = make_float2(0.f, 0.f);
}

#if TKM_ACT_BYTES == 2
template <int VP>
__device__ __forceinline__ void tkm_ld(const tkm_act_t* base, long long p, float2 (&v)[VP]) {
  const uint32_t* src = reinterpret_cast<const uint32_t*>(base) + p;
  if constexpr (VP == 4) {
    const uint4 w = __ldg(reinterpret_cast<const uint4*>(src));
    v[0] = tkm_bf16x2_to_f2(w.x); v[1] = tkm_bf16x2_to_f2(w.y);
    v[2] = tkm_bf16x2_to_f2(w.z); v[3] = tkm_bf16x2_to_f2(w.w);
  } else if constexpr (VP == 2) {
    const uint2 w = __ldg(reinterpret_cast<const uint2*>(src));
    v[0] = tkm_bf16x2_to_f2(w.x); v[1] = tkm_bf16x2_to_f2(w.y);
  } else {
    v[0] = tkm_bf16x2_to_f2(__ldg(src));
  }
}

template <int VP>
__device__ __forceinline__ void tkm_st(tkm_act_t* base, long long p, const float2 (&v)[VP]) {
  uint32_t* dst = reinterpret_cast<uint32_t*>(base) + p;
  if constexpr (VP == 4) {
    *reinterpret_cast<uint4*>(dst) = make_uint4(tkm_f2_to_bf16x2(v[0]), tkm_f2_to_bf16x2(v[1]),
                                                tkm_f2_to_bf16x2(v[2]), tkm_f2_to_bf16x2(v[3]));
  } else if constexpr (VP == 2) {
    *reinterpret_cast<uint2*>(dst) = make_uint2(tkm_f2_to_bf16x2(v[0]), tkm_f2_to_bf16x2(v[1]));
  } else {
    *dst = tkm_f2_to_bf16x2(v[0]);
  }
}
#else
template <int VP>
__device__ __forceinline__ void tkm_ld(const tkm_act_t* base, long long p, float2 (&v)[VP]) {
  const float2* src = reinterpret_cast<const float2*>(base) + p;
  if constexpr (VP == 2) {
    const float4 w = __ldg(reinterpret_cast<const float4*>(src));
    v[0] = make_float2(w.x, w.y); v[1] = make_float2(w.z, w.w);
  } else {
    v[0] = __ldg(src);
  }
}

template <int VP>
__device__ __forceinline__ void tkm_st(tkm_act_t* base, long long p, const float2 (&v)[VP]) {
  float2* dst = reinterpret_cast<float2*>(base) + p;
  if constexpr (VP == 2) {
    *reinterpret_cast<float4*>(dst) = make_float4(v[0].x, v[0].y, v[1].x, v[1].y);
  } else {
    *dst = v[0];
  }
}
#endif

// gradient accumulation into a slot that an earlier backward writer filled
template <int VP>
__device__ __forceinline__ void tkm_st_add(tkm_act_t* base, long long p, const float2 (&v)[VP]) {
  float2 o[VP];
  tkm_ld<VP>(base, p, o);
#pragma unroll
  for (int i = 0; i < VP; ++i) { o[i].x += v[i].x; o[i].y += v[i].y; }
  tkm_st<VP>(base, p, o);
}

// ----------------------------------------------------------- async row staging
// cp.async of one chunk (VP channel pairs) of a row into a shared-memory slot
// private to the thread; !ok fills the slot with zeros (no global read).
template <int VP>
__device__ __forceinline__ void tkm_cp(void* slot, const tkm_act_t* base, long long p, bool ok) {
  constexpr int BYTES = VP * 2 * TKM_ACT_BYTES;
  const tkm_act_t* src = ok ? base + 2 * p : base;
  const unsigned dst = static_cast<unsigned>(__cvta_generic_to_shared(slot));
  const int n = ok ? BYTES : 0;
  if constexpr (BYTES == 16)  // streamed once: not kept in L1
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
  else
    asm volatile("cp.async.ca.shared.global [%0], [%1], %2, %3;" ::"r"(dst), "l"(src), "n"(BYTES), "r"(n) : "memory");
}
__device__ __forceinline__ void tkm_cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void tkm_cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// a staged chunk back from the thread's slot
template <int VP>
__device__ __forceinline__ void tkm_lds(const void* slot, float2 (&v)[VP]) {
#if TKM_ACT_BYTES == 2
  const uint32_t* w = reinterpret_cast<const uint32_t*>(slot);
#pragma unroll
  for (int i = 0; i < VP; ++i) v[i] = tkm_bf16x2_to_f2(w[i]);
#else
  const float2* f = reinterpret_cast<const float2*>(slot);
#pragma unroll
  for (int i = 0; i < VP; ++i) v[i] = f[i];
#endif
}

// ----------------------------------------------------------- reductions
// Rows occupy TPR consecutive threads (TPR a power of two <= 32, or a
// multiple of 32); every thread of the block calls these.

#define TKM_RED_SLOTS(TPR, RPB) ((TPR) > 32 ? (RPB) * ((TPR) / 32) : 1)

template <int TPR, int RPB>
__device__ __forceinline__ float tkm_row_sum(float v, float* red) {
  if constexpr (TPR <= 32) {
#pragma unroll
    for (int m = TPR / 2; m >= 1; m >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, m);
    return v;
  } else {
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, m);
    constexpr int WPR = TPR / 32;
    const int slot = threadIdx.x / TPR, w = (threadIdx.x % TPR) / 32;
    if ((threadIdx.x & 31) == 0) red[slot * WPR + w] = v;
    __syncthreads();
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < WPR; ++i) s += red[slot * WPR + i];
    __syncthreads();
    return s;
  }
}

template <int TPR, int RPB>
__device__ __forceinline__ float2 tkm_row_sum2(float2 v, float2* red) {
  if constexpr (TPR <= 32) {
#pragma unroll
    for (int m = TPR / 2; m >= 1; m >>= 1) {
      v.x += __shfl_xor_sync(0xFFFFFFFFu, v.x, m);
      v.y += __shfl_xor_sync(0xFFFFFFFFu, v.y, m);
    }
    return v;
  } else {
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
      v.x += __shfl_xor_sync(0xFFFFFFFFu, v.x, m);
      v.y += __shfl_xor_sync(0xFFFFFFFFu, v.y, m);
    }
    constexpr int WPR = TPR / 32;
    const int slot = threadIdx.x / TPR, w = (threadIdx.x % TPR) / 32;
    if ((threadIdx.x & 31) == 0) red[slot * WPR + w] = v;
    __syncthreads();
    float2 s = make_float2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < WPR; ++i) { s.x += red[slot * WPR + i].x; s.y += red[slot * WPR + i].y; }
    __syncthreads();
    return s;
  }
}

// sum over N consecutive lanes (N a power of two <= 32, groups aligned to N)
template <int N>
__device__ __forceinline__ float tkm_group_sum(float v) {
#pragma unroll
  for (int m = N / 2; m >= 1; m >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, m);
  return v;
}

// One partial row of a per-channel parameter gradient for this block: the
// accumulators of the block's RPB row slots are summed (in slot order) and
// written to dst over this block's chunks.  lr: the thread's chunk lane in the
// row (column blocks included), ll: its lane in the block.  pbuf holds
// THREADS * KCH * VP float2 when RPB > 1.
template <int VP, int KCH, int TPR, int RPB, int NCH>
__device__ __forceinline__ void tkm_block_partial(const float2 (&acc)[KCH][VP], float2* __restrict__ dst,
                                                  float2* pbuf, int lr, int ll) {
  if constexpr (RPB == 1) {
#pragma unroll
    for (int k = 0; k < KCH; ++k) {
      const int ch = lr + k * TPR;
      if (ch < NCH) {
#pragma unroll
        for (int q = 0; q < VP; ++q) dst[ch * VP + q] = acc[k][q];
      }
    }
  } else {
#pragma unroll
    for (int k = 0; k < KCH; ++k)
#pragma unroll
      for (int q = 0; q < VP; ++q) pbuf[(threadIdx.x * KCH + k) * VP + q] = acc[k][q];
    __syncthreads();
    if (threadIdx.x < TPR) {
#pragma unroll
      for (int k = 0; k < KCH; ++k) {
        const int ch = lr + k * TPR;
        if (ch < NCH) {
#pragma unroll
          for (int q = 0; q < VP; ++q) {
            float2 s = make_float2(0.f, 0.f);
            for (int r = 0; r < RPB; ++r) {
              const float2 t = pbuf[((r * TPR + ll) * KCH + k) * VP + q];
              s.x += t.x;
              s.y += t.y;
            }
            dst[ch * VP + q] = s;
          }
        }
      }
    }
    __syncthreads();
  }
}

// tkm_block_partial for accumulators in shared memory: slot
// (k * VP + q) * THREADS + thread.  With RPB > 1 the caller has synchronised
// the block after the last accumulation.
template <int VP, int KCH, int TPR, int RPB, int NCH, int THREADS>
__device__ __forceinline__ void tkm_block_partial_s(const float2* acc, float2* __restrict__ dst, int lr, int ll) {
  if (threadIdx.x >= TPR) return;
#pragma unroll
  for (int k = 0; k < KCH; ++k) {
    const int ch = lr + k * TPR;
    if (ch < NCH) {
#pragma unroll
      for (int q = 0; q < VP; ++q) {
        float2 s = acc[(k * VP + q) * THREADS + ll];
        for (int r = 1; r < RPB; ++r) {
          const float2 t = acc[(k * VP + q) * THREADS + r * TPR + ll];
          s.x += t.x;
          s.y += t.y;
        }
        dst[ch * VP + q] = s;
      }
    }
  }
}

// Column sums of a parameter's partial rows part[nblk][C2] (float2 pairs) in
// two stages, in a fixed order (deterministic):
//   stage 1, blockIdx.z = segment: rows [16 z, 16 z + 16) are summed into row 16 z;
//   stage 2: rows 0, 16, 32, ... are summed into dst[2c], dst[2c + 1].
// Block: 256 threads = 32 pairs x 8 row slices; blockIdx.x covers the pairs.
#define TKM_COLSUM_SEG 16
__device__ __forceinline__ void tkm_colsum_pairs(float2* __restrict__ part, int nblk, int C2, int stage,
                                                 float* __restrict__ dst) {
  __shared__ float2 s[8][33];
  const int lane = threadIdx.x & 31, sl = threadIdx.x >> 5;
  const int pair = blockIdx.x * 32 + lane;
  float2 acc = make_float2(0.f, 0.f);
  const int r0 = stage == 1 ? blockIdx.z * TKM_COLSUM_SEG : 0;
  const int r1 = stage == 1 ? min(r0 + TKM_COLSUM_SEG, nblk) : nblk;
  const int step = stage == 1 ? 8 : 8 * TKM_COLSUM_SEG;
  if (pair < C2)
    for (int r = r0 + (stage == 1 ? sl : sl * TKM_COLSUM_SEG); r < r1; r += step) {
      const float2 v = part[(size_t)r * C2 + pair];
      acc.x += v.x;
      acc.y += v.y;
    }
  s[sl][lane] = acc;
  __syncthreads();
  if (sl == 0 && pair < C2) {
    float2 t = s[0][lane];
#pragma unroll
    for (int i = 1; i < 8; ++i) { t.x += s[i][lane].x; t.y += s[i][lane].y; }
    if (stage == 1) {
      part[(size_t)r0 * C2 + pair] = t;
    } else {
      dst[2 * pair] = t.x;
      dst[2 * pair + 1] = t.y;
    }
  }
}

// ------------------------------------------------- activation helpers

// logistic function with the hardware exponential and reciprocal (relative
// error ~1e-6, far below bf16 and within the fp32 mode's 1e-4 budget)
__device__ __forceinline__ float tkm_sigmoid(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }

// log(1 + e^x), taken as x above 20 (where the two agree in fp32)
__device__ __forceinline__ float tkm_softplus20(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

// GELU, tanh form: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))
__device__ __forceinline__ float tkm_gelu_tanh(float x) {
  const float u = 0.7978845608f * (x + 0.044715f * x * x * x);
  return 0.5f * x * (1.0f + tanhf(u));
}

__device__ __forceinline__ float tkm_gelu_tanh_grad(float x) {
  const float u = 0.7978845608f * (x + 0.044715f * x * x * x);
  const float t = tanhf(u);
  return 0.5f * (1.0f + t) + 0.5f * x * (1.0f - t * t) * 0.7978845608f * (1.0f + 3.0f * 0.044715f * x * x);
}

// ------------------------------------------------------------------ PRNGs
// The generators the DSL names (prng: / rng=): xorshift32 (Marsaglia 2003),
// a Wang integer hash followed by xorshift32, PCG-XSH-RR 64/32 (O'Neill 2014)
// and a 7-round Philox-style counter generator.  Each stream is seeded from
// (seed, idx) as the engine defines it so a given step draws the same numbers.

struct RngXorshift32 { uint32_t s; };
struct RngWangXorshift32 { uint32_t s; };
struct RngPcg32 { uint64_t state, inc; };
struct RngPhilox { uint32_t ctr, key, sub; };

__device__ __forceinline__ uint32_t tkm_xorshift32(uint32_t& s) {
  s ^= s << 13;
  s ^= s >> 17;
  s ^= s << 5;
  return s;
}

__device__ __forceinline__ void rng_init(RngXorshift32* r, uint32_t seed, uint32_t idx) {
  const uint32_t x = seed ^ (idx * 0x9E3779B9u + 0x7F4A7C15u);
  r->s = x ? x : 1u;
}
__device__ __forceinline__ uint32_t rng_u32(RngXorshift32* r) { return tkm_xorshift32(r->s); }

__device__ __forceinline__ uint32_t tkm_wang_hash(uint32_t k) {
  k = ~k + (k << 18);
  k ^= k >> 31;
  k = k * 21u;  // k + (k << 2) + (k << 4)
  k ^= k >> 11;
  k += k << 6;
  k ^= k >> 22;
  return k;
}
__device__ __forceinline__ void rng_init(RngWangXorshift32* r, uint32_t seed, uint32_t idx) {
  const uint32_t k = tkm_wang_hash(seed ^ idx);
  r->s = k ? k : 1u;
}
__device__ __forceinline__ uint32_t rng_u32(RngWangXorshift32* r) { return tkm_xorshift32(r->s); }

__device__ __forceinline__ uint32_t rng_u32(RngPcg32* r) {
  const uint64_t old = r->state;
  r->state = old * 6364136223846793005ull + r->inc;
  const uint32_t xorshifted = (uint32_t)(((old >> 18u) ^ old) >> 27u);
  const uint32_t rot = (uint32_t)(old >> 59u);
  return (xorshifted >> rot) | (xorshifted << ((32u - rot) & 31u));
}
__device__ __forceinline__ void rng_init(RngPcg32* r, uint32_t seed, uint32_t idx) {
  r->state = 0ull;
  r->inc = ((uint64_t)idx << 1u) | 1ull;
  rng_u32(r);
  r->state += (uint64_t)seed ^ 0x853C49E6748FEA9Bull;
  rng_u32(r);
}

__device__ __forceinline__ void rng_init(RngPhilox* r, uint32_t seed, uint32_t idx) {
  r->ctr = idx;
  r->key = seed;
  r->sub = 0u;
}
__device__ __forceinline__ uint32_t rng_u32(RngPhilox* r) {
  uint32_t c0 = r->ctr, c1 = r->sub++, k = r->key;
#pragma unroll
  for (int i = 0; i < 7; ++i) {
    const uint32_t hi = __umulhi(0xD2511F53u, c0), lo = 0xD2511F53u * c0;
    c0 = hi ^ c1 ^ k;
    c1 = lo;
    k += 0x9E3779B9u;
  }
  return c0;
}

// uniform in [0, 1) from the top 24 bits
template <typename R>
__device__ __forceinline__ float rng_uniform(R* r) {
  return (float)(rng_u32(r) >> 8) * (1.0f / 16777216.0f);
}

// two standard normals (Box-Muller)
template <typename R>
__device__ __forceinline__ float2 rng_normal2(R* r) {
  const float u1 = rng_uniform(r) + 1e-7f, u2 = rng_uniform(r);
  float s, c;
  sincosf(6.283185307f * u2, &s, &c);
  const float mag = sqrtf(-2.0f * logf(u1));
  return make_float2(mag * c, mag * s);
}

// ------------------------------------------- 16-bit float names for snippets
// Bodies written against the reference's half2 helpers still compile.
struct __align__(2) __half { uint16_t x; };
struct __align__(4) __half2 { uint16_t x, y; };
__device__ __forceinline__ float __half2float(__half h) {
  float f;
  asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"(h.x));
  return f;
}
__device__ __forceinline__ __half __float2half(float f) {
  __half h;
  asm("cvt.rn.f16.f32 %0, %1;" : "=h"(h.x) : "f"(f));
  return h;
}
__device__ __forceinline__ float2 __half22float2(__half2 h) {
  return make_float2(__half2float(__half{h.x}), __half2float(__half{h.y}));
}
__device__ __forceinline__ __half2 __float22half2_rn(float2 f) {
  return __half2{__float2half(f.x).x, __float2half(f.y).x};
}
__device__ __forceinline__ __half2 __floats2half2_rn(float a, float b) { return __float22half2_rn(make_float2(a, b)); }

// ------------------------------------------- runtime utility kernels

// fp32 -> activation storage (input upload)
extern "C" __global__ void __launch_bounds__(256) tkm_f32_to_act(const float* __restrict__ src, tkm_act_t* __restrict__ dst,
                                                                 long long n) {
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < n; i += (long long)gridDim.x * 256) {
#if TKM_ACT_BYTES == 2
    const uint32_t u = __float_as_uint(src[i]);
    // round to nearest even; NaN stays NaN
    const uint32_t r = ((u & 0x7F800000u) == 0x7F800000u && (u & 0x7FFFFFu)) ? (u | 0x400000u)
                                                                              : u + 0x7FFFu + ((u >> 16) & 1u);
    dst[i] = (tkm_act_t)(r >> 16);
#else
    dst[i] = src[i];
#endif
  }
}

// activation storage -> fp32 (output / gradient download)
extern "C" __global__ void __launch_bounds__(256) tkm_act_to_f32(const tkm_act_t* __restrict__ src, float* __restrict__ dst,
                                                                 long long n) {
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < n; i += (long long)gridDim.x * 256) {
#if TKM_ACT_BYTES == 2
    dst[i] = __uint_as_float((uint32_t)src[i] << 16);
#else
    dst[i] = src[i];
#endif
  }
}

// fp32 -> bf16, round to nearest even (NaN kept quiet): GEMM weights after a
// load, and gradients onto the bf16 all-reduce wire
__device__ __forceinline__ uint32_t tkm_bf16_bits(float f) {
  const uint32_t u = __float_as_uint(f);
  const uint32_t r = ((u & 0x7F800000u) == 0x7F800000u && (u & 0x7FFFFFu)) ? (u | 0x400000u)
                                                                          : u + 0x7FFFu + ((u >> 16) & 1u);
  return r >> 16;
}

// Eight values per thread and step (two 16-byte loads, one 16-byte store)
// when both pointers are 16-byte aligned, the rest one by one.
extern "C" __global__ void __launch_bounds__(256) tkm_f32_to_bf16(const float* __restrict__ src, uint16_t* __restrict__ dst,
                                                                  long long n) {
  const long long stride = (long long)gridDim.x * 256;
  long long done = 0;
  if ((((uint64_t)src | (uint64_t)dst) & 15) == 0) {
    const long long n8 = n >> 3;
    for (long long i = blockIdx.x * 256ll + threadIdx.x; i < n8; i += stride) {
      const float4 a = reinterpret_cast<const float4*>(src)[2 * i], b = reinterpret_cast<const float4*>(src)[2 * i + 1];
      uint4 o;
      o.x = tkm_bf16_bits(a.x) | (tkm_bf16_bits(a.y) << 16);
      o.y = tkm_bf16_bits(a.z) | (tkm_bf16_bits(a.w) << 16);
      o.z = tkm_bf16_bits(b.x) | (tkm_bf16_bits(b.y) << 16);
      o.w = tkm_bf16_bits(b.z) | (tkm_bf16_bits(b.w) << 16);
      reinterpret_cast<uint4*>(dst)[i] = o;
    }
    done = n8 << 3;
  }
  for (long long i = done + blockIdx.x * 256ll + threadIdx.x; i < n; i += stride) dst[i] = (uint16_t)tkm_bf16_bits(src[i]);
}

// bf16 -> fp32 (gradients coming back from a bf16 all-reduce), vectorised as above
extern "C" __global__ void __launch_bounds__(256) tkm_bf16_to_f32(const uint16_t* __restrict__ src, float* __restrict__ dst,
                                                                  long long n) {
  const long long stride = (long long)gridDim.x * 256;
  long long done = 0;
  if ((((uint64_t)src | (uint64_t)dst) & 15) == 0) {
    const long long n8 = n >> 3;
    for (long long i = blockIdx.x * 256ll + threadIdx.x; i < n8; i += stride) {
      const uint4 v = reinterpret_cast<const uint4*>(src)[i];
      reinterpret_cast<float4*>(dst)[2 * i] =
          make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xFFFF0000u), __uint_as_float(v.y << 16),
                      __uint_as_float(v.y & 0xFFFF0000u));
      reinterpret_cast<float4*>(dst)[2 * i + 1] =
          make_float4(__uint_as_float(v.z << 16), __uint_as_float(v.z & 0xFFFF0000u), __uint_as_float(v.w << 16),
                      __uint_as_float(v.w & 0xFFFF0000u));
    }
    done = n8 << 3;
  }
  for (long long i = done + blockIdx.x * 256ll + threadIdx.x; i < n; i += stride)
    dst[i] = __uint_as_float((uint32_t)src[i] << 16);
}

// ------------------------------------------- device-resident datasets
// One batch of a resident dataset: sample i of batch b is sample order[b*B + i]
// (b read from *batch).  Its `per` input values (activation storage) are copied
// by blockIdx.y-strided 16-byte chunks when they allow it, and its
// labels_per_sample int32 labels follow.  Grid (B, chunks).
extern "C" __global__ void __launch_bounds__(256) tkm_ds_gather(const tkm_act_t* __restrict__ src,
                                                                const int* __restrict__ labels,
                                                                const unsigned* __restrict__ order,
                                                                const unsigned* __restrict__ batch,
                                                                tkm_act_t* __restrict__ dst, int* __restrict__ dlabels,
                                                                long long per, int labels_per_sample, int B) {
  const int i = blockIdx.x;
  const unsigned s = order[(size_t)(*batch) * B + i];
  const tkm_act_t* in = src + (size_t)s * per;
  tkm_act_t* out = dst + (size_t)i * per;
  const int vec = 16 / (int)sizeof(tkm_act_t);
  if (per % vec == 0) {
    const long long nv = per / vec;
    for (long long k = blockIdx.y * 256ll + threadIdx.x; k < nv; k += (long long)gridDim.y * 256)
      reinterpret_cast<uint4*>(out)[k] = reinterpret_cast<const uint4*>(in)[k];
  } else {
    for (long long k = blockIdx.y * 256ll + threadIdx.x; k < per; k += (long long)gridDim.y * 256) out[k] = in[k];
  }
  if (blockIdx.y == 0)
    for (int k = threadIdx.x; k < labels_per_sample; k += 256)
      dlabels[(size_t)i * labels_per_sample + k] = labels[(size_t)s * labels_per_sample + k];
}

// One batch of token sequences: sequence i of batch b is order[b*B + i] in
// tokens[n][S+1]; input row (i, p) is the embedding row table[tokens[p]]
// (activation storage, C values) and its label is tokens[p+1].  Grid (B, S).
extern "C" __global__ void __launch_bounds__(256) tkm_ds_tokens(const tkm_act_t* __restrict__ table,
                                                                const int* __restrict__ tokens,
                                                                const unsigned* __restrict__ order,
                                                                const unsigned* __restrict__ batch,
                                                                tkm_act_t* __restrict__ dst, int* __restrict__ dlabels,
                                                                int S, int C, int B) {
  const int i = blockIdx.x, p = blockIdx.y;
  const unsigned s = order[(size_t)(*batch) * B + i];
  const int* seq = tokens + (size_t)s * (S + 1);
  const int tok = seq[p];
  const tkm_act_t* in = table + (size_t)tok * C;
  tkm_act_t* out = dst + ((size_t)i * S + p) * C;
  const int vec = 16 / (int)sizeof(tkm_act_t);
  if (C % vec == 0) {
    for (int k = threadIdx.x; k < C / vec; k += 256) reinterpret_cast<uint4*>(out)[k] = reinterpret_cast<const uint4*>(in)[k];
  } else {
    for (int k = threadIdx.x; k < C; k += 256) out[k] = in[k];
  }
  if (threadIdx.x == 0) dlabels[(size_t)i * S + p] = seq[p + 1];
}

// Learning rate of the step about to run: lr_table[*batch].
extern "C" __global__ void tkm_ds_lr(const float* __restrict__ lr_table, const unsigned* __restrict__ batch,
                                     float* __restrict__ lr) {
  if (threadIdx.x == 0) *lr = lr_table[*batch];
}

// After a step: the epoch's loss sum grows by the step's loss; next batch.
extern "C" __global__ void tkm_ds_end(const float* __restrict__ loss, float* __restrict__ loss_sum,
                                      unsigned* __restrict__ batch) {
  if (threadIdx.x == 0) {
    *loss_sum += *loss;
    *batch += 1u;
  }
}

// uint8 class labels (one per sample, the reference's format) -> int32 per row
extern "C" __global__ void __launch_bounds__(256) tkm_labels_u8(const uint8_t* __restrict__ src, int n_src,
                                                                int* __restrict__ dst, int rows) {
  for (int i = blockIdx.x * 256 + threadIdx.x; i < rows; i += gridDim.x * 256) dst[i] = i < n_src ? (int)src[i] : 0;
}

// learnable-tensor initialisation on the device: std > 0 draws N(0, std) from
// a counter-based generator (splitmix64 of seed and index, Box-Muller), else
// every value is `constant`
__device__ __forceinline__ uint64_t tkm_splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

extern "C" __global__ void __launch_bounds__(256) tkm_fill_param(float* __restrict__ p, long long n, uint64_t seed,
                                                                 float std, float constant) {
  for (long long i = (blockIdx.x * 256ll + threadIdx.x) * 2; i < n; i += (long long)gridDim.x * 512) {
    if (std > 0.f) {
      const uint64_t r = tkm_splitmix64(seed * 0x100000001B3ull + (uint64_t)i);
      const float u1 = ((float)(r >> 40) + 1.0f) * (1.0f / 16777217.0f);
      const float u2 = (float)((r >> 16) & 0xFFFFFFu) * (1.0f / 16777216.0f);
      const float m = sqrtf(-2.0f * logf(u1)) * std;
      float s, c;
      sincosf(6.283185307f * u2, &s, &c);
      p[i] = m * c;
      if (i + 1 < n) p[i + 1] = m * s;
    } else {
      p[i] = constant;
      if (i + 1 < n) p[i + 1] = constant;
    }
  }
}
