// attn_aux.cu -- helpers around the tcgen05 attention kernels:
//   * tensor-map construction (driver entry point fetched through the runtime,
//     so the library never links libcuda directly),
//   * the backward preprocess (Delta = rowsum(O*dO), LSE in log2 units, both
//     padded to a multiple of 128 rows per head).
#include "tkb_common.cuh"
#include "tkb_internal.h"

namespace tkb {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

cudaError_t make_tmap_rows(CUtensorMap* m, const void* base, bool bf16, long long cols, long long rows,
                           long long batch, long long row_stride, long long batch_stride) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_stride * 2) % 16 || (batch_stride * 2) % 16)
    return cudaErrorMisalignedAddress;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(row_stride * 2), static_cast<cuuint64_t>(batch_stride * 2)};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// 2-D tensor map over a row-major 16-bit (bf16) array of `outer` rows of `inner`
// elements, rows `ld` elements apart; box {box_inner, box_outer}, 128-byte swizzle.
cudaError_t make_tmap_2d(CUtensorMap* m, const void* base, long long inner, long long outer, long long ld,
                         int box_inner, int box_outer) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld * 2) % 16) return cudaErrorMisalignedAddress;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// Rows of the padded sequence are spread over the lanes: D/8 lanes per row
// (one 16-byte chunk of O and of dO each), 32/(D/8) rows per warp per pass,
// UNROLL passes with their loads issued before any reduction.  A warp's
// ROWS rows (8 or 16, dividing the 128-row padding) share one (batch, head),
// so the row decomposition takes one 32-bit division pair per warp pass; with
// 64-bit divisions per row the kernel was issue-bound (57 % issue active, 70
// registers, 0.39 of peak DRAM throughput): 89 -> 51 us at B=8, H=16,
// S=4096, D=128 (5.3 TB/s), 44 -> 28 us at D=64.  Eight passes in flight per
// warp instead of four (103 registers) measured 63 us.
template <int D, bool BF16>
__global__ void __launch_bounds__(256) attn_bwd_pre_kernel(const void* __restrict__ out, const void* __restrict__ dout,
                                                           const float* __restrict__ lse, float* __restrict__ nlse2,
                                                           float* __restrict__ delta, long long o_row_stride, long long o_batch_stride, int B,
                                                           int S, int S_pad, int Hq) {
  constexpr int LPR = D / 8, RPW = 32 / LPR, UNROLL = 4, ROWS = RPW * UNROLL;
  const unsigned total = static_cast<unsigned>(B) * Hq * S_pad;
  const int lane = threadIdx.x & 31, sub = lane / LPR, chunk = lane % LPR;
  const unsigned warps = (gridDim.x * blockDim.x) >> 5;
  const long long rstride = o_row_stride * 2;
  for (unsigned w0 = ((blockIdx.x * blockDim.x + threadIdx.x) >> 5) * ROWS; w0 < total; w0 += warps * ROWS) {
    const unsigned bh = w0 / static_cast<unsigned>(S_pad);
    const int row0 = static_cast<int>(w0 - bh * static_cast<unsigned>(S_pad));
    const unsigned b = bh / static_cast<unsigned>(Hq), h = bh - b * static_cast<unsigned>(Hq);
    const long long base = (static_cast<long long>(b) * o_batch_stride + static_cast<long long>(row0 + sub) * o_row_stride +
                            static_cast<long long>(h) * D) * 2 + chunk * 16;
    const uint8_t* po = reinterpret_cast<const uint8_t*>(out) + base;
    const uint8_t* pd = reinterpret_cast<const uint8_t*>(dout) + base;
    uint4 o[UNROLL], d[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      o[u] = d[u] = make_uint4(0, 0, 0, 0);
      if (row0 + u * RPW + sub < S) {
        o[u] = __ldcs(reinterpret_cast<const uint4*>(po + u * RPW * rstride));
        d[u] = __ldcs(reinterpret_cast<const uint4*>(pd + u * RPW * rstride));
      }
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const uint32_t* ow = reinterpret_cast<const uint32_t*>(&o[u]);
      const uint32_t* dw = reinterpret_cast<const uint32_t*>(&d[u]);
      float acc = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 a = unpack2<BF16>(ow[e]), c = unpack2<BF16>(dw[e]);
        acc = fmaf(a.x, c.x, fmaf(a.y, c.y, acc));
      }
#pragma unroll
      for (int m = LPR / 2; m >= 1; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
      const int row = row0 + u * RPW + sub;
      if (chunk == 0) {
        const unsigned wrow = w0 + u * RPW + sub;
        delta[wrow] = row < S ? acc : 0.f;
        nlse2[wrow] = row < S ? lse[static_cast<long long>(bh) * S + row] * -1.4426950408889634f : -INFINITY;
      }
    }
  }
}

static int grid_for(long long work, int per_block) {
  long long g = (work + per_block - 1) / per_block;
  const long long cap = 148LL * 16;
  return static_cast<int>(g < 1 ? 1 : (g > cap ? cap : g));
}

cudaError_t attn_bwd_pre(const void* out, const void* dout, const float* lse, float* nlse2, float* delta,
                         long long o_row_stride, long long o_batch_stride, int B, int S, int S_pad,
                         int Hq, int D, bool bf16, cudaStream_t st) {
  // 8 warps per block, each covering 8 (D = 128) or 16 (D = 64) rows per pass;
  // row indices are 32-bit
  if (static_cast<long long>(B) * Hq * S_pad >= (1LL << 31)) return cudaErrorInvalidValue;
  const int grid = grid_for(static_cast<long long>(B) * Hq * S_pad, 8 * (D == 64 ? 16 : 8));
#define TKB_PRE(DD, BB) \
  attn_bwd_pre_kernel<DD, BB><<<grid, 256, 0, st>>>(out, dout, lse, nlse2, delta, o_row_stride, o_batch_stride, B, S, S_pad, Hq)
  if (D == 128) { if (bf16) TKB_PRE(128, true); else TKB_PRE(128, false); }
  else if (D == 64) { if (bf16) TKB_PRE(64, true); else TKB_PRE(64, false); }
  else return cudaErrorInvalidValue;
#undef TKB_PRE
  return cudaGetLastError();
}

}  // namespace tkb
