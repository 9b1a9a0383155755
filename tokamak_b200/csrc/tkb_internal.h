// tkb_internal.h -- launch parameter blocks and internal entry points shared
// between the kernel translation units and the C ABI layer (capi.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace tkb {

// Forward attention parameters.  Tensor maps are 3-D {columns, rows, batch}
// views of the Q, K and V column ranges (box 64 x 128 x 1, 128-byte swizzle).
struct alignas(64) FwdParams {
  CUtensorMap tmQ, tmK, tmV;
  void* out;                  // [B][S] rows of out_row_stride elements, head h at h*D
  float* lse;                 // [B*Hq][S], natural log
  long long out_row_stride;   // elements
  long long out_batch_stride; // elements
  int B, S, Hq, Hkv;
  int n_pairs;                // ceil(ceil(S/128) / 2)
  int causal;
  float scale_log2;           // softmax scale * log2(e)
};

// Backward attention parameters.
struct alignas(64) BwdParams {
  CUtensorMap tmQ, tmK, tmV, tmdO;
  uint16_t* ds;               // null: dQ recomputes S and dP; else dS tiles (see ds_tile)
  long long ds_tiles;         // dS tiles per (batch, q head)
  const float* lse2;          // [B*Hq][S_pad]  LSE * log2(e), +inf on padded rows
  const float* delta;         // [B*Hq][S_pad]  rowsum(O * dO), 0 on padded rows
  void* dq;                   // row-major, dkv_row_stride elements per row, head h at h*D
  void* dk;                   // row-major, dkv_row_stride elements per row, head g at g*D
  void* dv;
  long long dkv_row_stride;   // elements (dQ, dK, dV share the packed layout)
  long long dkv_batch_stride; // elements
  int B, S, S_pad, Hq, Hkv;
  int causal;
  float scale;                // softmax scale
  float scale_log2;           // softmax scale * log2(e)
};

cudaError_t attn_fwd_tc(const FwdParams& p, int D, bool bf16, cudaStream_t stream);
cudaError_t attn_bwd_tc(const BwdParams& p, int D, bool bf16, cudaStream_t stream);

// Builds a 3-D tensor map over a row-major [batch][rows][cols] 16-bit array
// whose rows are row_stride elements apart.  Box: 64 columns x 128 rows.
cudaError_t make_tmap_rows(CUtensorMap* m, const void* base, bool bf16, long long cols, long long rows,
                           long long batch, long long row_stride, long long batch_stride);

}  // namespace tkb
