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
  const float* nlse2;         // [B*Hq][S_pad]  -LSE * log2(e), -inf on padded rows
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

// GEMM parameters: C[M][N] (+)= A[M][K] B[K][N], bf16 operands, fp32 accumulation.
// tmA / tmB are 2-D maps with 128-byte swizzle: a K-major operand (K contiguous)
// as {K, rows} with box {64, 128 (A) or 256 (B)}; an MN-major operand (M or N
// contiguous) as {cols, K} with box {64, 64}.
struct alignas(64) GemmParams {
  CUtensorMap tmA, tmB;
  void* c;                    // C, row-major, ldc elements per row (bf16 or fp32)
  long long ldc;
  void* h;                    // SwiGLU: h[M][F], ldh elements per row (bf16)
  long long ldh;
  const float* bias;          // per-column bias of C (or the gate bias for SwiGLU); may be null
  const float* bias2;         // SwiGLU: up bias; may be null
  int M, N, K;                // N: columns of C (SwiGLU: F, the columns of h)
  int tiles_m, tiles_n;
  int b_split;                // SwiGLU: column of B where the up half starts (F)
  int accumulate;             // C += result
  int out_f32;                // C is fp32 (else bf16)
  int splits;                 // CTA-pair form, fp32 C: K split over this many partial sums (1: none)
  int kb_per_split;           // 64-deep K blocks per split
  float* ws;                  // splits > 1: partial sums [splits][M][N], summed into C in split order
  // LM head + softmax cross-entropy (C = logits + bias, never stored):
  const int* labels;          // [M] class of each row
  float4* ce_part;            // statistics pass: [M][tiles_n] (tile max, sum of exp(x - max), argmax bits, 0)
  float* ce_lab;              // statistics pass: [M] the label's logit
  const float* ce_lse;        // gradient pass: [M] log-sum-exp of each row
  float ce_scale;             // gradient pass: 1 / rows
};

cudaError_t gemm_tc(const GemmParams& p, bool a_mn, bool b_mn, int epi, cudaStream_t stream);
// The same on CTA pairs (256 x 256 tiles; tiles_m counts 256-row tiles, a
// K-major B map has 128-row boxes).
cudaError_t gemm_pair_tc(const GemmParams& p, bool a_mn, bool b_mn, int epi, cudaStream_t stream);
// C (+)= sum over s of ws[s][M][N], s in order (the split-K partials; fp32 C).
cudaError_t gemm_splitk_reduce(const GemmParams& p, cudaStream_t stream);
// Per row: LSE from the statistics pass's tile partials, the cross-entropy
// term min(LSE - label logit, -ln 1e-7) / rows into row_loss, correct += argmax == label.
cudaError_t ce_combine(const float4* part, int tiles_n, const float* lab_logit, const int* labels, float* lse,
                       float* row_loss, int* correct, int rows, float inv_rows, cudaStream_t stream);

cudaError_t attn_fwd_tc(const FwdParams& p, int D, bool bf16, cudaStream_t stream);
cudaError_t attn_bwd_tc(const BwdParams& p, int D, bool bf16, cudaStream_t stream);

// Builds a 3-D tensor map over a row-major [batch][rows][cols] 16-bit array
// whose rows are row_stride elements apart.  Box: 64 columns x 128 rows.
cudaError_t make_tmap_rows(CUtensorMap* m, const void* base, bool bf16, long long cols, long long rows,
                           long long batch, long long row_stride, long long batch_stride);

}  // namespace tkb
