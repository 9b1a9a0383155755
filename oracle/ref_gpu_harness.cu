// ref_gpu_harness.cu -- TEST INFRASTRUCTURE ONLY.
//
// Compiles the reference's own src/tkm_gpu.cu where it lies (the include path
// is given by oracle/build_ref.py) together with its other sources into
// oracle/_ref/libtkm_ref.so, and adds extern "C" launchers for the reference's
// static kernels so the parity tests can run them on the B200 with the exact
// grids of the reference's launch sites.  Nothing here is part of the product.
#include "tkm_gpu.cu"

extern "C" {

// Launch site src/tkm_gpu.cu:1252-1265.
int ref_attn_fwd(const void* qkv, void* out, float* lse, int B, int S, int Hq, int Hkv, int D, float scale,
                 int causal, void* stream) {
  cudaStream_t st = (cudaStream_t)stream;
  dim3 grid(B * Hq, (S + 31) / 32);
  if (D == 64)
    k_gqa_flash_attn_tc_fwd<64><<<grid, 64, 0, st>>>((const __half*)qkv, (__half*)out, lse, B, S, Hq, Hkv, scale,
                                                    causal);
  else if (D == 128)
    k_gqa_flash_attn_tc_fwd<128><<<grid, 64, 0, st>>>((const __half*)qkv, (__half*)out, lse, B, S, Hq, Hkv, scale,
                                                     causal);
  else
    return -1;
  return (int)cudaGetLastError();
}

// Launch site src/tkm_gpu.cu:1389-1403.
int ref_attn_bwd(const void* qkv, const void* out, const void* dout, const float* lse, void* dqkv, int B, int S,
                 int Hq, int Hkv, int D, float scale, int causal, void* stream) {
  cudaStream_t st = (cudaStream_t)stream;
  dim3 grid(B * Hq, (S + 31) / 32);
  if (D == 64)
    k_gqa_flash_attn_tc_bwd<64><<<grid, 64, 0, st>>>((const __half*)qkv, (const __half*)out, (const __half*)dout,
                                                    lse, (__half*)dqkv, B, S, Hq, Hkv, scale, causal);
  else if (D == 128)
    k_gqa_flash_attn_tc_bwd<128><<<grid, 64, 0, st>>>((const __half*)qkv, (const __half*)out, (const __half*)dout,
                                                     lse, (__half*)dqkv, B, S, Hq, Hkv, scale, causal);
  else
    return -1;
  return (int)cudaGetLastError();
}

// Launch site src/tkm_gpu.cu:1275-1284 (training mode: is_eval = 0).
int ref_softmax_loss(const void* logits, const uint8_t* labels, void* dlogits, float* loss, int* correct, int rows,
                     int cols, int kind, float gamma, void* stream) {
  cudaStream_t st = (cudaStream_t)stream;
  k_softmax_loss_fwd_bwd_h<<<(rows + 255) / 256, 256, 0, st>>>((const __half*)logits, labels, (__half*)dlogits, loss,
                                                              correct, rows, cols, 0, rows, kind, gamma);
  return (int)cudaGetLastError();
}

// Launch sites src/tkm_gpu.cu:1270-1274 and 1409-1412.
int ref_softmax_fwd(const void* x, void* p, int rows, int cols, void* stream) {
  k_softmax_fwd_h<<<(rows + 255) / 256, 256, 0, (cudaStream_t)stream>>>((const __half*)x, (__half*)p, rows, cols);
  return (int)cudaGetLastError();
}
int ref_softmax_bwd(const void* p, const void* dp, void* dx, int rows, int cols, void* stream) {
  k_softmax_bwd_h<<<(rows + 255) / 256, 256, 0, (cudaStream_t)stream>>>((const __half*)p, (const __half*)dp,
                                                                        (__half*)dx, rows, cols);
  return (int)cudaGetLastError();
}

}  // extern "C"
