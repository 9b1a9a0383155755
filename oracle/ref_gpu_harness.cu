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

// Launch site src/tkm_gpu.cu:1417-1420, with the tensor table the runtime
// uploads at src/tkm_gpu.cu:1127 (SgdTensorList in constant memory).  The
// pointer arrays are host arrays of device pointers; fp16[i] may be null.
int ref_sgd(float* const* master, __half* const* fp16, float* const* vel, const float* const* grad,
            const int* sizes, int count, const float* d_lr, float momentum, float wd, uint32_t* d_seed,
            void* stream) {
  if (count <= 0 || count > TKM_MAX_TENSORS) return -1;
  SgdTensorList h;
  memset(&h, 0, sizeof(h));
  h.count = count;
  for (int i = 0; i < count; i++) {
    h.master[i] = master[i];
    h.fp16_w[i] = fp16[i];
    h.vel[i] = vel[i];
    h.grad[i] = grad[i];
    h.size[i] = sizes[i];
    h.offset[i + 1] = h.offset[i] + sizes[i];
  }
  cudaError_t e = cudaMemcpyToSymbol(c_tkm_sgd, &h, sizeof(SgdTensorList));
  if (e != cudaSuccess) return (int)e;
  const int total = h.offset[count];
  k_tkm_multi_tensor_sgd<<<(total + 255) / 256, 256, 0, (cudaStream_t)stream>>>(d_lr, momentum, wd, d_seed);
  return (int)cudaGetLastError();
}

// The fused QKV-prep group of a reference runtime after a forward pass: the
// node ids of the fused [Q|K|V] GEMM (the group's input) and of the prep node
// (src/tkm_registry.c:701-770 rewrites the Q chain's first node into it), and
// their fp16 activations copied to host buffers of `elems` halves each.
int ref_qkv_prep_acts(TkmRuntime* rt, int* gemm_id, int* prep_id, void* h_in, void* h_out, size_t elems) {
  const TkmGraph* g = &rt->graph;
  int prep = -1;
  for (int i = 0; i < g->num_nodes; i++)
    if (!g->nodes[i].dead && g->nodes[i].op == OP_QKNORM && g->nodes[i].in0 >= 0 &&
        g->nodes[g->nodes[i].in0].op == OP_FC_QKV_FUSED)
      prep = i;
  if (prep < 0) return -1;
  const TkmNode* pn = &g->nodes[prep];
  const TkmNode* fn = &g->nodes[pn->in0];
  const size_t need = (size_t)g->batch_size * pn->H * pn->W * pn->c_out;
  if (need != elems) return -2;
  cudaDeviceSynchronize();
  cudaError_t e = cudaMemcpy(h_in, rt->d_arena + fn->out_offset, elems * sizeof(__half), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess)
    e = cudaMemcpy(h_out, rt->d_arena + pn->out_offset, elems * sizeof(__half), cudaMemcpyDeviceToHost);
  *gemm_id = fn->id;
  *prep_id = prep;
  return (int)e;
}

}  // extern "C"
