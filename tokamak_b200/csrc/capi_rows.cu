// capi_rows.cu -- extern "C" entry points of the row kernels (include/tkm_b200.h).
// Compiled in the same translation unit as rows.cu and capi.cu (tkb_all.cu).
#include <cmath>
#include <cstring>

namespace {

int row_check(const char* who, int rows, int C, int dtype) {
  if (rows <= 0 || C <= 0) return fail(TKB_ERR_ARG, "%s: rows and C must be positive", who);
  if (C % 2) return fail(TKB_ERR_ARG, "%s: C must be even (got %d)", who, C);
  if (!dtype_ok(dtype)) return fail(TKB_ERR_ARG, "%s: bad dtype %d", who, dtype);
  return TKB_OK;
}

// Row pointers for the softmax losses: rows whose width is a multiple of 8
// move in 16-byte vectors (and 16-bit rows of 8192-32768 by bulk copies,
// which need 16-byte addresses); other widths in pairs of elements.
bool loss_rows_aligned(const void* p, int C, int dtype) {
  if (!p) return true;
  const uintptr_t need = C % 8 == 0 ? 16u : (dtype == TKB_F32 ? 8u : 4u);
  return reinterpret_cast<uintptr_t>(p) % need == 0;
}

// Calls F<T>(...) for the runtime dtype.
#define TKB_BY_DTYPE(DT, CALL)                         \
  ((DT) == TKB_F32    ? CALL(float)                    \
   : (DT) == TKB_BF16 ? CALL(__nv_bfloat16)            \
                      : CALL(__half))

}  // namespace

extern "C" {

int tkb_add_rmsnorm_fwd(const void* x, const void* r, void* s, void* y, const float* gamma, float* istd, int rows,
                        int C, float eps, int dtype, void* stream) {
  int rc = row_check("tkb_add_rmsnorm_fwd", rows, C, dtype);
  if (rc) return rc;
  if (!x || !y || !gamma) return fail(TKB_ERR_ARG, "tkb_add_rmsnorm_fwd: null pointer");
  if (r && !s) return fail(TKB_ERR_ARG, "tkb_add_rmsnorm_fwd: s is required when r is given");
  if (C > 256 * 8 * 16) return fail(TKB_ERR_UNSUPPORTED, "tkb_add_rmsnorm_fwd: C > 32768");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define CALL(T) add_rmsnorm_fwd_t<T>(x, r, s, y, gamma, istd, rows, C, eps, st)
  return cuda_status(TKB_BY_DTYPE(dtype, CALL), "tkb_add_rmsnorm_fwd", 1);
#undef CALL
}

size_t tkb_add_rmsnorm_bwd_workspace(int rows, int C) {
  if (rows <= 0 || C <= 0) return 0;
  return round256(static_cast<size_t>(add_rmsnorm_bwd_grid(rows)) * C * 4);
}

int tkb_add_rmsnorm_bwd(const void* dy, const void* s, const float* gamma, const float* istd, const void* ds_skip,
                        void* dx, float* dgamma, void* workspace, size_t workspace_bytes, int rows, int C, int dtype,
                        void* stream) {
  int rc = row_check("tkb_add_rmsnorm_bwd", rows, C, dtype);
  if (rc) return rc;
  if (!dy || !s || !gamma || !istd || !dx) return fail(TKB_ERR_ARG, "tkb_add_rmsnorm_bwd: null pointer");
  if (C > 256 * 8 * 16) return fail(TKB_ERR_UNSUPPORTED, "tkb_add_rmsnorm_bwd: C > 32768");
  if (dgamma && (!workspace || workspace_bytes < tkb_add_rmsnorm_bwd_workspace(rows, C)))
    return fail(TKB_ERR_WORKSPACE, "tkb_add_rmsnorm_bwd: workspace of %zu bytes required",
                tkb_add_rmsnorm_bwd_workspace(rows, C));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define CALL(T) add_rmsnorm_bwd_t<T>(dy, s, gamma, istd, ds_skip, dx, dgamma, static_cast<float*>(workspace), rows, C, st)
  return cuda_status(TKB_BY_DTYPE(dtype, CALL), "tkb_add_rmsnorm_bwd", dgamma ? 2 : 1);
#undef CALL
}

int tkb_swiglu_fwd(const void* gu, const float* bg, const float* bu, void* h, int rows, int F, int dtype,
                   void* stream) {
  int rc = row_check("tkb_swiglu_fwd", rows, F, dtype);
  if (rc) return rc;
  if (!gu || !h) return fail(TKB_ERR_ARG, "tkb_swiglu_fwd: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define CALL(T) swiglu_fwd_t<T>(gu, bg, bu, h, rows, F, st)
  return cuda_status(TKB_BY_DTYPE(dtype, CALL), "tkb_swiglu_fwd", 1);
#undef CALL
}

size_t tkb_swiglu_bwd_workspace(int rows, int F) {
  if (rows <= 0 || F <= 0) return 0;
  int gx, gy;
  swiglu_grid(rows, F, (F % 8 == 0) ? 8 : 2, gx, gy);
  return round256(static_cast<size_t>(gy) * 2 * F * 4);
}

int tkb_swiglu_bwd(const void* dh, const void* gu, const float* bg, const float* bu, void* dgu, float* dbg,
                   float* dbu, void* workspace, size_t workspace_bytes, int rows, int F, int dtype, void* stream) {
  int rc = row_check("tkb_swiglu_bwd", rows, F, dtype);
  if (rc) return rc;
  if (!dh || !gu || !dgu) return fail(TKB_ERR_ARG, "tkb_swiglu_bwd: null pointer");
  if ((dbg || dbu) && (!workspace || workspace_bytes < tkb_swiglu_bwd_workspace(rows, F)))
    return fail(TKB_ERR_WORKSPACE, "tkb_swiglu_bwd: workspace of %zu bytes required", tkb_swiglu_bwd_workspace(rows, F));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define CALL(T) swiglu_bwd_t<T>(dh, gu, bg, bu, dgu, dbg, dbu, static_cast<float*>(workspace), rows, F, st)
  return cuda_status(TKB_BY_DTYPE(dtype, CALL), "tkb_swiglu_bwd", (dbg || dbu) ? 2 : 1);
#undef CALL
}

}  // extern "C"

namespace {

int qkv_check(const char* who, int rows, int S, int Hq, int Hkv, int D, int dtype) {
  if (rows <= 0 || S <= 0 || Hq <= 0 || Hkv < 0) return fail(TKB_ERR_ARG, "%s: bad shape", who);
  if (D != 64 && D != 128 && D != 32 && D != 16) return fail(TKB_ERR_UNSUPPORTED, "%s: head dim %d", who, D);
  if (!dtype_ok(dtype)) return fail(TKB_ERR_ARG, "%s: bad dtype %d", who, dtype);
  return TKB_OK;
}

// Per-pair inverse frequencies, src/tkm_codegen.c:43-70, evaluated in double.
RopeTable rope_table(int D, float theta, float scale, float lowf, float highf, float octx) {
  RopeTable t;
  memset(&t, 0, sizeof(t));
  for (int i = 0; i < D / 2 && i < 64; ++i) {
    double inv = std::exp(-std::log(static_cast<double>(theta)) * i / static_cast<double>(D));
    if (scale > 1.0f) {
      const double wavelen = 6.283185307179586 / inv;
      const double low_w = static_cast<double>(octx) / lowf, high_w = static_cast<double>(octx) / highf;
      if (wavelen > low_w) inv /= scale;
      else if (wavelen >= high_w) {
        const double smooth = (static_cast<double>(octx) / wavelen - lowf) / (static_cast<double>(highf) - lowf);
        inv *= 1.0 - smooth * (1.0 - 1.0 / scale);
      }
    }
    t.inv_freq[i] = inv;
  }
  return t;
}

}  // namespace

extern "C" {

int tkb_qkv_prep_fwd(const void* in, const float* bias, const float* qk_gain, void* out, float* save_istd, int rows,
                     int S, int Hq, int Hkv, int D, int has_qknorm, int has_rope, float theta, float rope_scale,
                     float low_ff, float high_ff, float octx, int dtype, void* stream) {
  int rc = qkv_check("tkb_qkv_prep_fwd", rows, S, Hq, Hkv, D, dtype);
  if (rc) return rc;
  if (!in || !out) return fail(TKB_ERR_ARG, "tkb_qkv_prep_fwd: null pointer");
  if (has_qknorm && !save_istd) return fail(TKB_ERR_ARG, "tkb_qkv_prep_fwd: QKNorm needs save_istd");
  const RopeTable tab = rope_table(D, theta, rope_scale, low_ff, high_ff, octx);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define CALL(T) qkv_prep_fwd_t<T>(in, bias, qk_gain, out, save_istd, rows, S, Hq, Hkv, D, has_qknorm, has_rope, tab, st)
  return cuda_status(TKB_BY_DTYPE(dtype, CALL), "tkb_qkv_prep_fwd", 1);
#undef CALL
}

size_t tkb_qkv_prep_bwd_workspace(int rows, int Hq, int Hkv, int D) {
  if (rows <= 0 || Hq <= 0 || D <= 0) return 0;
  const size_t C = static_cast<size_t>(Hq + 2 * Hkv) * D, G = static_cast<size_t>(Hq + Hkv) * D;
  return round256(static_cast<size_t>(qkv_prep_bwd_grid(rows)) * (C + G) * 4);
}

int tkb_qkv_prep_bwd(const void* dout, const void* in, const float* bias, const float* qk_gain,
                     const float* save_istd, void* din, float* dbias, float* dgain, void* workspace,
                     size_t workspace_bytes, int rows, int S, int Hq, int Hkv, int D, int has_qknorm, int has_rope,
                     float theta, float rope_scale, float low_ff, float high_ff, float octx, int dtype, void* stream) {
  int rc = qkv_check("tkb_qkv_prep_bwd", rows, S, Hq, Hkv, D, dtype);
  if (rc) return rc;
  if (!dout || !din || (has_qknorm && (!in || !save_istd))) return fail(TKB_ERR_ARG, "tkb_qkv_prep_bwd: null pointer");
  const bool want = dbias || (has_qknorm && dgain);
  if (want && (!workspace || workspace_bytes < tkb_qkv_prep_bwd_workspace(rows, Hq, Hkv, D)))
    return fail(TKB_ERR_WORKSPACE, "tkb_qkv_prep_bwd: workspace of %zu bytes required",
                tkb_qkv_prep_bwd_workspace(rows, Hq, Hkv, D));
  const RopeTable tab = rope_table(D, theta, rope_scale, low_ff, high_ff, octx);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define CALL(T)                                                                                                    \
  qkv_prep_bwd_t<T>(dout, in, bias, qk_gain, save_istd, din, dbias, dgain, static_cast<float*>(workspace), rows, S, \
                    Hq, Hkv, D, has_qknorm, has_rope, tab, st)
  return cuda_status(TKB_BY_DTYPE(dtype, CALL), "tkb_qkv_prep_bwd", want ? 2 : 1);
#undef CALL
}

int tkb_softmax_fwd(const void* x, void* p, int rows, int C, int dtype, void* stream) {
  int rc = row_check("tkb_softmax_fwd", rows, C, dtype);
  if (rc) return rc;
  if (!x || !p) return fail(TKB_ERR_ARG, "tkb_softmax_fwd: null pointer");
  if (C > 256 * 8 * 16) return fail(TKB_ERR_UNSUPPORTED, "tkb_softmax_fwd: C > 32768");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define CALL(T) softmax_fwd_t<T>(x, p, rows, C, st)
  return cuda_status(TKB_BY_DTYPE(dtype, CALL), "tkb_softmax_fwd", 1);
#undef CALL
}

int tkb_softmax_bwd(const void* p, const void* dp, void* dx, int rows, int C, int dtype, void* stream) {
  int rc = row_check("tkb_softmax_bwd", rows, C, dtype);
  if (rc) return rc;
  if (!p || !dp || !dx) return fail(TKB_ERR_ARG, "tkb_softmax_bwd: null pointer");
  if (C > 256 * 8 * 16) return fail(TKB_ERR_UNSUPPORTED, "tkb_softmax_bwd: C > 32768");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define CALL(T) softmax_bwd_t<T>(p, dp, dx, rows, C, st)
  return cuda_status(TKB_BY_DTYPE(dtype, CALL), "tkb_softmax_bwd", 1);
#undef CALL
}

size_t tkb_softmax_loss_workspace(int rows) { return rows > 0 ? round256(static_cast<size_t>(rows) * 4) : 0; }

int tkb_softmax_loss(const void* logits, const int32_t* labels, void* dlogits, float* loss, int* correct,
                     void* workspace, size_t workspace_bytes, int rows, int C, int kind, float gamma, int dtype,
                     void* stream) {
  int rc = row_check("tkb_softmax_loss", rows, C, dtype);
  if (rc) return rc;
  if (!logits) return fail(TKB_ERR_ARG, "tkb_softmax_loss: null logits");
  if (kind < 0 || kind > 2) return fail(TKB_ERR_ARG, "tkb_softmax_loss: kind %d not in {0,1,2}", kind);
  if (C > 256 * 8 * 16) return fail(TKB_ERR_UNSUPPORTED, "tkb_softmax_loss: C > 32768");
  if (!loss_rows_aligned(logits, C, dtype) || !loss_rows_aligned(dlogits, C, dtype))
    return fail(TKB_ERR_ARG, "tkb_softmax_loss: logits and dlogits must be 16-byte aligned when C %% 8 == 0 "
                "(else aligned to two elements)");
  if (loss && (!workspace || workspace_bytes < tkb_softmax_loss_workspace(rows)))
    return fail(TKB_ERR_WORKSPACE, "tkb_softmax_loss: workspace of %zu bytes required", tkb_softmax_loss_workspace(rows));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define CALL(T) softmax_loss_t<T>(logits, labels, dlogits, loss, correct, static_cast<float*>(workspace), rows, C, kind, gamma, st)
  return cuda_status(TKB_BY_DTYPE(dtype, CALL), "tkb_softmax_loss", loss ? 2 : 1);
#undef CALL
}

int tkb_sgd_step(const tkb_sgd_tensor* table, int n_tensors, const float* lr, float momentum, float weight_decay,
                 uint32_t* seed, void* stream) {
  if (!table || n_tensors <= 0 || !lr) return fail(TKB_ERR_ARG, "tkb_sgd_step: bad arguments");
  static_assert(sizeof(tkb_sgd_tensor) == sizeof(SgdTensor), "SGD record layout");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n_tensors <= SGD_MAXT) {
    sgd_kernel<<<148 * 8, 256, 0, st>>>(reinterpret_cast<const SgdTensor*>(table), n_tensors, lr, momentum,
                                        weight_decay, seed);
  } else {
    const int gy = n_tensors < 65535 ? n_tensors : 65535;
    sgd_kernel_many<<<dim3(64, gy), 256, 0, st>>>(reinterpret_cast<const SgdTensor*>(table), n_tensors, lr,
                                                  momentum, weight_decay, seed);
  }
  return cuda_status(cudaGetLastError(), "tkb_sgd_step", 1);
}

}  // extern "C"
