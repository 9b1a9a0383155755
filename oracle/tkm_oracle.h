/*
 * tkm_oracle.h -- CPU restatement of Tokamak's GPU hot-path semantics.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * sm_100a kernels in tokamak_b200/csrc.  Only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline / --impl reference leg may load it.  Nothing on
 * the product path links or calls it.
 *
 * Every routine reads and writes fp32 host arrays and accumulates in fp64.
 * Each one cites the reference (BSODsystem32/Tokamak v4.1.0) file:line whose
 * behaviour it restates.  Where the reference GPU code has a defect the
 * oracle implements the documented math and says so in the comment.
 */
#ifndef TKM_ORACLE_H
#define TKM_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Packed QKV attention forward.
 * qkv  [B][S][(Hq+2*Hkv)*D]: Q heads at columns [h*D,(h+1)*D), K head g at
 *      (Hq+g)*D, V head g at (Hq+Hkv+g)*D            (src/tkm_gpu.cu:338,366-368)
 * out  [B][S][Hq*D]                                   (src/tkm_gpu.cu:311,431)
 * lse  [B*Hq][S], natural log: m + ln(l + 1e-8)        (src/tkm_gpu.cu:429-430)
 * GQA: kv head = q_head / (Hq/Hkv)                    (src/tkm_gpu.cu:315-316)
 * Causal mask: key > query excluded                    (src/tkm_gpu.cu:393) */
void tko_attn_fwd(const float *qkv, float *out, float *lse,
                  int B, int S, int Hq, int Hkv, int D, float scale, int causal);

/* Attention backward with the true gradients.  The reference kernel
 * (src/tkm_gpu.cu:440-598) computes D_i = rowsum(O*dO) (503-512),
 * P = exp(s*scale - LSE), dS = P*(dP - D)*scale (545-553) and dQ = dS*K
 * (557-564), but then writes dK := dQ and dV := dO (588-596).  The oracle
 * writes dK = dS^T Q and dV = P^T dO, summed over the query heads of each
 * KV head.  dqkv uses the packed layout of qkv and is overwritten. */
void tko_attn_bwd(const float *qkv, const float *out, const float *dout,
                  const float *lse, float *dqkv,
                  int B, int S, int Hq, int Hkv, int D, float scale, int causal);

/* Residual add followed by RMSNorm (src/tkm_registry.c:228-245 RMSNorm spec,
 * 435-439 Add spec; docs/SPEC_DSL.md RMSNorm: x / RMS(x) * gamma).
 * s = x + r (r may be NULL), istd = 1/sqrt(mean(s^2) + eps), y = s*istd*gamma.
 * The reduction spans the whole row; the reference's generated kernel only
 * reduces one warp when C > 64 (src/tkm_codegen.c:491,496). */
void tko_add_rmsnorm_fwd(const float *x, const float *r, float *s, float *y,
                         const float *gamma, float *istd, int rows, int C, float eps);

/* Backward of tko_add_rmsnorm_fwd (src/tkm_registry.c:239-245):
 * xh = s*istd, dx = istd*(g*dy - xh*mean(g*dy*xh)) + ds_skip (ds_skip may be
 * NULL), dgamma += sum_rows(dy*xh).  dgamma is accumulated, not overwritten. */
void tko_add_rmsnorm_bwd(const float *dy, const float *s, const float *gamma,
                         const float *istd, const float *ds_skip, float *dx,
                         float *dgamma, int rows, int C);

/* SwiGLU twin epilogue (src/tkm_registry.c:653-686 twin merge,
 * src/tkm_codegen.c:511-518 fwd, 540-598 bwd; SiLU spec tkm_registry.c:272-278).
 * gu [rows][2F]: gate in [0,F), up in [F,2F).  a = g + bg, b = u + bu,
 * h = silu(a) * b.  Biases may be NULL (treated as zero). */
void tko_swiglu_fwd(const float *gu, const float *bg, const float *bu, float *h,
                    int rows, int F);
/* dgu overwritten; dbg/dbu accumulated (may be NULL). */
void tko_swiglu_bwd(const float *dh, const float *gu, const float *bg, const float *bu,
                    float *dgu, float *dbg, float *dbu, int rows, int F);

/* QKV prep: bias add, optional per-head QKNorm, RoPE on the Q and K columns
 * (src/tkm_codegen.c:211-252 fwd, 43-70 rotation).  Pair index i within a
 * head rotates by pos * theta^(-i/hd) (the reference's convention), with the
 * reference's Llama-3 frequency adjustment when rope_scale > 1.  pos = row % S.
 * qk_gain has Hq*D + Hkv*D entries (QKNorm gamma), may be NULL without QKNorm.
 * save_istd is [rows][Hq+Hkv] (one value per head; the reference stores one
 * per row, src/tkm_codegen.c:243, which loses all but one head). */
void tko_qkv_prep_fwd(const float *in, const float *bias, const float *qk_gain,
                      float *out, float *save_istd,
                      int rows, int S, int Hq, int Hkv, int D,
                      int has_qknorm, int has_rope, float theta, float rope_scale,
                      float low_ff, float high_ff, float orig_ctx);
/* Backward (src/tkm_codegen.c:254-295): inverse rotation, QKNorm VJP,
 * din accumulated, dbias accumulated, dgain accumulated (the reference's
 * dgain flush never runs, src/tkm_codegen.c:276). */
void tko_qkv_prep_bwd(const float *dout, const float *in, const float *bias,
                      const float *qk_gain, const float *save_istd,
                      float *din, float *dbias, float *dgain,
                      int rows, int S, int Hq, int Hkv, int D,
                      int has_qknorm, int has_rope, float theta, float rope_scale,
                      float low_ff, float high_ff, float orig_ctx);

/* Row softmax and its VJP (src/tkm_gpu.cu:600-630); dx is accumulated. */
void tko_softmax_fwd(const float *x, float *p, int rows, int C);
void tko_softmax_bwd(const float *p, const float *dp, float *dx, int rows, int C);

/* Fused softmax loss forward+backward (src/tkm_gpu.cu:632-682).
 * kind 0 = cross-entropy, 1 = focal(gamma), 2 = Brier.  Labels are one int32
 * per row.  Returns the loss (mean over rows).  dlogits overwritten.
 * *correct (may be NULL) receives the argmax==label count. */
float tko_softmax_loss(const float *logits, const int32_t *labels, float *dlogits,
                       int *correct, int rows, int C, int kind, float gamma);

/* SGD with momentum as in src/tkm_gpu.cu:695-720: g += wd*p when apply_wd,
 * v = m*v + g, p -= lr*(m*v + g). */
void tko_sgd(float *p, float *v, const float *g, long n, float lr, float momentum,
             float wd, int apply_wd);

/* Number of OpenMP threads the oracle will use. */
int tko_num_threads(void);
void tko_set_num_threads(int n);

#ifdef __cplusplus
}
#endif
#endif
