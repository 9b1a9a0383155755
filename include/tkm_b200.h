/*
 * tkm_b200.h -- thin C ABI of the B200 (sm_100a) hot-path kernels.
 *
 * Plain pointers and sizes only.  Every pointer argument except those marked
 * "host" is a device pointer; `stream` is a cudaStream_t (NULL = legacy
 * default stream).  All calls are asynchronous on `stream` and return a
 * tkb_status; on failure tkb_last_error() gives a one-line reason.  A kernel
 * whose bounded internal wait ran out records a code that tkb_device_error()
 * reports (the kernel returns; the context stays usable).
 *
 * Each entry point names the reference (BSODsystem32/Tokamak v4.1.0) kernel
 * and launch site it replaces.  dtype selects the storage type of the
 * activation tensors: TKB_F32, TKB_BF16 or TKB_F16.  Parameter vectors
 * (RMSNorm gain, biases) are fp32 master copies, as in the reference
 * (NodeGpuState, src/tkm_gpu.cu:829-839).
 */
#ifndef TKM_B200_H
#define TKM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum { TKB_F32 = 0, TKB_BF16 = 1, TKB_F16 = 2 } tkb_dtype;

typedef enum {
    TKB_OK = 0,
    TKB_ERR_ARG = -1,         /* invalid shape, dtype, pointer or alignment */
    TKB_ERR_CUDA = -2,        /* a CUDA runtime call failed */
    TKB_ERR_UNSUPPORTED = -3, /* shape/dtype combination not implemented */
    TKB_ERR_WORKSPACE = -4    /* workspace missing or too small */
} tkb_status;

/* Library version string. */
const char *tkb_version(void);
/* Message describing the last failing call made from this host thread. */
const char *tkb_last_error(void);
/* Synchronizes `stream`, reads and clears the device error word (0 = none).
 * Bit 0: a bounded wait inside a kernel timed out; bit 1: bad launch. */
int tkb_device_error(unsigned int *code, void *stream);
/* Number of kernels this library launched since load (all entry points). */
unsigned long long tkb_launch_count(void);
/* Self-test of the failure path (no counterpart in the reference): one
 * kernel waits, for at most limit_ns (<= 2 s), on an mbarrier that nothing
 * arrives on, gives up like a pipeline kernel whose partner stopped, and
 * records bit 0 in the device error word (read it with tkb_device_error). */
int tkb_selftest_wait_timeout(unsigned long long limit_ns, void *stream);

/* ------------------------------------------------------------ attention
 * Packed layout of the reference (src/tkm_gpu.cu:331-338, 366-368):
 *   qkv  [B][S][(Hq + 2*Hkv)*D]  Q head h at column h*D, K head g at
 *        (Hq+g)*D, V head g at (Hq+Hkv+g)*D; query head h reads kv head
 *        h / (Hq/Hkv).
 *   out  [B][S][Hq*D]
 *   lse  [B*Hq][S] fp32, natural log of the softmax denominator.
 * D must be 64 or 128; Hq % Hkv == 0.  Causal masks key > query.
 * bf16/f16 run on tcgen05 tensor cores (fp32 accumulation); f32 runs fp32 FMA. */

/* Replaces k_gqa_flash_attn_tc_fwd<HEAD_DIM> (src/tkm_gpu.cu:302-438),
 * launched at src/tkm_gpu.cu:1252-1265. */
int tkb_gqa_attn_fwd(const void *qkv, void *out, float *lse,
                     int B, int S, int Hq, int Hkv, int D, float scale, int causal,
                     int dtype, void *stream);

/* Workspace bytes tkb_gqa_attn_bwd needs (per-row Delta and LSE*log2(e), fp32). */
size_t tkb_gqa_attn_bwd_workspace(int B, int S, int Hq, int D, int dtype);

/* Workspace bytes with which tkb_gqa_attn_bwd keeps every dS tile (16-bit,
 * B * Hq * tiles * 32 KB; causal stores only the lower triangle of tiles)
 * and computes dQ as a GEMM over them instead of recomputing S, P and dP.
 * Equal to tkb_gqa_attn_bwd_workspace when that area would exceed 32 GiB.
 * Any size between the two selects the recompute path. */
size_t tkb_gqa_attn_bwd_workspace_ex(int B, int S, int Hq, int D, int causal, int dtype);

/* Replaces k_gqa_flash_attn_tc_bwd<HEAD_DIM> (src/tkm_gpu.cu:440-598),
 * launched at src/tkm_gpu.cu:1389-1403.  Writes all of dqkv (dQ, dK, dV
 * slices; the reference leaves dK/dV wrong, src/tkm_gpu.cu:588-596).
 * dK/dV are summed over the query heads that share a kv head. */
int tkb_gqa_attn_bwd(const void *qkv, const void *out, const void *dout, const float *lse,
                     void *dqkv, void *workspace, size_t workspace_bytes,
                     int B, int S, int Hq, int Hkv, int D, float scale, int causal,
                     int dtype, void *stream);

/* ------------------------------------------------------------ residual + RMSNorm
 * Replaces the residual Add plasma group and the RMSNorm plasma group
 * emitted by src/tkm_codegen.c:484-523 (specs src/tkm_registry.c:228-245,
 * 435-439).  s = x + r (r may be NULL; s may be NULL when r is NULL),
 * istd[row] = 1/sqrt(mean(s^2) + eps), y = s * istd * gamma.  C even. */
int tkb_add_rmsnorm_fwd(const void *x, const void *r, void *s, void *y,
                        const float *gamma, float *istd, int rows, int C, float eps,
                        int dtype, void *stream);

size_t tkb_add_rmsnorm_bwd_workspace(int rows, int C);

/* Backward (src/tkm_codegen.c:525-624 for an RMSNorm group; spec
 * src/tkm_registry.c:239-245): dx = istd*(g*dy - xh*mean(g*dy*xh)) + ds_skip
 * with xh = s*istd (ds_skip may be NULL); dgamma += sum_rows(dy*xh)
 * (dgamma may be NULL). */
int tkb_add_rmsnorm_bwd(const void *dy, const void *s, const float *gamma, const float *istd,
                        const void *ds_skip, void *dx, float *dgamma,
                        void *workspace, size_t workspace_bytes,
                        int rows, int C, int dtype, void *stream);

/* ------------------------------------------------------------ SwiGLU twin epilogue
 * Replaces the twin-branch plasma group (src/tkm_codegen.c:511-518 fwd,
 * 540-598 bwd; rule src/tkm_registry.c:653-686).  gu [rows][2F] holds the
 * fused gate|up GEMM output; h = silu(g + bg) * (u + bu) [rows][F].
 * bg/bu may be NULL (zero). */
int tkb_swiglu_fwd(const void *gu, const float *bg, const float *bu, void *h,
                   int rows, int F, int dtype, void *stream);

size_t tkb_swiglu_bwd_workspace(int rows, int F);

/* dgu [rows][2F] overwritten; dbg/dbu accumulated (may be NULL). */
int tkb_swiglu_bwd(const void *dh, const void *gu, const float *bg, const float *bu,
                   void *dgu, float *dbg, float *dbu, void *workspace, size_t workspace_bytes,
                   int rows, int F, int dtype, void *stream);

/* ------------------------------------------------------------ QKV prep
 * Replaces the QKV-prep plasma group (src/tkm_codegen.c:211-295, rotation
 * 43-70; rule src/tkm_registry.c:688-770).  Row layout as the packed qkv
 * above; position = row % S.  Bias add on every column; QKNorm (per-head
 * RMS over D, eps 1e-5, gain qk_gain[(Hq+Hkv)*D]) and RoPE on the Q and K
 * heads.  RoPE rotates pair i of a head by pos * theta^(-i/D), with the
 * reference's frequency adjustment when rope_scale > 1.
 * save_istd [rows][Hq+Hkv] (needed with QKNorm). */
int tkb_qkv_prep_fwd(const void *in, const float *bias, const float *qk_gain, void *out,
                     float *save_istd, int rows, int S, int Hq, int Hkv, int D,
                     int has_qknorm, int has_rope, float theta, float rope_scale,
                     float low_freq_factor, float high_freq_factor,
                     float original_context_length, int dtype, void *stream);

size_t tkb_qkv_prep_bwd_workspace(int rows, int Hq, int Hkv, int D);

/* din accumulated (+=), dbias and dgain accumulated (may be NULL). */
int tkb_qkv_prep_bwd(const void *dout, const void *in, const float *bias, const float *qk_gain,
                     const float *save_istd, void *din, float *dbias, float *dgain,
                     void *workspace, size_t workspace_bytes,
                     int rows, int S, int Hq, int Hkv, int D,
                     int has_qknorm, int has_rope, float theta, float rope_scale,
                     float low_freq_factor, float high_freq_factor,
                     float original_context_length, int dtype, void *stream);

/* ------------------------------------------------------------ softmax, losses
 * Replaces k_softmax_fwd_h / k_softmax_bwd_h (src/tkm_gpu.cu:600-630,
 * launches 1270-1274 and 1409-1412).  dx is accumulated (+=). */
int tkb_softmax_fwd(const void *x, void *p, int rows, int C, int dtype, void *stream);
int tkb_softmax_bwd(const void *p, const void *dp, void *dx, int rows, int C, int dtype, void *stream);

size_t tkb_softmax_loss_workspace(int rows);

/* Replaces k_softmax_loss_fwd_bwd_h (src/tkm_gpu.cu:632-682, launch
 * 1275-1284).  kind 0 cross-entropy, 1 focal(gamma), 2 Brier.  labels: one
 * int32 per row (the reference reads uint8 labels[r], src/tkm_gpu.cu:646).
 * loss += mean over rows (summed in a fixed order); dlogits = dloss/dlogits
 * (may be NULL); correct += number of rows whose argmax equals the label
 * (may be NULL).  C <= 32768.  logits and dlogits 16-byte aligned when
 * C % 8 == 0 (else aligned to two elements); TKB_ERR_ARG otherwise. */
int tkb_softmax_loss(const void *logits, const int32_t *labels, void *dlogits,
                     float *loss, int *correct, void *workspace, size_t workspace_bytes,
                     int rows, int C, int kind, float gamma, int dtype, void *stream);

/* Variant of tkb_softmax_loss for callers that cannot allocate device memory
 * (no counterpart in the reference).  Code running while a CUDA graph is being
 * captured in global mode cannot call cudaMalloc, and foreign-language callers
 * may hold only raw device pointers from another framework's allocator; this
 * entry point needs no workspace.  Its per-row scratch is a fixed array inside
 * the library (1 MiB per GPU, held until exit), so rows must be at most
 * 262144; larger calls return TKB_ERR_ARG.  The first call on a device looks up
 * the array's address for that device: make it before any stream capture.
 * All calls share the array; calls that overlap on the GPU race on it.
 * Alignment as for tkb_softmax_loss. */
int tkb_softmax_loss_noalloc(const void *logits, const int32_t *labels, void *dlogits,
                             float *loss, int *correct, int rows, int C, int kind, float gamma,
                             int dtype, void *stream);

/* ------------------------------------------------------------ SGD
 * Replaces k_tkm_multi_tensor_sgd (src/tkm_gpu.cu:684-720, launch
 * 1417-1420).  `table` is device memory holding n_tensors tkb_sgd_tensor
 * records.  g += wd*p when apply_wd, v = momentum*v + g,
 * p -= lr*(momentum*v + g), lowp (if set) refreshed, *seed += 0x9E3779B9. */
typedef struct {
    float *master;
    float *vel;
    const float *grad;
    void *lowp;          /* 16-bit copy of master, or NULL */
    long long n;
    int apply_wd;
    int lowp_dtype;      /* TKB_BF16 or TKB_F16 */
} tkb_sgd_tensor;

int tkb_sgd_step(const tkb_sgd_tensor *table, int n_tensors, const float *lr,
                 float momentum, float weight_decay, uint32_t *seed, void *stream);

/* ------------------------------------------------------------ GEMM
 * Replaces the cuBLAS GEMMs of the FC layers (cublasGemmEx at
 * src/tkm_gpu.cu:1207-1236 forward, 1330-1372 input and weight gradients):
 * C[M][N] = A B (+ C when accumulate, + bias[n] when bias is not NULL),
 * bf16 operands, fp32 accumulation on the tcgen05 tensor cores.
 *   a_trans 0: A stored [M][K], lda elements per row; 1: A stored [K][M].
 *   b_trans 0: B stored [K][N], ldb elements per row; 1: B stored [N][K].
 *   c_dtype TKB_BF16 or TKB_F32 (C row-major, ldc elements per row).
 * Forward X W: (X, 0, W, 0); input gradient dY W^T: (dY, 0, W, 1); weight
 * gradient X^T dY: (X, 1, dY, 0).  lda and ldb must be multiples of 8, ldc
 * of 8 (bf16) or 4 (fp32); pointers 16-byte aligned.  bias needs a_trans 0.
 * An fp32 C whose tiles would leave the GPU's last wave mostly idle (weight
 * gradients: few output tiles, long K) splits K into partial sums kept in
 * `workspace` and added in a fixed order (deterministic); give it
 * tkb_gemm_workspace(M, N, K, c_dtype) bytes, or NULL to run unsplit. */
size_t tkb_gemm_workspace(int M, int N, int K, int c_dtype);
int tkb_gemm(const void *A, long long lda, int a_trans, const void *B, long long ldb, int b_trans,
             void *C, long long ldc, int c_dtype, int accumulate, const float *bias,
             int M, int N, int K, void *workspace, size_t workspace_bytes, void *stream);

/* The twin [gate | up] FC with its SwiGLU epilogue in one kernel (replaces
 * the cuBLAS GEMM of FC_TWIN_FUSED, src/tkm_gpu.cu:1207-1236, and the twin
 * epilogue group emitted at src/tkm_codegen.c:511-598): with [G | U] = A B,
 * A stored [M][K], B stored [K][2F] (gate columns 0..F-1, up F..2F-1),
 * GU[M][2F] receives [G | U] in bf16 (what the backward replays from) and
 * H[M][F] = SiLU(G + bias_gate) * (U + bias_up), computed from the bf16 G
 * and U.  F must be a multiple of 8; the biases may be NULL. */
int tkb_gemm_swiglu(const void *A, long long lda, const void *B, long long ldb, int F,
                    const float *bias_gate, const float *bias_up, void *GU, long long ldgu,
                    void *H, long long ldh, int M, int K, void *stream);

/* The LM head and its softmax cross-entropy without the logits in memory
 * (replaces the cuBLAS head GEMM, the Bias group and k_softmax_loss_fwd_bwd_h
 * with kind 0, src/tkm_gpu.cu:632-682 and 1275-1284): logits = X W + bias for
 * X [rows][d] (ldx per row), W [d][V] (ldw per row), bias [V] (may be NULL),
 * computed tile by tile on the tcgen05 CTA-pair GEMM.  A first pass keeps
 * per-row statistics (tile maxima, sums of exponentials, argmax, the label's
 * logit); *loss += mean over rows of -ln(max(p_label, 1e-7)); *correct (may
 * be NULL) += rows whose first argmax is the label; when dlogits is not
 * NULL a second pass recomputes each tile and writes d logits = (softmax -
 * onehot) / rows in bf16 ([rows][ldd]).  Every logit is recomputed instead of
 * stored: the [rows][V] logits buffer is never written.  Workspace:
 * tkb_lmhead_ce_workspace(rows, V) bytes, 256-byte aligned.  d and V must be
 * multiples of 8. */
size_t tkb_lmhead_ce_workspace(int rows, int V);
int tkb_lmhead_ce(const void *X, long long ldx, const void *W, long long ldw, const float *bias,
                  const int32_t *labels, void *dlogits, long long ldd, float *loss, int *correct,
                  void *workspace, size_t workspace_bytes, int rows, int d, int V, void *stream);

#ifdef __cplusplus
}
#endif
#endif
