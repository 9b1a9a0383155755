// capi.cu -- extern "C" entry points declared in include/tkm_b200.h.
// Argument checking, workspace carving, tensor-map construction and launch.
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>

#include "tkb_common.cuh"
#include "tkb_internal.h"
#include "../../include/tkm_b200.h"

namespace tkb {
cudaError_t attn_f32_fwd(const float*, float*, float*, int, int, int, int, int, float, int, cudaStream_t);
cudaError_t attn_f32_bwd(const float*, const float*, const float*, const float*, float*, int, int, int, int, int,
                         float, int, cudaStream_t);
cudaError_t attn_bwd_pre(const void*, const void*, const float*, float*, float*, long long, long long, int, int, int,
                         int, int, bool, cudaStream_t);
}  // namespace tkb

namespace {

thread_local char g_err[512] = "";
std::atomic<unsigned long long> g_launches{0};

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_status(cudaError_t e, const char* what, unsigned kernels) {
  if (e != cudaSuccess) return fail(TKB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  g_launches += kernels;
  return TKB_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
size_t round256(size_t x) { return (x + 255) & ~size_t(255); }
bool dtype_ok(int dt) { return dt == TKB_F32 || dt == TKB_BF16 || dt == TKB_F16; }

int check_attn(int B, int S, int Hq, int Hkv, int D, int dtype) {
  if (B <= 0 || S <= 0 || Hq <= 0 || Hkv <= 0) return fail(TKB_ERR_ARG, "attention: B, S, Hq, Hkv must be positive");
  if (Hq % Hkv) return fail(TKB_ERR_ARG, "attention: Hq (%d) must be a multiple of Hkv (%d)", Hq, Hkv);
  if (D != 64 && D != 128) return fail(TKB_ERR_UNSUPPORTED, "attention: head dim %d not in {64, 128}", D);
  if (!dtype_ok(dtype)) return fail(TKB_ERR_ARG, "attention: bad dtype %d", dtype);
  return TKB_OK;
}

}  // namespace

using namespace tkb;

extern "C" {

const char* tkb_version(void) { return "tokamak_b200 0.1 (sm_100a)"; }
const char* tkb_last_error(void) { return g_err; }
unsigned long long tkb_launch_count(void) { return g_launches.load(); }

int tkb_device_error(unsigned int* code, void* stream) {
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(TKB_ERR_CUDA, "tkb_device_error: %s", cudaGetErrorString(e));
  unsigned int v = 0, zero = 0;
  e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero));
  if (e != cudaSuccess) return fail(TKB_ERR_CUDA, "tkb_device_error: %s", cudaGetErrorString(e));
  if (code) *code = v;
  return TKB_OK;
}

// ------------------------------------------------------------------ self-test
}  // extern "C"

namespace tkb {
// Waits, with a limit of limit_ns, on an mbarrier that nothing arrives on:
// the bounded-wait path every pipeline kernel takes when a partner role
// stops, run on purpose.  The wait ends by itself and records the code.
__global__ void wait_timeout_selftest_kernel(unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait_limit(&bar, 0, &abort_flag, limit_ns);
  __syncthreads();
}
}  // namespace tkb

extern "C" {

int tkb_selftest_wait_timeout(unsigned long long limit_ns, void* stream) {
  if (limit_ns == 0 || limit_ns > 2000000000ull)
    return fail(TKB_ERR_ARG, "tkb_selftest_wait_timeout: limit must be in (0, 2 s]");
  tkb::wait_timeout_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit_ns);
  return cuda_status(cudaGetLastError(), "tkb_selftest_wait_timeout", 1);
}

// ------------------------------------------------------------------ attention
int tkb_gqa_attn_fwd(const void* qkv, void* out, float* lse, int B, int S, int Hq, int Hkv, int D, float scale,
                     int causal, int dtype, void* stream) {
  int rc = check_attn(B, S, Hq, Hkv, D, dtype);
  if (rc) return rc;
  if (!qkv || !out || !lse) return fail(TKB_ERR_ARG, "tkb_gqa_attn_fwd: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == TKB_F32)
    return cuda_status(attn_f32_fwd(static_cast<const float*>(qkv), static_cast<float*>(out), lse, B, S, Hq, Hkv, D,
                                    scale, causal, st),
                       "tkb_gqa_attn_fwd(f32)", 1);
  if (!aligned16(qkv) || !aligned16(out)) return fail(TKB_ERR_ARG, "tkb_gqa_attn_fwd: pointers must be 16-byte aligned");
  const bool bf16 = dtype == TKB_BF16;
  const long long ld = static_cast<long long>(Hq + 2 * Hkv) * D;
  FwdParams p;
  memset(&p, 0, sizeof(p));
  const uint16_t* base = static_cast<const uint16_t*>(qkv);
  cudaError_t e = make_tmap_rows(&p.tmQ, base, bf16, static_cast<long long>(Hq) * D, S, B, ld, ld * S);
  if (e == cudaSuccess)
    e = make_tmap_rows(&p.tmK, base + static_cast<long long>(Hq) * D, bf16, static_cast<long long>(Hkv) * D, S, B, ld,
                       ld * S);
  if (e == cudaSuccess)
    e = make_tmap_rows(&p.tmV, base + static_cast<long long>(Hq + Hkv) * D, bf16, static_cast<long long>(Hkv) * D, S,
                       B, ld, ld * S);
  if (e != cudaSuccess) return cuda_status(e, "tkb_gqa_attn_fwd: tensor map", 0);
  p.out = out;
  p.lse = lse;
  p.out_row_stride = static_cast<long long>(Hq) * D;
  p.out_batch_stride = p.out_row_stride * S;
  p.B = B;
  p.S = S;
  p.Hq = Hq;
  p.Hkv = Hkv;
  const int nq = (S + 127) / 128;
  p.n_pairs = (nq + 1) / 2;
  p.causal = causal ? 1 : 0;
  p.scale_log2 = scale * 1.4426950408889634f;
  return cuda_status(attn_fwd_tc(p, D, bf16, st), "tkb_gqa_attn_fwd", 1);
}

size_t tkb_gqa_attn_bwd_workspace(int B, int S, int Hq, int D, int dtype) {
  if (dtype == TKB_F32 || B <= 0 || S <= 0 || Hq <= 0 || D <= 0) return 0;
  const size_t spad = static_cast<size_t>((S + 127) / 128) * 128;
  const size_t rows = static_cast<size_t>(B) * Hq * spad;
  return 2 * round256(rows * 4);
}

}  // extern "C"

namespace {
// dS tiles (128 x 128, 16-bit) one (batch, q head) needs: the lower triangle
// of query x key tiles when causal, else all of them.
long long ds_tiles_per_head(int S, int causal) {
  const long long nq = (S + 127) / 128;
  return causal ? nq * (nq + 1) / 2 : nq * nq;
}
// Largest dS area tkb_gqa_attn_bwd_workspace_ex offers (beyond it dQ is
// recomputed instead of read back).  32 GiB of the 180 GB covers the
// long-context shape S=16384 with 64 query heads (17.3 GB; backward 14.6 ->
// 12.8 ms against the recompute path); S=32768 (69 GB) recomputes.
constexpr size_t kMaxDsBytes = size_t(32) << 30;
}  // namespace

extern "C" {

size_t tkb_gqa_attn_bwd_workspace_ex(int B, int S, int Hq, int D, int causal, int dtype) {
  const size_t base = tkb_gqa_attn_bwd_workspace(B, S, Hq, D, dtype);
  if (!base) return 0;
  const size_t ds = static_cast<size_t>(B) * Hq * ds_tiles_per_head(S, causal) * 128 * 128 * 2;
  return ds <= kMaxDsBytes ? base + ds : base;
}

int tkb_gqa_attn_bwd(const void* qkv, const void* out, const void* dout, const float* lse, void* dqkv,
                     void* workspace, size_t workspace_bytes, int B, int S, int Hq, int Hkv, int D, float scale,
                     int causal, int dtype, void* stream) {
  int rc = check_attn(B, S, Hq, Hkv, D, dtype);
  if (rc) return rc;
  if (!qkv || !out || !dout || !lse || !dqkv) return fail(TKB_ERR_ARG, "tkb_gqa_attn_bwd: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == TKB_F32)
    return cuda_status(attn_f32_bwd(static_cast<const float*>(qkv), static_cast<const float*>(out),
                                    static_cast<const float*>(dout), lse, static_cast<float*>(dqkv), B, S, Hq, Hkv, D,
                                    scale, causal, st),
                       "tkb_gqa_attn_bwd(f32)", 2);
  const size_t need = tkb_gqa_attn_bwd_workspace(B, S, Hq, D, dtype);
  if (!workspace || workspace_bytes < need)
    return fail(TKB_ERR_WORKSPACE, "tkb_gqa_attn_bwd: workspace of %zu bytes required", need);
  if (!aligned16(qkv) || !aligned16(out) || !aligned16(dout) || !aligned16(dqkv) || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return fail(TKB_ERR_ARG, "tkb_gqa_attn_bwd: pointers must be 16-byte aligned (workspace 256-byte)");
  const bool bf16 = dtype == TKB_BF16;
  const int S_pad = (S + 127) / 128 * 128;
  const size_t rows = static_cast<size_t>(B) * Hq * S_pad;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  float* nlse2 = reinterpret_cast<float*>(ws);
  float* delta = reinterpret_cast<float*>(ws + round256(rows * 4));
  const long long ld = static_cast<long long>(Hq + 2 * Hkv) * D, ldo = static_cast<long long>(Hq) * D;

  cudaError_t e = attn_bwd_pre(out, dout, lse, nlse2, delta, ldo, ldo * S, B, S, S_pad, Hq, D, bf16, st);
  if (e != cudaSuccess) return cuda_status(e, "tkb_gqa_attn_bwd: preprocess", 0);

  BwdParams p;
  memset(&p, 0, sizeof(p));
  const uint16_t* base = static_cast<const uint16_t*>(qkv);
  e = make_tmap_rows(&p.tmQ, base, bf16, static_cast<long long>(Hq) * D, S, B, ld, ld * S);
  if (e == cudaSuccess)
    e = make_tmap_rows(&p.tmK, base + static_cast<long long>(Hq) * D, bf16, static_cast<long long>(Hkv) * D, S, B, ld,
                       ld * S);
  if (e == cudaSuccess)
    e = make_tmap_rows(&p.tmV, base + static_cast<long long>(Hq + Hkv) * D, bf16, static_cast<long long>(Hkv) * D, S,
                       B, ld, ld * S);
  if (e == cudaSuccess) e = make_tmap_rows(&p.tmdO, dout, bf16, ldo, S, B, ldo, ldo * S);
  if (e != cudaSuccess) return cuda_status(e, "tkb_gqa_attn_bwd: tensor map", 0);
  p.nlse2 = nlse2;
  p.delta = delta;
  uint16_t* dbase = static_cast<uint16_t*>(dqkv);
  p.dq = dbase;
  p.dk = dbase + static_cast<long long>(Hq) * D;
  p.dv = dbase + static_cast<long long>(Hq + Hkv) * D;
  p.dkv_row_stride = ld;
  p.dkv_batch_stride = ld * S;
  p.B = B;
  p.S = S;
  p.S_pad = S_pad;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.causal = causal ? 1 : 0;
  p.scale = scale;
  p.scale_log2 = scale * 1.4426950408889634f;
  // dS path: the workspace holds every dS tile after LSE and Delta
  const size_t ex = tkb_gqa_attn_bwd_workspace_ex(B, S, Hq, D, causal, dtype);
  if (ex > need && workspace_bytes >= ex) {
    p.ds = reinterpret_cast<uint16_t*>(ws + need);
    p.ds_tiles = ds_tiles_per_head(S, causal);
  }
  e = attn_bwd_tc(p, D, bf16, st);
  return cuda_status(e, "tkb_gqa_attn_bwd: dK/dV and dQ kernels", 3);
}

}  // extern "C"
