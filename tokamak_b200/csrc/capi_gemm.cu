// capi_gemm.cu -- extern "C" GEMM entry points of include/tkm_b200.h:
// argument checks, the two tensor maps and the launch of gemm.cu's kernel.
#include <cstdlib>

#include "tkb_common.cuh"
#include "tkb_internal.h"
#include "../../include/tkm_b200.h"

namespace tkb {
cudaError_t make_tmap_2d(CUtensorMap* m, const void* base, long long inner, long long outer, long long ld,
                         int box_inner, int box_outer);
}

namespace {

// CTA-pair kernels unless TKB_GEMM_PAIR=0 (read once per process).
bool use_pairs() {
  static const bool v = [] {
    const char* e = getenv("TKB_GEMM_PAIR");
    return !(e && e[0] == '0');
  }();
  return v;
}

// A K-major operand (K contiguous) is loaded as {64 K, rows} boxes; an
// MN-major one as {64 columns, 64 K} boxes.
int gemm_operand_map(CUtensorMap* m, const void* X, long long ld, bool mn_major, long long mn, long long k,
                     int rows_box, const char* what) {
  if (!X || !aligned16(X)) return fail(TKB_ERR_ARG, "tkb_gemm: %s must be non-null and 16-byte aligned", what);
  if (ld % 8) return fail(TKB_ERR_ARG, "tkb_gemm: leading dimension of %s (%lld) must be a multiple of 8", what, ld);
  if (ld < (mn_major ? mn : k)) return fail(TKB_ERR_ARG, "tkb_gemm: leading dimension of %s too small", what);
  cudaError_t e = mn_major ? tkb::make_tmap_2d(m, X, mn, k, ld, 64, 64) : tkb::make_tmap_2d(m, X, k, mn, ld, 64, rows_box);
  if (e != cudaSuccess) return fail(TKB_ERR_CUDA, "tkb_gemm: tensor map of %s: %s", what, cudaGetErrorString(e));
  return TKB_OK;
}

}  // namespace

extern "C" {

int tkb_gemm(const void* A, long long lda, int a_trans, const void* B, long long ldb, int b_trans, void* C,
             long long ldc, int c_dtype, int accumulate, const float* bias, int M, int N, int K, void* stream) {
  if (M <= 0 || N <= 0 || K <= 0) return fail(TKB_ERR_ARG, "tkb_gemm: M, N, K must be positive");
  if (c_dtype != TKB_BF16 && c_dtype != TKB_F32) return fail(TKB_ERR_ARG, "tkb_gemm: C must be bf16 or fp32");
  if (!C || !aligned16(C)) return fail(TKB_ERR_ARG, "tkb_gemm: C must be non-null and 16-byte aligned");
  if (ldc < N || ldc % (c_dtype == TKB_F32 ? 4 : 8))
    return fail(TKB_ERR_ARG, "tkb_gemm: ldc (%lld) must be >= N and a multiple of %d", ldc, c_dtype == TKB_F32 ? 4 : 8);
  tkb::GemmParams p{};
  const bool a_mn = a_trans != 0, b_mn = b_trans == 0;  // B stored [K][N] is N-contiguous
  const bool pair = use_pairs();
  int rc = gemm_operand_map(&p.tmA, A, lda, a_mn, M, K, 128, "A");
  if (rc) return rc;
  rc = gemm_operand_map(&p.tmB, B, ldb, b_mn, N, K, pair ? 128 : 256, "B");
  if (rc) return rc;
  p.c = C;
  p.ldc = ldc;
  p.bias = bias;
  p.M = M;
  p.N = N;
  p.K = K;
  p.tiles_m = pair ? (M + 255) / 256 : (M + 127) / 128;
  p.tiles_n = (N + 255) / 256;
  p.accumulate = accumulate != 0;
  p.out_f32 = c_dtype == TKB_F32;
  const int epi = bias ? 1 : 0;
  if (bias && a_mn) return fail(TKB_ERR_UNSUPPORTED, "tkb_gemm: bias with A stored [K][M]");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return cuda_status(pair ? tkb::gemm_pair_tc(p, a_mn, b_mn, epi, st) : tkb::gemm_tc(p, a_mn, b_mn, epi, st),
                     "tkb_gemm", 1);
}

int tkb_gemm_swiglu(const void* A, long long lda, const void* B, long long ldb, int F, const float* bias_gate,
                    const float* bias_up, void* GU, long long ldgu, void* H, long long ldh, int M, int K,
                    void* stream) {
  if (M <= 0 || F <= 0 || K <= 0) return fail(TKB_ERR_ARG, "tkb_gemm_swiglu: M, F, K must be positive");
  if (F % 8) return fail(TKB_ERR_ARG, "tkb_gemm_swiglu: F (%d) must be a multiple of 8", F);
  if (!GU || !H || !aligned16(GU) || !aligned16(H))
    return fail(TKB_ERR_ARG, "tkb_gemm_swiglu: GU and H must be non-null and 16-byte aligned");
  if (ldgu < 2LL * F || ldgu % 8 || ldh < F || ldh % 8)
    return fail(TKB_ERR_ARG, "tkb_gemm_swiglu: ldgu >= 2F, ldh >= F, both multiples of 8");
  tkb::GemmParams p{};
  int rc = gemm_operand_map(&p.tmA, A, lda, false, M, K, 128, "A");
  if (rc) return rc;
  rc = gemm_operand_map(&p.tmB, B, ldb, true, 2LL * F, K, 256, "B");
  if (rc) return rc;
  p.c = GU;
  p.ldc = ldgu;
  p.h = H;
  p.ldh = ldh;
  p.bias = bias_gate;
  p.bias2 = bias_up;
  p.M = M;
  p.N = F;
  p.K = K;
  const bool pair = use_pairs();
  p.tiles_m = pair ? (M + 255) / 256 : (M + 127) / 128;
  p.tiles_n = (F + 127) / 128;
  p.b_split = F;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return cuda_status(pair ? tkb::gemm_pair_tc(p, false, true, 2, st) : tkb::gemm_tc(p, false, true, 2, st),
                     "tkb_gemm_swiglu", 1);
}

}  // extern "C"
