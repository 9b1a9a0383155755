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

int num_sms() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

// K splits for an fp32 C on CTA pairs: the count that minimises the waves of
// pair tiles per split (a small charge per extra split for the reduction),
// with at least 8 K blocks of 64 per split.  Only shapes whose tiles leave
// a late wave mostly idle (few, large-K tiles: weight gradients) split.
int choose_splits(int M, int N, int K) {
  const long long tiles = static_cast<long long>((M + 255) / 256) * ((N + 255) / 256);
  const long long clusters = num_sms() / 2;
  const int nk = (K + 63) / 64;
  int best = 1;
  double best_cost = static_cast<double>((tiles + clusters - 1) / clusters);
  for (int s = 2; s <= 8 && nk / s >= 8; ++s) {
    const double cost = static_cast<double>((tiles * s + clusters - 1) / clusters) / s + 0.02 * (s - 1);
    if (cost < 0.97 * best_cost) {
      best = s;
      best_cost = cost;
    }
  }
  return best;
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

size_t tkb_gemm_workspace(int M, int N, int K, int c_dtype) {
  if (M <= 0 || N <= 0 || K <= 0 || c_dtype != TKB_F32 || !use_pairs()) return 0;
  const int s = choose_splits(M, N, K);
  return s > 1 ? static_cast<size_t>(s) * M * N * sizeof(float) : 0;
}

int tkb_gemm(const void* A, long long lda, int a_trans, const void* B, long long ldb, int b_trans, void* C,
             long long ldc, int c_dtype, int accumulate, const float* bias, int M, int N, int K, void* workspace,
             size_t workspace_bytes, void* stream) {
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
  const int nk = (K + 63) / 64;
  p.splits = 1;
  p.kb_per_split = nk;
  const int epi = bias ? 1 : 0;
  if (bias && a_mn) return fail(TKB_ERR_UNSUPPORTED, "tkb_gemm: bias with A stored [K][M]");
  if (pair && c_dtype == TKB_F32 && !bias) {
    const int s = choose_splits(M, N, K);
    const size_t need = static_cast<size_t>(s) * M * N * sizeof(float);
    if (s > 1 && workspace && workspace_bytes >= need && aligned16(workspace)) {
      p.kb_per_split = (nk + s - 1) / s;
      p.splits = (nk + p.kb_per_split - 1) / p.kb_per_split;
      p.ws = static_cast<float*>(workspace);
    }
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (!pair) return cuda_status(tkb::gemm_tc(p, a_mn, b_mn, epi, st), "tkb_gemm", 1);
  cudaError_t e = tkb::gemm_pair_tc(p, a_mn, b_mn, epi, st);
  if (e == cudaSuccess && p.splits > 1) e = tkb::gemm_splitk_reduce(p, st);
  return cuda_status(e, "tkb_gemm", p.splits > 1 ? 2 : 1);
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
  p.splits = 1;
  p.kb_per_split = (K + 63) / 64;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return cuda_status(pair ? tkb::gemm_pair_tc(p, false, true, 2, st) : tkb::gemm_tc(p, false, true, 2, st),
                     "tkb_gemm_swiglu", 1);
}

}  // extern "C"

namespace {
// Workspace of tkb_lmhead_ce: tile partials, label logits, LSE and per-row losses.
struct CeWs {
  float4* part;
  float *lab, *lse, *row_loss;
  size_t bytes;
};
CeWs ce_layout(void* base, int rows, int V) {
  const size_t tiles_n = (static_cast<size_t>(V) + 255) / 256;
  CeWs w{};
  char* b = static_cast<char*>(base);
  size_t off = 0;
  w.part = reinterpret_cast<float4*>(b + off);
  off += round256(static_cast<size_t>(rows) * tiles_n * sizeof(float4));
  w.lab = reinterpret_cast<float*>(b + off);
  off += round256(static_cast<size_t>(rows) * sizeof(float));
  w.lse = reinterpret_cast<float*>(b + off);
  off += round256(static_cast<size_t>(rows) * sizeof(float));
  w.row_loss = reinterpret_cast<float*>(b + off);
  off += round256(static_cast<size_t>(rows) * sizeof(float));
  w.bytes = off;
  return w;
}
}  // namespace

namespace tkb {
cudaError_t sum_rows(const float* row_loss, int rows, float* loss, cudaStream_t st);
}

extern "C" {

size_t tkb_lmhead_ce_workspace(int rows, int V) {
  if (rows <= 0 || V <= 0) return 0;
  return ce_layout(nullptr, rows, V).bytes;
}

int tkb_lmhead_ce(const void* X, long long ldx, const void* W, long long ldw, const float* bias,
                  const int32_t* labels, void* dlogits, long long ldd, float* loss, int* correct, void* workspace,
                  size_t workspace_bytes, int rows, int d, int V, void* stream) {
  if (rows <= 0 || d <= 0 || V <= 0) return fail(TKB_ERR_ARG, "tkb_lmhead_ce: rows, d, V must be positive");
  if (!labels || !loss) return fail(TKB_ERR_ARG, "tkb_lmhead_ce: labels and loss are required");
  if (!use_pairs()) return fail(TKB_ERR_UNSUPPORTED, "tkb_lmhead_ce: needs the CTA-pair GEMM (TKB_GEMM_PAIR=0 set)");
  const CeWs need = ce_layout(nullptr, rows, V);
  if (!workspace || workspace_bytes < need.bytes || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return fail(TKB_ERR_WORKSPACE, "tkb_lmhead_ce: workspace of %zu bytes (256-byte aligned) required", need.bytes);
  if (dlogits && (!aligned16(dlogits) || ldd < V || ldd % 8))
    return fail(TKB_ERR_ARG, "tkb_lmhead_ce: dlogits 16-byte aligned with ldd >= V, a multiple of 8");
  tkb::GemmParams p{};
  int rc = gemm_operand_map(&p.tmA, X, ldx, false, rows, d, 128, "X");
  if (rc) return rc;
  rc = gemm_operand_map(&p.tmB, W, ldw, true, V, d, 128, "W");
  if (rc) return rc;
  const CeWs w = ce_layout(workspace, rows, V);
  p.bias = bias;
  p.M = rows;
  p.N = V;
  p.K = d;
  p.tiles_m = (rows + 255) / 256;
  p.tiles_n = (V + 255) / 256;
  p.splits = 1;
  p.kb_per_split = (d + 63) / 64;
  p.labels = labels;
  p.ce_part = w.part;
  p.ce_lab = w.lab;
  p.ce_lse = w.lse;
  p.ce_scale = 1.0f / static_cast<float>(rows);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = tkb::gemm_pair_tc(p, false, true, 3, st);
  if (e == cudaSuccess)
    e = tkb::ce_combine(w.part, p.tiles_n, w.lab, labels, w.lse, w.row_loss, correct, rows, p.ce_scale, st);
  if (e == cudaSuccess) e = tkb::sum_rows(w.row_loss, rows, loss, st);
  unsigned kernels = 3;
  if (e == cudaSuccess && dlogits) {
    p.c = dlogits;
    p.ldc = ldd;
    e = tkb::gemm_pair_tc(p, false, true, 4, st);
    kernels = 4;
  }
  return cuda_status(e, "tkb_lmhead_ce", kernels);
}

}  // extern "C"
