// noalloc.cu -- tkb_softmax_loss_noalloc: the fused softmax-loss kernel for
// callers that cannot allocate device memory.
//
// tkb_softmax_loss needs a caller-provided workspace of one float per row
// (the per-row losses it sums in a fixed order).  Some callers cannot get one:
// code that runs while a CUDA graph is being captured in global mode (the
// reference's training step is captured that way, and any cudaMalloc in the
// process fails during such a capture), and foreign-language callers that
// only hold raw device pointers handed over by another framework's allocator.
// This variant takes no workspace.  Its scratch is a fixed array in this
// library's device memory, so every GPU that loads the library holds it
// (kMaxRows floats = 1 MiB) until the process exits.
//
// Rules for callers:
//   * rows must not exceed kMaxRows; larger calls are rejected with TKB_ERR_ARG.
//   * The first call on a device looks up the array's device address for that
//     device (cudaGetSymbolAddress).  Make that first call before any stream
//     capture begins on that device; a first call made while its stream is
//     capturing is rejected with TKB_ERR_ARG and leaves the capture intact.
//   * The looked-up address is kept for the life of the process.  After
//     cudaDeviceReset on a device it is stale: do not call this entry point on
//     that device again in the same process.
//   * All calls share the one array.  Each call writes the per-row entries it
//     later reads, so nothing carries over between calls, but calls whose
//     kernels overlap on the GPU (different streams, or different host
//     threads on one device) race on the array and must be serialized.
#include <mutex>

namespace tkb {

constexpr int kNoallocMaxRows = 1 << 18;

// Per-row loss scratch for tkb_softmax_loss_noalloc (see the rules above).
static __device__ __align__(256) float g_noalloc_row_loss[kNoallocMaxRows];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kMaxDevices] = {nullptr};

// Device address of the scratch array on the current device (looked up once
// per device).  The lookup may load this library's module on the device,
// which must not happen inside a stream capture: if the first call on a
// device comes while `st` is capturing, *in_capture is set and nothing is
// looked up.
cudaError_t noalloc_scratch(float** out, cudaStream_t st, bool* in_capture) {
  *in_capture = false;
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
      *in_capture = true;
      return cudaSuccess;
    }
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_row_loss);
    if (e != cudaSuccess) return e;
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return cudaSuccess;
}
}  // namespace

}  // namespace tkb

extern "C" int tkb_softmax_loss_noalloc(const void* logits, const int32_t* labels, void* dlogits, float* loss,
                                        int* correct, int rows, int C, int kind, float gamma, int dtype,
                                        void* stream) {
  using namespace tkb;
  int rc = row_check("tkb_softmax_loss_noalloc", rows, C, dtype);
  if (rc) return rc;
  if (!logits) return fail(TKB_ERR_ARG, "tkb_softmax_loss_noalloc: null logits");
  if (kind < 0 || kind > 2) return fail(TKB_ERR_ARG, "tkb_softmax_loss_noalloc: kind %d not in {0,1,2}", kind);
  if (C > 256 * 8 * 16) return fail(TKB_ERR_UNSUPPORTED, "tkb_softmax_loss_noalloc: C > 32768");
  if (!loss_rows_aligned(logits, C, dtype) || !loss_rows_aligned(dlogits, C, dtype))
    return fail(TKB_ERR_ARG, "tkb_softmax_loss_noalloc: logits and dlogits must be 16-byte aligned when C %% 8 == 0 "
                "(else aligned to two elements)");
  if (rows > kNoallocMaxRows)
    return fail(TKB_ERR_ARG, "tkb_softmax_loss_noalloc: rows %d exceeds the built-in scratch limit of %d rows", rows,
                kNoallocMaxRows);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float* scratch = nullptr;
  bool in_capture = false;
  cudaError_t e = noalloc_scratch(&scratch, st, &in_capture);
  if (e != cudaSuccess) return cuda_status(e, "tkb_softmax_loss_noalloc: scratch address", 0);
  if (in_capture)
    return fail(TKB_ERR_ARG,
                "tkb_softmax_loss_noalloc: the first call on a device must come before any stream capture "
                "(it looks up the scratch array's device address)");
#define CALL(T) softmax_loss_t<T>(logits, labels, dlogits, loss, correct, scratch, rows, C, kind, gamma, st)
  return cuda_status(TKB_BY_DTYPE(dtype, CALL), "tkb_softmax_loss_noalloc", loss ? 2 : 1);
#undef CALL
}
