// tkb_all.cu -- single translation unit of libtkm_b200.so.  The kernels share
// the device error word and inline helpers, so they are compiled together.
#include "attn_aux.cu"
#include "attn_fwd.cu"
#include "attn_bwd.cu"
#include "attn_f32.cu"
#include "gemm.cu"
#include "rows.cu"
#include "capi.cu"
#include "capi_rows.cu"
#include "capi_gemm.cu"
#include "noalloc.cu"
