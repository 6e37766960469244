// iw_lib.cu -- the whole library as one translation unit: every kernel file
// is included here so that device globals (the status word) have a single
// definition and cross-file device functions inline without -rdc.
#include "gemm_i8.cu"
#include "gemm_cm.cu"
#include "kernels.cu"
#include "attn_tc.cu"
#include "frontend.cu"
#include "capi.cu"
#include "noalloc.cu"
