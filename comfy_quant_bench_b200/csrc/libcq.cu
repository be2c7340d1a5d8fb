// Unity build of libcq_b200.so: one translation unit, so the device status word and every kernel live in the
// same module (no relocatable device code needed).
#include "rotquant.cu"
#include "gemm_sm100.cu"
#include "gemm_pair.cu"
#include "gemv.cu"
#include "dit.cu"
#include "selftest.cu"
#include "capi.cu"
#include "noalloc.cu"
