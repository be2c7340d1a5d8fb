// Declarations shared by the kernel files and the C ABI layer (one translation unit: libcq.cu).
#pragma once
#include "cq_common.cuh"

namespace cq {

struct RotQuantArgs {
  const void* x;        // bf16 [rows, K] (or [rows, 2K] with SwiGLU), or f32/bf16 [rows, K] for weights
  int64_t rows;         // M (or N for weights)
  int64_t rows_pad;     // >= rows; padding rows are written as zeros
  int K;
  int act_group;        // 64/128 for the per-group modes
  int int4_as_int8;     // int4 modes: write int8 codes [rows_pad, K] instead of packed nibbles
  void* q;
  void* scale;          // f32 [rows_pad] | f32 [K/G, rows_pad] | bf16 [K/G, rows_pad] (affine)
  void* zeros;          // bf16 [K/G, rows_pad] (affine)
  float* gsum;          // f32 [K/128, rows_pad] or null
};

cudaError_t launch_act_rotquant(int rot, bool swiglu, int mode, const RotQuantArgs& a, cudaStream_t st);
cudaError_t launch_weight_rotquant(int rot, bool w_bf16, int mode, const RotQuantArgs& a, cudaStream_t st);
cudaError_t launch_unpack_int4(const void* src, int64_t n_bytes, void* dst, cudaStream_t st);
int launch_gemm_rowcol(const int8_t* a, const float* sa, const void* b, int b_format, const float* sb,
                       const void* bias, void* out, int M, int N, int K, cudaStream_t st);
int launch_gemm_affine(const int8_t* a, const float* sa, const float* gsum, int64_t gsum_ld, const void* b,
                       const void* s, const void* z, const void* bias, void* out, int M, int N, int K,
                       cudaStream_t st);

}  // namespace cq
