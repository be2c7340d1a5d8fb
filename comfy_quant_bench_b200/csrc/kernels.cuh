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
  int kperm;            // int8 outputs: store each 8-column block in the order 0,2,4,6,1,3,5,7 (the K order
                        // the int4-weight GEMMs unpack their nibbles into)
  void* q;
  void* scale;          // f32 [rows_pad] | f32 [K/G, rows_pad] | bf16 [K/G, rows_pad] (affine)
  void* zeros;          // bf16 [K/G, rows_pad] (affine)
  __nv_bfloat16* rsplit;  // bf16 [rows_pad, rs_cols] or null: per-token code sums over 128-wide K groups, split
                          // exactly into hi = 128*floor(R/128) (columns [0, G)) and lo = R - hi (columns [G, 2G))
  int rs_cols;            // 64 * ceil(G / 32), G = K / 128; columns [2G, rs_cols) are zero
  // per-token int8 activations only: if ln_shift is set, the kernel quantizes the modulated layer norm
  // bf16(ln_shift + bf16((x - mean) * rsqrt(var + ln_eps)) * ln_scale1p) instead of x (bf16 [K] vectors)
  const __nv_bfloat16* ln_shift;
  const __nv_bfloat16* ln_scale1p;
  float ln_eps;
  int ln_scale_plus_one;  // ln_scale1p holds the modulation scale itself; the kernel forms bf16(1 + scale)
  // per-token int8 activations whose K columns are split over ranks (row-parallel linears).  amax_out set: the
  // kernel only writes, per token t, the NaN-ignoring maximum of |rotated x| over its columns (amax_out[t]) and
  // 1 if a NaN was among them, else 0 (amax_out[rows_pad + t]).  amax_in set (the same two rows, combined over the
  // ranks by a maximum): the kernel quantizes with those instead of its own maximum, so every rank derives the
  // scale the whole row would give.
  float* amax_out;
  const float* amax_in;
};

// columns of the split group-sum array for a K (the affine GEMM's zero-point operand)
__host__ __device__ constexpr int rsplit_cols(int K) { return 64 * ((K / 128 + 31) / 32); }

// DiT glue: per-head RMSNorm + rotary embedding of q and k, and the joint-attention layout of q, k, v
struct QkvRopeArgs {
  const __nv_bfloat16* y;     // [S, 3, H, D]: one stream's QKV linear output
  const __nv_bfloat16* qw;    // [D] RMSNorm weight of q
  const __nv_bfloat16* kw;    // [D] RMSNorm weight of k
  const float* rope;          // [S, D/2, 2]: (cos, sin) of each token's position
  __nv_bfloat16* q;           // [H, s_all, D] (head-major) or [s_all, H, D] (token-major)
  __nv_bfloat16* k;
  __nv_bfloat16* v;
  int64_t S, s_all, s0;       // tokens of this stream, tokens of the joint sequence, this stream's first token
  int H, D;
  float eps;
  int64_t tok_stride;         // elements between tokens: D (head-major) or H*D (token-major)
  int64_t head_stride;        // elements between heads: s_all*D (head-major) or D (token-major)
};
cudaError_t launch_qkv_rmsnorm_rope(const QkvRopeArgs& a, cudaStream_t st);

// DiT glue: head-major attention output -> [tokens, hidden] rows in up to kMaxOutBuffers buffers
struct HeadsToRowsArgs {
  const __nv_bfloat16* src;   // [Hp, S, D]
  __nv_bfloat16* outs[8];     // [S, ldo] each
  int n_out;
  int64_t S;
  int Hp, D;
  int64_t col0, ldo;
};
cudaError_t launch_heads_to_rows(const HeadsToRowsArgs& a, cudaStream_t st);

// DiT glue: RMSNorm over whole rows (a Wan-style q/k norm over the hidden dim), then optionally the rotary rotation of
// each D-wide head's interleaved pairs
struct RmsRopeArgs {
  const __nv_bfloat16* x;     // [S, C]
  const __nv_bfloat16* w;     // [C] norm weight
  const float* rope;          // [S, D/2, 2] (cos, sin) or null: no rotation
  __nv_bfloat16* out;         // [S, C]; may be x
  int64_t S;
  int C, D;
  float eps;
  int chunks;                 // 8-column chunks per thread
};
cudaError_t launch_rmsnorm_rope_rows(const RmsRopeArgs& a, cudaStream_t st);

cudaError_t launch_act_rotquant(int rot, bool swiglu, int mode, const RotQuantArgs& a, cudaStream_t st);
cudaError_t launch_weight_rotquant(int rot, bool w_bf16, int mode, const RotQuantArgs& a, cudaStream_t st);
cudaError_t launch_unpack_int4(const void* src, int64_t n_bytes, void* dst, cudaStream_t st);
// pdl: launch with programmatic stream serialization (the fused linears, whose previous kernel in the stream is
// their own activation kernel): the GEMM's prologue overlaps that kernel's tail
struct OutOp;
// op: an output operation (GELU-tanh, gated residual) in the epilogue, or null / OUT_PLAIN for the plain output
int launch_gemm_rowcol(const int8_t* a, int a_kperm, const float* sa, const void* b, int b_format, const float* sb,
                       const void* bias, void* out, int M, int N, int K, cudaStream_t st, bool pdl = false,
                       const OutOp* op = nullptr);
int launch_gemm_rowcol_glu(const int8_t* a, const float* sa, const void* b, const float* sb, const void* bias,
                           void* out, int M, int N, int K, cudaStream_t st, bool pdl = false);
constexpr int kMaxOutBuffers = 8;   // output buffers of one column-parallel affine launch

// outs != nullptr: write the result into n_outs (<= kMaxOutBuffers) buffers of [M, ldo] bf16 at columns [col0, col0 + N)
// instead of `out` (column-parallel layers)
// output operation of the affine epilogue (cq_out_op): kind 0 plain, 1 GELU-tanh, 2 gated residual
struct OutOp {
  int kind;
  const void* res;
  int64_t res_ld;
  const void* gate;
};
int launch_gemm_affine(const int8_t* a, int a_kperm, const float* sa, const void* rsplit, const void* b,
                       const void* s, const void* zt, const void* bias, void* out, int M, int N, int K,
                       cudaStream_t st, void* const* outs = nullptr, int n_outs = 0, int col0 = 0, int64_t ldo = 0,
                       const OutOp* op = nullptr, bool pdl = false, float* partial = nullptr);
// K splits the affine GEMM takes for a shape when given room for fp32 partial sums [S, M, N] (1: no split)
int affine_ksplit(int M, int N, int K);
cudaError_t launch_prep_zt(const void* z, int N, int K, void* zt, cudaStream_t st);
// per-group scales on both sides (policy 4): sag f32 [K/128, sag_ld], sbg f32 [K/128, N]; CTA-pair kernel
int launch_gemm_group(const int8_t* a, int a_kperm, const float* sag, int64_t sag_ld, const void* b, const float* sbg,
                      const void* bias, void* out, int M, int N, int K, cudaStream_t st);
// integer weight ratios per 64- or 128-wide group (policies 5/7/15/17): cw int32 or uint8 [K/cw_group, N]; CTA pair
int launch_gemm_intratio(const int8_t* a, int a_kperm, const float* sa, const void* b, const float* sb, const void* cw,
                         int cw_u8, int cw_group, const void* bias, void* out, int M, int N, int K, cudaStream_t st);
// process-wide kernel choice for the packed-int4-weight GEMMs (cq_gemm_variant values)
int set_gemm_variant(int variant);
// failure-path self-test: two waits on mbarriers nothing arrives on; sites kSelftestSite and kSelftestSite + 1
constexpr int kSelftestSite = 90;
cudaError_t launch_selftest_wait(cudaStream_t st);
// small-M W4A8 affine product (M <= 8, K-permuted activations): one warp per weight row, read once
bool gemv_affine_fits(int M, int a_kperm);
cudaError_t launch_gemv_affine(const int8_t* a, const float* sa, const void* b, const void* s, const void* zt,
                               const void* bias, void* out, int M, int N, int K, cudaStream_t st, bool pdl = false);

}  // namespace cq
