/*
 * comfy-quant-bench B200 hot path: C ABI of libcq_b200.so.
 *
 * The quantized-linear path that comfy-quant-bench's formats execute inside ComfyUI, rebuilt for sm_100a:
 *   1. activation rotation (block Hadamard, groups 256/64/16) fused with dynamic quantization (+ SwiGLU);
 *   2. packed-int4-weight x int8/int4-activation GEMM on tcgen05 kind::i8 tensor cores (TMEM accumulators);
 *   3. fused dequant epilogue back to bf16 (per-group affine weight scale/zero, per-token activation scale,
 *      bias);
 * plus the converter's weight rotate-and-quantize step as a kernel.
 *
 * Conventions
 *   - All tensor arguments are raw DEVICE pointers to contiguous row-major arrays owned by the caller;
 *     sizes are element counts.  bf16 data is passed as `const void*` / `void*` (2 bytes per element).
 *   - Packed int4 stores two codes per byte, the low nibble holding the even column (the layout of
 *     comfy-kitchen's int4 tensors and of tools/_formats.py in comfy-quant-bench).
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  Calls are asynchronous: they enqueue
 *     kernels and return.  Nothing here allocates device memory except where noted.
 *   - Return value: CQ_OK (0) or a cq_status code.  Argument errors are detected on the host before any
 *     launch.  Device-side failures (a bounded wait that ran out) are recorded in a device status word read
 *     by cq_take_device_status().
 */
#ifndef CQ_B200_H
#define CQ_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define CQ_API __attribute__((visibility("default")))
#else
#define CQ_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  CQ_OK = 0,
  CQ_ERR_ARG = 1,          /* null pointer, bad enum value */
  CQ_ERR_SHAPE = 2,        /* size / divisibility constraint violated */
  CQ_ERR_ALIGN = 3,        /* pointer not 16-byte aligned where TMA or vector access needs it */
  CQ_ERR_CUDA = 4,         /* a CUDA runtime / driver call failed */
  CQ_ERR_TIMEOUT = 5,      /* device: a bounded wait ran out (recorded in the device status word) */
  CQ_ERR_UNSUPPORTED = 6,  /* device is not sm_100 */
  CQ_ERR_CAPACITY = 7      /* problem larger than a fixed internal limit */
} cq_status;

/* Activation quantization modes (cq_rotquant). */
typedef enum {
  CQ_ACT_INT8_ROW = 0,   /* per token, symmetric int8 (int8_linear / W4A8): scale = max(absmax/127, 1e-10)   */
  CQ_ACT_INT4_ROW = 1,   /* per token, symmetric int4 (ConvRot W4A4):        scale = max(absmax/7, 1e-10)     */
  CQ_ACT_INT4_GROUP = 2  /* per (token, act_group) int4, scale rounded UP to bf16; scales laid out [K/G, M_pad] */
} cq_act_mode;

/* Weight quantization modes (cq_weight_rotquant). */
typedef enum {
  CQ_W_INT4_ROW = 0,          /* ConvRot W4A4: s[n] = max(amax/7, 1e-12), signed int4 packed [N, K/2]        */
  CQ_W_INT8_ROW = 1,          /* int8_tensorwise: s[n] = max(amax/127, 1e-12), int8 [N, K]                   */
  CQ_W_AFFINE_INT4_GROUP = 2, /* awq layout: W = (q - 8) * s + z, q uint4 packed [N, K/2], s/z bf16 [K/G, N]    */
  CQ_W_INT4_GROUP_BF16UP = 3  /* per-group symmetric int4, s = bf16_up(amax/7) f32 [K/G, N]                    */
} cq_weight_mode;

/* cq_rotquant output flags. */
#define CQ_Q_INT8_CODES 1  /* int4 modes: write int8 codes [M_pad, K] instead of packed nibbles            */
#define CQ_Q_KPERM 2       /* int8 code outputs: store each 8-column block of K in the order 0,2,4,6,1,3,5,7 -
                              the order the int4-weight GEMMs unpack nibbles into (see cq_gemm_rowcol)    */

/* Weight operand encodings accepted by the GEMMs. */
typedef enum {
  CQ_B_INT4_SIGNED = 0,  /* packed signed int4 [N, K/2] (ConvRot W4A4)             */
  CQ_B_INT8 = 1          /* int8 [N, K] (int8_tensorwise, decoded W4A8)           */
} cq_b_format;

/* Kernel forms of the packed-int4-weight GEMMs (cq_gemm_affine, cq_gemm_rowcol with CQ_B_INT4_SIGNED, the fused
 * linears and the SwiGLU-output GEMM). */
typedef enum {
  CQ_GEMM_AUTO = 0,    /* by shape: the CTA-pair kernel when M >= 1024 and there are at least 74 tiles of 256 x 256 */
  CQ_GEMM_ONE_SM = 1,  /* one CTA per 128-weight-row x 256-token tile (tcgen05 cta_group::1)                        */
  CQ_GEMM_PAIR = 2     /* a cluster of two CTAs per 256 x 256 tile (tcgen05 cta_group::2), half the activation
                          operand's shared-memory traffic per SM and a deeper load ring                              */
} cq_gemm_variant;

/* Library version string, e.g. "cq_b200 0.1.0 sm_100a". */
CQ_API const char* cq_version(void);
/* Human-readable name of a cq_status code. */
CQ_API const char* cq_status_string(int status);

/* Select the GEMM kernel form for every later call in this process (cq_gemm_variant; the default is CQ_GEMM_AUTO).
 * Both forms compute the same integer sums and the same epilogue, so results agree to the last bit.  A tuning and
 * testing switch with no counterpart in the reference; it is process-wide and not synchronized with calls running
 * on other host threads.  Returns CQ_OK or CQ_ERR_ARG. */
CQ_API int cq_set_gemm_variant(int variant);

/* Copy the device status word of the current device into status[0..1] (code, site) and clear it.
 * Synchronizes `stream`.  Returns CQ_OK or CQ_ERR_CUDA. */
CQ_API int cq_take_device_status(int* status, void* stream);

/* Self-test of the failure path (no reference counterpart): enqueues one small kernel whose two waits, on
 * mbarriers nothing arrives on, give up after the library's wait limit (2 s), record CQ_ERR_TIMEOUT with site 90 or
 * 91 in the device status word and return.  The context stays usable; read the status with cq_take_device_status().
 * Returns CQ_OK, CQ_ERR_CUDA, or CQ_ERR_UNSUPPORTED on a device that is not sm_100. */
CQ_API int cq_selftest_bounded_wait(void* stream);

/*
 * Activation rotation + dynamic quantization.
 * Replaces comfy-kitchen's quantize_int4_rowwise_convrot64(x, 256) (called at
 * experiments/qwen21-kernel/kernels/g64_quant_test.py:105-112, experiments/qwen21-kernel/node/__init__.py:148),
 * the fused swiglu_quantize_int4_rowwise_convrot64(h) (tools/ck_swiglu/swiglu_quant.cu:111-137), the per-group
 * quant(x, group, swiglu, pad) (experiments/qwen21-kernel/kernels/g64_quant.cu:113-130) and the int8 activation
 * quantization inside w4a8_int8_linear / int8_linear (tools/_native_probe.py:201-255).
 *
 *   x          bf16 [M, K], or [M, 2K] = [gate | up] when swiglu != 0 (the product silu(gate)*up is quantized)
 *   rot_group  0 (no rotation), 16, 64 or 256; every group divides K, which the constraints below make a
 *              multiple of 256 (with swiglu, x holds 2K columns and the rotation runs over the K product columns)
 *   mode       cq_act_mode
 *   act_group  64 or 128 for CQ_ACT_INT4_GROUP, else ignored
 *   M_pad      >= M; rows M..M_pad-1 of q (and of scale for CQ_ACT_INT4_GROUP) are written as 0
 *   flags      CQ_Q_INT8_CODES | CQ_Q_KPERM (see above), 0 for the reference's layouts
 *   q          int8 [M_pad, K] for CQ_ACT_INT8_ROW; packed int4 [M_pad, K/2] for the int4 modes,
 *              or int8 codes [M_pad, K] with CQ_Q_INT8_CODES (what the fused linears feed the GEMM)
 *   scale      f32 [M_pad] for the per-token modes, f32 [K/act_group, M_pad] for CQ_ACT_INT4_GROUP
 *   group_sums NULL, or bf16 [M_pad, cq_group_sum_cols(K)]: the sum R of each token's codes over each
 *              128-wide K group g (G = K/128 groups), split exactly into hi = 128*floor(R/128) in column g
 *              and lo = R - hi in column G + g, remaining columns 0 (the affine zero-point operand of
 *              cq_gemm_affine)
 * Constraints: K % 512 == 0 or K % 256 == 0 (multiple of 256), K <= 32768; M >= 0.
 */
CQ_API int cq_rotquant(const void* x, int64_t M, int64_t K, int rot_group, int swiglu, int mode, int act_group,
                       int64_t M_pad, int flags, void* q, float* scale, void* group_sums, void* stream);

/* Columns of cq_rotquant's split group-sum array (and of the prepared zero-point operand of
 * cq_prepare_affine_zeros) for a given K: 64 * ceil(K / 4096). */
CQ_API int64_t cq_group_sum_cols(int64_t K);

/*
 * Prepare the zero-point operand of the affine W4A8 GEMM from the awq-layout zeros, once per weight:
 *   zt[n, j] = z[j mod G, n] for j < 2G, 0 for 2G <= j < cq_group_sum_cols(K)   (G = K / group)
 *   z   bf16 [K/group, N] (patches/comfyui_awq_w4a16_format.patch:79-80 layout);  zt bf16 [N, cq_group_sum_cols(K)]
 */
CQ_API int cq_prepare_affine_zeros(const void* z_bf16, int64_t N, int64_t K, int group, void* zt_bf16, void* stream);

/*
 * Weight rotate-and-quantize (the converter kernel).
 * Replaces comfy-kitchen's quantize_convrot_w4a4_weight(w, convrot_groupsize, quant_group_size=64, 0)
 * (tools/_formats.py:72-76; restated at experiments/qwen21-kernel/node/__init__.py:89-126),
 * quantize_int8_convrot_weight (tools/_formats.py:149-156) and produces the awq_w4a16 affine layout
 * (tools/_formats.py:191-212, patches/comfyui_awq_w4a16_format.patch:79-80) used by the W4A8 linear.
 *
 *   w        f32 [N, K] (w_is_bf16 == 0) or bf16 [N, K]
 *   q        packed int4 [N, K/2] (modes INT4_ROW, AFFINE, INT4_GROUP_BF16UP) or int8 [N, K] (INT8_ROW)
 *   scale    f32 [N] (INT4_ROW, INT8_ROW), bf16 [K/group, N] (AFFINE), f32 [K/group, N] (INT4_GROUP_BF16UP)
 *   zeros    bf16 [K/group, N] for AFFINE, else NULL
 */
CQ_API int cq_weight_rotquant(const void* w, int w_is_bf16, int64_t N, int64_t K, int rot_group, int mode, int group,
                       void* q, void* scale, void* zeros, void* stream);

/*
 * Unpack int4 codes to int8 codes: src packed [R, C/2] -> dst int8 [R, C] (signed nibbles).
 * Lets a caller holding comfy-kitchen-style packed int4 activations feed cq_gemm_rowcol.
 */
CQ_API int cq_unpack_int4(const void* src, int64_t R, int64_t C, void* dst, void* stream);

/*
 * out[m, n] = bf16( (sum_k a[m,k] * b[n,k]) * sa[m] * sb[n] + bias[n] )
 * Replaces comfy-kitchen's int4_linear(qact, qweight, x_scale, wscales, bias, out_dtype)
 * (experiments/qwen21-kernel/kernels/g64_bench6.py:109, patches/comfy_kitchen_swiglu_w4a4_fused.patch:37)
 * and the int8 GEMM of int8_linear (tools/_native_probe.py:234-255), and the reference's own scale policy 0
 * of g64_gemm6.gemm (experiments/qwen21-kernel/kernels/g64_gemm6.cu:383-411).
 *
 *   a      int8 codes [M, K] (int8, or int4 values held in int8)
 *   a_kperm 1 when `a` was written with CQ_Q_KPERM (int4 weights only; the unpack then needs no byte
 *          shuffles), 0 for natural K order
 *   sa     f32 [M]
 *   b      CQ_B_INT4_SIGNED: packed [N, K/2]; CQ_B_INT8: int8 [N, K]
 *   sb     f32 [N]
 *   bias   bf16 [N] or NULL
 *   out    bf16 [M, N]
 * Constraints: K % 128 == 0; N % 16 == 0; pointers 16-byte aligned.
 */
CQ_API int cq_gemm_rowcol(const int8_t* a, int a_kperm, const float* sa, const void* b, int b_format,
                          const float* sb, const void* bias, void* out, int64_t M, int64_t N, int64_t K,
                          void* stream);

/*
 * Per-group scales on both sides, the reference GEMM's policy 4
 * (experiments/qwen21-kernel/kernels/g64_gemm6.cu:5-7, 228-229, 383-411; called from
 * experiments/qwen21-kernel/node/__init__.py:152-187 after the per-group quantizer quant(x, 128, swiglu, pad)):
 *   out[m, n] = bf16( sum_g ( round(P_g[m,n] * sb_g[g,n]) * sa_g[g,m] ) + bias[n] ),  P_g = sum_{k in g} a[m,k]*b[n,k]
 * accumulated in fp32 over g = 0..K/128-1 in order, each step one fused multiply-add, as the reference's epilogue
 * acc = fma(fma(D, w, -M*w), a, acc) does.
 *   a       int4 activation values held as int8 codes [M, K] (cq_rotquant CQ_ACT_INT4_GROUP with CQ_Q_INT8_CODES;
 *           a_kperm as for cq_gemm_rowcol)
 *   sa_g    f32 [K/128, sa_ld] (the per-group quantizer's scale layout), sa_ld >= M, sa_ld % 4 == 0
 *   b       packed signed int4 [N, K/2] (cq_weight_rotquant CQ_W_INT4_GROUP_BF16UP);  sb_g f32 [K/128, N]
 *   bias    bf16 [N] or NULL;  out bf16 [M, N];  group 128
 * Runs the CTA-pair GEMM whatever cq_set_gemm_variant selected.
 */
CQ_API int cq_gemm_groupwise(const int8_t* a, int a_kperm, const float* sa_g, int64_t sa_ld, const void* b_packed,
                             const float* sb_g, const void* bias, void* out, int64_t M, int64_t N, int64_t K, int group,
                             void* stream);

/*
 * Integer weight ratios per group: the reference GEMM's policies 5, 7, 15 and 17
 * (experiments/qwen21-kernel/kernels/g64_gemm6.cu:8-11, 93-343; called as g64_gemm6.gemm(a, b, sa, sb, ca, cw, bias,
 * pol, cfg), g64_gemm6.cu:383-411):
 *   acc[m, n] = sum_g cw[g, n] * sum_{k in group g} a[m, k] * b[n, k]     (int32, exact)
 *   out[m, n] = bf16( float(acc) * sa[m] * sb[n] + bias[n] )
 *   a        int4 values held as int8 [M, K] (a_kperm as for cq_gemm_rowcol);  b_packed packed signed int4 [N, K/2]
 *   sa       f32 [M];  sb f32 [N] (the reference passes the row scale / 255)
 *   cw       [K/cw_group, N] int32 (policies 5, 7) or, with cw_u8 = 1, uint8 (15, 17); values in [1, 255]
 *   cw_group 64 (policies 5, 15) or 128 (7, 17)
 * K < 171840 (the reference's bound on the int32 accumulator).  Runs the CTA-pair GEMM.
 */
CQ_API int cq_gemm_intratio(const int8_t* a, int a_kperm, const float* sa, const void* b_packed, const float* sb,
                            const void* cw, int cw_u8, int cw_group, const void* bias, void* out, int64_t M, int64_t N,
                            int64_t K, void* stream);

/*
 * W4A8 affine linear, the headline GEMM:
 *   out[m, n] = bf16( sa[m] * sum_g ( s[g,n] * sum_{k in g} a[m,k]*(q[n,k]-8) + z[g,n] * gsum[g,m] ) + bias[n] )
 * with q the awq_w4a16 uint4 codes (packed [N, K/2]), s bf16 [K/group, N] and the zeros z passed as zt, the
 * operand cq_prepare_affine_zeros builds from z bf16 [K/group, N]
 * (patches/comfyui_awq_w4a16_format.patch:79-80; the int8 x int4 policy family of
 * experiments/qwen21-kernel/kernels/g64_gemm6.cu:5-11, 93-343).
 *   a       int8 [M, K] (a_kperm as for cq_gemm_rowcol);  sa f32 [M];
 *   gsplit  bf16 [M, cq_group_sum_cols(K)]: the split group sums of `a` written by cq_rotquant
 *   group   128
 * The zero-point term sum_g z[g,n] * gsum[g,m] runs on the tensor core (bf16 x bf16 -> fp32, exact products)
 * and seeds the fp32 accumulator that the per-group int32 partial sums are scaled into.
 * M <= 8 with a_kperm = 1 runs a CUDA-core product instead (one warp per four weight rows, dp4a, the weights read
 * once; gsplit unused).  Its fp32 summation order differs from the tensor-core path's, so for the same inputs
 * the two agree to fp32 rounding (an output may differ by one bf16 step), not bit for bit.  This applies to every
 * W4A8 affine entry point below except the column-parallel (_peers) forms, which always use the GEMM.
 */
CQ_API int cq_gemm_affine(const int8_t* a, int a_kperm, const float* sa, const void* gsplit, const void* b_packed,
                          const void* s_bf16, const void* zt_bf16, const void* bias, void* out, int64_t M, int64_t N,
                          int64_t K, int group, void* stream);

/*
 * The elementwise step that follows a DiT block's linear, applied by the W4A8 affine GEMM (and the row/col GEMM of
 * cq_linear_convrot_w4a4_op / cq_linear_w8a8_op) to its bf16 result before the store.  y = the bf16 output the plain
 * GEMM writes for the same inputs; then
 *   CQ_OUT_PLAIN            out = y
 *   CQ_OUT_GELU_TANH        out = bf16(gelu_tanh(y)),  gelu_tanh(y) = y / (1 + exp(-2 sqrt(2/pi) (y + 0.044715 y^3)))
 *                           (torch F.gelu(y, approximate="tanh"), the MLP-up activation; the sigmoid form of
 *                           0.5 y (1 + tanh(u)), within a few fp32 ulp of torch's value before the bf16 rounding)
 *   CQ_OUT_GATED_RESIDUAL   out = bf16(residual + gate[n] * y)  (torch.addcmul(residual, gate, y), the gated residual
 *                           after the attention-output and MLP-down linears; one bf16 fused multiply-add, which
 *                           rounds the exact value once: torch's fp32-then-bf16 rounding can differ from it only
 *                           where the fp32 value is a bf16 rounding tie, about one output in 2^16, by one step)
 * residual: bf16 [M, residual_ld] (residual_ld >= N); it may be the output buffer itself (same pointer, same row
 * stride: each element is read before it is overwritten) but must not overlap it otherwise.  gate: bf16 [N].
 * The operations other than CQ_OUT_PLAIN need N % 8 == 0 and a 16-byte aligned output.
 * No counterpart in the reference, whose model code runs these as torch ops on the linear's output.
 */
typedef enum {
  CQ_OUT_PLAIN = 0,
  CQ_OUT_GELU_TANH = 1,
  CQ_OUT_GATED_RESIDUAL = 2
} cq_out_kind;

typedef struct {
  int kind;                /* cq_out_kind */
  const void* residual;    /* CQ_OUT_GATED_RESIDUAL: bf16 [M, residual_ld], 2-byte aligned */
  int64_t residual_ld;     /*   row stride in elements */
  const void* gate;        /*   bf16 [N] */
} cq_out_op;

/* cq_gemm_affine followed by the output operation `op` (NULL: CQ_OUT_PLAIN). */
CQ_API int cq_gemm_affine_op(const int8_t* a, int a_kperm, const float* sa, const void* gsplit, const void* b_packed,
                             const void* s_bf16, const void* zt_bf16, const void* bias, const cq_out_op* op, void* out,
                             int64_t M, int64_t N, int64_t K, int group, void* stream);

/*
 * Fused linears (activation stage + GEMM) with caller-provided scratch.  `workspace` must hold at least
 * cq_linear_workspace_bytes(M, K) bytes of device memory (16-byte aligned).
 *
 * cq_linear_convrot_w4a4: comfy-kitchen convrot_w4a4_linear(x, qweight, wscales, bias, convrot_groupsize,
 *   quant_group_size=64, linear_dtype, input_act) (signature: patches/comfy_kitchen_swiglu_w4a4_fused.patch:41-50,
 *   compile_support.py:84-113).  act_bits 4 or 8 (linear_dtype "int4" / "int8"); swiglu: x is [M, 2K].
 * cq_linear_w4a8_affine: the affine W4A8 linear (rotation optional, per-token int8 activations); the zeros are
 *   passed prepared (zt from cq_prepare_affine_zeros, computed once per weight).
 * cq_linear_w8a8: comfy-kitchen int8_linear(x, weight, weight_scale, bias, out_dtype, convrot, convrot_groupsize,
 *   input_act) (tools/_native_probe.py:234-255).
 */
CQ_API int64_t cq_linear_workspace_bytes(int64_t M, int64_t K);
/* The workspace for the W4A8 affine linears (cq_linear_w4a8_affine, _lnmod, cq_linear_w4a8_op) of an N-output
 * linear, with room for the K-split partial sums the GEMM uses when its tiles leave most SMs idle (few tokens, e.g.
 * a DiT's 256-token text stream): fp32 [S, M, N] after the cq_linear_workspace_bytes(M, K) bytes, S <= 8 chosen by
 * shape.  Given at least this much, those linears split K over more CTAs and add the S partial sums in a fixed
 * order (deterministic) in a second kernel; given only cq_linear_workspace_bytes(M, K), they run unsplit.  The two
 * results agree to fp32 rounding, not bit for bit. */
CQ_API int64_t cq_linear_workspace_bytes_n(int64_t M, int64_t K, int64_t N);
CQ_API int cq_linear_convrot_w4a4(const void* x, int64_t M, int64_t K, int64_t N, int rot_group, int swiglu, int act_bits,
                           const void* qweight, const float* wscale, const void* bias, void* out, void* workspace,
                           int64_t workspace_bytes, void* stream);
CQ_API int cq_linear_w4a8_affine(const void* x, int64_t M, int64_t K, int64_t N, int rot_group, int swiglu,
                                 const void* qweight, const void* s_bf16, const void* zt_bf16, int group,
                                 const void* bias, void* out, void* workspace, int64_t workspace_bytes, void* stream);
CQ_API int cq_linear_w8a8(const void* x, int64_t M, int64_t K, int64_t N, int rot_group, int swiglu, const int8_t* weight,
                   const float* wscale, const void* bias, void* out, void* workspace, int64_t workspace_bytes,
                   void* stream);
/*
 * cq_linear_convrot_w4a4_op / cq_linear_w8a8_op: the same linears (no SwiGLU input) with the output operation `op`
 * (cq_out_op, NULL: CQ_OUT_PLAIN) applied in the row/col GEMM's epilogue to its bf16 result, and, when shift is not
 * NULL, the activation stage quantizing the modulated layer norm
 *   xn = bf16( shift + bf16( (x - mean) * rsqrt(var + eps) ) * bf16(1 + mod_scale) )
 * per token over its K columns (shift, mod_scale bf16 [K], 16-byte aligned; K % 256 == 0, K <= 24576) instead of
 * x: a Wan-style DiT block's norm + modulation before its QKV and MLP-up linears, its GELU after MLP-up and its
 * gated residuals after the attention-output and MLP-down linears.  The operations need N % 8 == 0 and a 16-byte
 * aligned output.  No counterpart in the reference, whose model code runs these as torch ops.
 */
CQ_API int cq_linear_convrot_w4a4_op(const void* x, int64_t M, int64_t K, int64_t N, int rot_group, int act_bits,
                                     const void* shift, const void* mod_scale, float eps, const void* qweight,
                                     const float* wscale, const void* bias, const cq_out_op* op, void* out,
                                     void* workspace, int64_t workspace_bytes, void* stream);
CQ_API int cq_linear_w8a8_op(const void* x, int64_t M, int64_t K, int64_t N, int rot_group, const void* shift,
                             const void* mod_scale, float eps, const int8_t* weight, const float* wscale,
                             const void* bias, const cq_out_op* op, void* out, void* workspace,
                             int64_t workspace_bytes, void* stream);

/*
 * W4A4 row/col GEMM / ConvRot W4A4 linear with the SwiGLU output fused into the epilogue
 * (silu(y[:, :N/2]) * y[:, N/2:] of the N-column linear y):
 *   out[m, j] = bf16( bf16(silu(y[m, j])) * y[m, N/2 + j] ),  y = bf16(linear output),  out bf16 [M, N/2]
 * (torch's silu and mul on the bf16 linear output).  The weight rows, scales and bias are passed interleaved in
 * groups of 32: row p of b_glu / sb / bias is original row (p / 32) * 16 + p % 32 for p % 32 < 16 (gate) and
 * N/2 + (p / 32) * 16 + p % 32 - 16 otherwise (up); ops.prepare_swiglu_output_weight builds them once.
 * N % 128 == 0.  a: int4 values held as int8 codes with CQ_Q_KPERM; b: packed signed int4.  No counterpart in the
 * reference, which applies the activation to the linear's output afterwards.
 */
CQ_API int cq_gemm_rowcol_swiglu(const int8_t* a, const float* sa, const void* b_glu, const float* sb,
                                 const void* bias, void* out, int64_t M, int64_t N, int64_t K, void* stream);
CQ_API int cq_linear_convrot_w4a4_swiglu(const void* x, int64_t M, int64_t K, int64_t N, int rot_group, int act_bits,
                                         const void* qweight_glu, const float* wscale_glu, const void* bias_glu,
                                         void* out, void* workspace, int64_t workspace_bytes, void* stream);

/*
 * Column-parallel forms of cq_gemm_affine / cq_linear_w4a8_affine: the launch computes N output columns (one rank's
 * shard of a layer with ldo = N_total outputs) and writes them, as they are produced, into each of the n_outs
 * (1..8) output buffers outs[i] (bf16 [M, ldo], 16-byte aligned) at columns [col0, col0 + N).  Passing every
 * rank's output buffer (peer pointers mapped into this process, e.g. symmetric memory) assembles the gathered
 * [M, ldo] output over NVLink inside the GEMM, with no separate all-gather; the caller still synchronizes the ranks
 * before reading it.  Requires N % 32 == 0, col0 % 8 == 0, ldo % 8 == 0, col0 + N <= ldo.  No counterpart in the
 * reference, which runs one GPU: these replace its per-layer output with a sharded layer plus an all-gather.
 */
CQ_API int cq_gemm_affine_peers(const int8_t* a, int a_kperm, const float* sa, const void* gsplit, const void* b_packed,
                                const void* s_bf16, const void* zt_bf16, const void* bias, void* const* outs,
                                int n_outs, int64_t col0, int64_t ldo, int64_t M, int64_t N, int64_t K, int group,
                                void* stream);
CQ_API int cq_linear_w4a8_affine_peers(const void* x, int64_t M, int64_t K, int64_t N, int rot_group, int swiglu,
                                       const void* qweight, const void* s_bf16, const void* zt_bf16, int group,
                                       const void* bias, void* const* outs, int n_outs, int64_t col0, int64_t ldo,
                                       void* workspace, int64_t workspace_bytes, void* stream);

/*
 * cq_linear_w4a8_affine without a workspace argument: for callers that cannot allocate device memory where
 * they run the linear (a frozen or defragmenting memory pool, allocator hooks that must not re-enter the
 * allocator, plugins handed only input and output buffers).  No counterpart in the reference.
 * The scratch (activation codes, scales, split group sums) is a fixed 32 MiB device array inside this library,
 * held by every GPU that loads it until the process exits; problems needing more than that
 * (cq_linear_workspace_bytes(M, K) > 32 MiB, e.g. M = 8192 at K = 3072 fits, M = 16384 does not) return
 * CQ_ERR_CAPACITY.  All calls share the array: calls that overlap on the GPU race, so serialize them on one
 * stream.  The first call on each device looks up the array's device address, and so does the first call after
 * the device's context was reset (cudaDeviceReset); make those calls before any stream capture.  It calls no
 * cudaMalloc / cudaFree, and its GEMM never splits K (its results equal cq_linear_w4a8_affine's given the
 * cq_linear_workspace_bytes(M, K) workspace).
 */
CQ_API int cq_linear_w4a8_affine_noalloc(const void* x, int64_t M, int64_t K, int64_t N, int rot_group, int swiglu,
                                         const void* qweight, const void* s_bf16, const void* zt_bf16, int group,
                                         const void* bias, void* out, void* stream);

/*
 * DiT-step glue around the quantized linears of a dual-stream MMDiT block (SD3 / Flux / Qwen-Image layout).
 * No counterpart in the reference, whose model code runs these steps as torch ops on bf16 tensors
 * (layer_norm, addcmul, rms_norm, the rotary multiply and the copies into the attention layout).
 *
 * cq_rotquant_lnmod: cq_rotquant (per-token int8, CQ_ACT_INT8_ROW) of the modulated layer norm
 *   xn = bf16( shift + bf16( (x - mean) * rsqrt(var + eps) ) * scale1p )
 * per token over its K columns (biased variance, no affine), shift and scale1p bf16 [K] (scale1p = 1 + scale,
 * rounded to bf16 by the caller), computed in fp32 with the two bf16 roundings of the torch ops it replaces.
 * Writes the same outputs as cq_rotquant (flags: CQ_Q_KPERM only).  K % 256 == 0, K <= 24576.
 * cq_linear_w4a8_affine_lnmod: cq_linear_w4a8_affine of that xn.
 *
 * cq_qkv_rmsnorm_rope: y bf16 [S, 3, H, D] (one stream's QKV linear output, q | k | v) ->
 *   q[h, s0+s, :] = rope(bf16(rmsnorm(y[s,0,h,:]) * q_norm)),  k likewise with k_norm,  v[h, s0+s, :] = y[s,2,h,:]
 * with q, k, v bf16 [H, s_all, D] (the joint attention layout, batch 1), rmsnorm(x) = x * rsqrt(mean(x^2) + eps)
 * in fp32, and rope rotating the interleaved pairs (x[2p], x[2p+1]) by rope[s, p] = (cos, sin) (f32 [S, D/2, 2]),
 * in fp32, rounded to bf16.  D = 64 or 128.
 * cq_qkv_rmsnorm_rope_layout: the same with token_major = 1 writing q, k, v as bf16 [s_all, H, D] (the [tokens,
 *   hidden] layout: an attention kernel given these as strided [1, H, s_all, D] views writes its output in the same
 *   token-major layout, which the output projection reads as it is); token_major = 0 is cq_qkv_rmsnorm_rope.
 */
CQ_API int cq_rotquant_lnmod(const void* x, int64_t M, int64_t K, int rot_group, const void* shift,
                             const void* scale1p, float eps, int64_t M_pad, int flags, void* q, float* scale,
                             void* group_sums, void* stream);
CQ_API int cq_linear_w4a8_affine_lnmod(const void* x, int64_t M, int64_t K, int64_t N, int rot_group,
                                       const void* shift, const void* scale1p, float eps, const void* qweight,
                                       const void* s_bf16, const void* zt_bf16, int group, const void* bias,
                                       void* out, void* workspace, int64_t workspace_bytes, void* stream);
/*
 * cq_linear_w4a8_op: one DiT-block linear with the glue on both sides fused into its two kernels:
 *   shift == NULL:  cq_linear_w4a8_affine of x (rotation rot_group, per-token int8)
 *   shift != NULL:  cq_linear_w4a8_affine_lnmod of x with scale1p = bf16(1 + mod_scale) formed inside the
 *                   activation kernel (mod_scale bf16 [K], the adaLN scale as the modulation linear produced it;
 *                   torch's `1 + scale` on a bf16 tensor), eps
 * followed by the output operation `op` in the GEMM's epilogue (cq_gemm_affine_op; NULL: CQ_OUT_PLAIN).
 */
CQ_API int cq_linear_w4a8_op(const void* x, int64_t M, int64_t K, int64_t N, int rot_group, const void* shift,
                             const void* mod_scale, float eps, const void* qweight, const void* s_bf16,
                             const void* zt_bf16, int group, const void* bias, const cq_out_op* op, void* out,
                             void* workspace, int64_t workspace_bytes, void* stream);
/*
 * Per-token int8 activations of a row-parallel linear, whose K columns are split over ranks: each rank holds
 * x bf16 [M, K] = its columns of the full rows, and the scale must be the one the whole row gives.
 * cq_rotquant_absmax: per token t, amax[t] = the NaN-ignoring maximum of |rotated x| over this rank's columns and
 *   amax[M_pad + t] = 1 if one of them is NaN, else 0 (f32 [2, M_pad]; padding tokens 0).
 * cq_rotquant_scaled: after the ranks combine their amax arrays elementwise by a maximum (an all-reduce MAX), the
 *   same outputs as cq_rotquant (CQ_ACT_INT8_ROW; flags: CQ_Q_KPERM only) with scale[t] =
 *   max(amax[t] / 127, 1e-10); a token whose combined flag or maximum is not finite takes the non-finite rule of
 *   cq_rotquant (NaN products give code 0).  The codes then equal, column for column, those cq_rotquant gives for
 *   the unsplit rows, and each rank's GEMM over its K slice yields a partial sum of the linear.
 * K % 256 == 0, K <= 24576, the rotation groups inside each rank's columns.  No counterpart in the reference (one
 * GPU).
 */
CQ_API int cq_rotquant_absmax(const void* x, int64_t M, int64_t K, int rot_group, int64_t M_pad, float* amax,
                              void* stream);
CQ_API int cq_rotquant_scaled(const void* x, int64_t M, int64_t K, int rot_group, const float* amax, int64_t M_pad,
                              int flags, void* q, float* scale, void* group_sums, void* stream);

/*
 * cq_heads_to_rows: attention output o bf16 [Hp, S, D] (head-major, batch 1) -> outs[i][s, col0 + h*D + d] for
 * every buffer outs[i] (bf16 [S, ldo], 16-byte aligned, 1..8 buffers).  With one local buffer it is the transpose
 * to the [tokens, hidden] layout of the output projection; with the peer buffers of a head-parallel attention it
 * gathers every rank's heads into every rank's rows.  D = 64 or 128, Hp * D <= 8192, col0 % 8 == 0, ldo % 8 == 0.
 */
CQ_API int cq_heads_to_rows(const void* o, int64_t S, int Hp, int D, void* const* outs, int n_outs, int64_t col0,
                            int64_t ldo, void* stream);
CQ_API int cq_qkv_rmsnorm_rope(const void* y, int64_t S, int H, int D, const void* q_norm, const void* k_norm,
                               float eps, const float* rope, void* q, void* k, void* v, int64_t s_all, int64_t s0,
                               void* stream);
/*
 * cq_rmsnorm_rope_rows: out[s, :] = rope(bf16(x[s, :] * rsqrt(mean(x[s, :]^2) + eps) * w)) for bf16 rows x [S, C]:
 * RMSNorm over the whole row (a Wan-style q/k norm over the hidden dim) in fp32, one bf16 rounding; then, when rope
 * is not null, each D-wide head's interleaved pairs (x[2p], x[2p+1]) rotated by rope[s, p] = (cos, sin) (f32
 * [S, D/2, 2]) in fp32 and rounded to bf16.  w bf16 [C].  out may be x.  C % 8 == 0, C <= 16384; with rope,
 * D = 64 or 128 and C % D == 0.  x, w, out 16-byte aligned.  No counterpart in the reference (its model code runs
 * rms_norm, a float copy, a complex multiply and a bf16 copy).
 */
CQ_API int cq_rmsnorm_rope_rows(const void* x, int64_t S, int C, const void* w, float eps, const float* rope, int D,
                                void* out, void* stream);
CQ_API int cq_qkv_rmsnorm_rope_layout(const void* y, int64_t S, int H, int D, const void* q_norm,
                                      const void* k_norm, float eps, const float* rope, void* q, void* k, void* v,
                                      int64_t s_all, int64_t s0, int token_major, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CQ_B200_H */
