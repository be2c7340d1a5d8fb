// extern "C" entry points of libcq_b200.so (declared in include/cq_b200.h): argument checks on the host,
// then kernel launches on the caller's stream.  No entry point here allocates device memory.
#include <cstdint>

#include "kernels.cuh"


namespace {

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

int check_device() {
  static int cached = -1;
  if (cached < 0) {
    int dev = 0, major = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return CQ_ERR_CUDA;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return CQ_ERR_CUDA;
    cached = (major == 10) ? CQ_OK : CQ_ERR_UNSUPPORTED;
  }
  return cached;
}

int cuda_status(cudaError_t e) { return e == cudaSuccess ? CQ_OK : CQ_ERR_CUDA; }

bool valid_rot(int r) { return r == 0 || r == 16 || r == 64 || r == 256; }

int64_t round_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

constexpr int64_t kMaxK = 32768;
constexpr int64_t kMaxLnModK = 24576;   // the two-token activation kernel: 16 warps x 3 chunks x 512 columns
constexpr int64_t kMaxRows = 0x7FFFFFFF;

}  // namespace

extern "C" {

const char* cq_version(void) { return "cq_b200 0.1.0 sm_100a"; }

const char* cq_status_string(int status) {
  switch (status) {
    case CQ_OK: return "ok";
    case CQ_ERR_ARG: return "invalid argument";
    case CQ_ERR_SHAPE: return "unsupported shape";
    case CQ_ERR_ALIGN: return "misaligned pointer";
    case CQ_ERR_CUDA: return "CUDA error";
    case CQ_ERR_TIMEOUT: return "device wait timed out";
    case CQ_ERR_UNSUPPORTED: return "device is not sm_100";
    case CQ_ERR_CAPACITY: return "problem exceeds a fixed internal limit";
    default: return "unknown status";
  }
}

int cq_take_device_status(int* status, void* stream) {
  if (status == nullptr) return CQ_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int host[2] = {0, 0};
  const int zero[2] = {0, 0};
  if (cudaMemcpyFromSymbolAsync(host, cq::g_device_status, sizeof(host), 0, cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return CQ_ERR_CUDA;
  if (cudaMemcpyToSymbolAsync(cq::g_device_status, zero, sizeof(zero), 0, cudaMemcpyHostToDevice, st) != cudaSuccess)
    return CQ_ERR_CUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return CQ_ERR_CUDA;
  status[0] = host[0];
  status[1] = host[1];
  return CQ_OK;
}

int cq_set_gemm_variant(int variant) { return cq::set_gemm_variant(variant); }

int cq_selftest_bounded_wait(void* stream) {
  if (int dv = check_device()) return dv;
  return cuda_status(cq::launch_selftest_wait(static_cast<cudaStream_t>(stream)));
}

int64_t cq_group_sum_cols(int64_t K) { return K > 0 ? 64 * ((K / 128 + 31) / 32) : 0; }

int cq_prepare_affine_zeros(const void* z_bf16, int64_t N, int64_t K, int group, void* zt_bf16, void* stream) {
  if (group != 128) return CQ_ERR_ARG;
  if (N < 0 || N > kMaxRows || K < 128 || K % 128 != 0 || K > kMaxK) return CQ_ERR_SHAPE;
  if (N == 0) return CQ_OK;
  if (z_bf16 == nullptr || zt_bf16 == nullptr) return CQ_ERR_ARG;
  if (!aligned(z_bf16, 2) || !aligned(zt_bf16, 16)) return CQ_ERR_ALIGN;
  if (int dv = check_device()) return dv;
  return cuda_status(cq::launch_prep_zt(z_bf16, static_cast<int>(N), static_cast<int>(K), zt_bf16,
                                        static_cast<cudaStream_t>(stream)));
}

int cq_rotquant(const void* x, int64_t M, int64_t K, int rot_group, int swiglu, int mode, int act_group,
                int64_t M_pad, int flags, void* q, float* scale, void* group_sums, void* stream) {
  if (M < 0 || M_pad < M || M_pad > kMaxRows) return CQ_ERR_SHAPE;
  if (K < 256 || K % 256 != 0 || K > kMaxK) return CQ_ERR_SHAPE;
  if (!valid_rot(rot_group)) return CQ_ERR_ARG;
  if (mode != CQ_ACT_INT8_ROW && mode != CQ_ACT_INT4_ROW && mode != CQ_ACT_INT4_GROUP) return CQ_ERR_ARG;
  if (mode == CQ_ACT_INT4_GROUP && act_group != 64 && act_group != 128) return CQ_ERR_ARG;
  if (flags & ~(CQ_Q_INT8_CODES | CQ_Q_KPERM)) return CQ_ERR_ARG;
  const int int8_codes = (mode == CQ_ACT_INT8_ROW) || (flags & CQ_Q_INT8_CODES);
  if ((flags & CQ_Q_KPERM) && !int8_codes) return CQ_ERR_ARG;
  if (M_pad == 0) return CQ_OK;
  if ((M > 0 && x == nullptr) || q == nullptr || scale == nullptr) return CQ_ERR_ARG;
  if (!aligned(x, 16) || !aligned(q, 16) || !aligned(scale, 4) || !aligned(group_sums, 16)) return CQ_ERR_ALIGN;
  if (int dv = check_device()) return dv;
  cq::RotQuantArgs a{x, M, M_pad, static_cast<int>(K), act_group, (flags & CQ_Q_INT8_CODES) ? 1 : 0,
                     (flags & CQ_Q_KPERM) ? 1 : 0, q, scale, nullptr,
                     static_cast<__nv_bfloat16*>(group_sums), cq::rsplit_cols(static_cast<int>(K))};
  return cuda_status(cq::launch_act_rotquant(rot_group, swiglu != 0, mode, a, static_cast<cudaStream_t>(stream)));
}

static int rotquant_lnmod(const void* x, int64_t M, int64_t K, int rot_group, const void* shift, const void* scale1p,
                          float eps, int64_t M_pad, int flags, void* q, float* scale, void* group_sums, void* stream,
                          bool scale_plus_one, int mode = CQ_ACT_INT8_ROW);

int cq_rotquant_lnmod(const void* x, int64_t M, int64_t K, int rot_group, const void* shift, const void* scale1p,
                      float eps, int64_t M_pad, int flags, void* q, float* scale, void* group_sums, void* stream) {
  return rotquant_lnmod(x, M, K, rot_group, shift, scale1p, eps, M_pad, flags, q, scale, group_sums, stream, false);
}

// scale_plus_one: `scale1p` holds the modulation scale; the kernel forms bf16(1 + scale) itself.  mode
// CQ_ACT_INT4_ROW: per-token int4 values held as int8 codes (the W4A4 GEMM's operand), no group sums.
static int rotquant_lnmod(const void* x, int64_t M, int64_t K, int rot_group, const void* shift, const void* scale1p,
                          float eps, int64_t M_pad, int flags, void* q, float* scale, void* group_sums, void* stream,
                          bool scale_plus_one, int mode) {
  if (M < 0 || M_pad < M || M_pad > kMaxRows) return CQ_ERR_SHAPE;
  if (K < 256 || K % 256 != 0 || K > kMaxLnModK) return CQ_ERR_SHAPE;
  if (!valid_rot(rot_group)) return CQ_ERR_ARG;
  if (flags & ~CQ_Q_KPERM) return CQ_ERR_ARG;
  if (!(eps >= 0.0f)) return CQ_ERR_ARG;
  if (M_pad == 0) return CQ_OK;
  if ((M > 0 && x == nullptr) || q == nullptr || scale == nullptr || shift == nullptr || scale1p == nullptr)
    return CQ_ERR_ARG;
  if (!aligned(x, 16) || !aligned(q, 16) || !aligned(scale, 4) || !aligned(group_sums, 16) || !aligned(shift, 16) ||
      !aligned(scale1p, 16))
    return CQ_ERR_ALIGN;
  if (int dv = check_device()) return dv;
  cq::RotQuantArgs a{x, M, M_pad, static_cast<int>(K), 0, mode == CQ_ACT_INT4_ROW ? 1 : 0,
                     (flags & CQ_Q_KPERM) ? 1 : 0, q, scale, nullptr,
                     static_cast<__nv_bfloat16*>(group_sums), cq::rsplit_cols(static_cast<int>(K)),
                     static_cast<const __nv_bfloat16*>(shift), static_cast<const __nv_bfloat16*>(scale1p), eps,
                     scale_plus_one ? 1 : 0};
  return cuda_status(cq::launch_act_rotquant(rot_group, false, mode, a, static_cast<cudaStream_t>(stream)));
}

// the two phases of per-token int8 activations for a row-parallel linear (K split over ranks)
static int check_sharded_act(const void* x, int64_t M, int64_t K, int rot_group, int64_t M_pad) {
  if (M < 0 || M_pad < M || M_pad > kMaxRows) return CQ_ERR_SHAPE;
  if (K < 256 || K % 256 != 0 || K > kMaxLnModK) return CQ_ERR_SHAPE;
  if (!valid_rot(rot_group)) return CQ_ERR_ARG;
  if (M > 0 && x == nullptr) return CQ_ERR_ARG;
  if (!aligned(x, 16)) return CQ_ERR_ALIGN;
  return CQ_OK;
}

int cq_rotquant_absmax(const void* x, int64_t M, int64_t K, int rot_group, int64_t M_pad, float* amax, void* stream) {
  if (int e = check_sharded_act(x, M, K, rot_group, M_pad)) return e;
  if (M_pad == 0) return CQ_OK;
  if (amax == nullptr) return CQ_ERR_ARG;
  if (!aligned(amax, 4)) return CQ_ERR_ALIGN;
  if (int dv = check_device()) return dv;
  cq::RotQuantArgs a{x, M, M_pad, static_cast<int>(K), 0, 0, 0, nullptr, nullptr, nullptr, nullptr,
                     cq::rsplit_cols(static_cast<int>(K))};
  a.amax_out = amax;
  return cuda_status(cq::launch_act_rotquant(rot_group, false, CQ_ACT_INT8_ROW, a, static_cast<cudaStream_t>(stream)));
}

int cq_rotquant_scaled(const void* x, int64_t M, int64_t K, int rot_group, const float* amax, int64_t M_pad,
                       int flags, void* q, float* scale, void* group_sums, void* stream) {
  if (int e = check_sharded_act(x, M, K, rot_group, M_pad)) return e;
  if (flags & ~CQ_Q_KPERM) return CQ_ERR_ARG;
  if (M_pad == 0) return CQ_OK;
  if (amax == nullptr || q == nullptr || scale == nullptr) return CQ_ERR_ARG;
  if (!aligned(amax, 4) || !aligned(q, 16) || !aligned(scale, 4) || !aligned(group_sums, 16)) return CQ_ERR_ALIGN;
  if (int dv = check_device()) return dv;
  cq::RotQuantArgs a{x, M, M_pad, static_cast<int>(K), 0, 0, (flags & CQ_Q_KPERM) ? 1 : 0, q, scale, nullptr,
                     static_cast<__nv_bfloat16*>(group_sums), cq::rsplit_cols(static_cast<int>(K))};
  a.amax_in = amax;
  return cuda_status(cq::launch_act_rotquant(rot_group, false, CQ_ACT_INT8_ROW, a, static_cast<cudaStream_t>(stream)));
}

int cq_qkv_rmsnorm_rope(const void* y, int64_t S, int H, int D, const void* q_norm, const void* k_norm, float eps,
                        const float* rope, void* q, void* k, void* v, int64_t s_all, int64_t s0, void* stream) {
  return cq_qkv_rmsnorm_rope_layout(y, S, H, D, q_norm, k_norm, eps, rope, q, k, v, s_all, s0, 0, stream);
}

int cq_qkv_rmsnorm_rope_layout(const void* y, int64_t S, int H, int D, const void* q_norm, const void* k_norm,
                               float eps, const float* rope, void* q, void* k, void* v, int64_t s_all, int64_t s0,
                               int token_major, void* stream) {
  if (token_major != 0 && token_major != 1) return CQ_ERR_ARG;
  if (S < 0 || S > kMaxRows || H < 1 || H > 4096 || (D != 64 && D != 128)) return CQ_ERR_SHAPE;
  if (s0 < 0 || s_all < s0 + S || s_all > kMaxRows) return CQ_ERR_SHAPE;
  if (!(eps >= 0.0f)) return CQ_ERR_ARG;
  if (S == 0) return CQ_OK;
  if (y == nullptr || q_norm == nullptr || k_norm == nullptr || rope == nullptr || q == nullptr || k == nullptr ||
      v == nullptr)
    return CQ_ERR_ARG;
  if (!aligned(y, 8) || !aligned(q, 8) || !aligned(k, 8) || !aligned(v, 8) || !aligned(rope, 8) ||
      !aligned(q_norm, 8) || !aligned(k_norm, 8))
    return CQ_ERR_ALIGN;
  if (int dv = check_device()) return dv;
  cq::QkvRopeArgs a{static_cast<const __nv_bfloat16*>(y), static_cast<const __nv_bfloat16*>(q_norm),
                    static_cast<const __nv_bfloat16*>(k_norm), rope, static_cast<__nv_bfloat16*>(q),
                    static_cast<__nv_bfloat16*>(k), static_cast<__nv_bfloat16*>(v), S, s_all, s0, H, D, eps,
                    token_major ? static_cast<int64_t>(H) * D : D, token_major ? D : s_all * D};
  return cuda_status(cq::launch_qkv_rmsnorm_rope(a, static_cast<cudaStream_t>(stream)));
}

int cq_rmsnorm_rope_rows(const void* x, int64_t S, int C, const void* w, float eps, const float* rope, int D,
                         void* out, void* stream) {
  if (S < 0 || S > kMaxRows || C < 8 || C % 8 != 0 || C > 16384) return CQ_ERR_SHAPE;
  if (rope != nullptr && ((D != 64 && D != 128) || C % D != 0)) return CQ_ERR_SHAPE;
  if (!(eps >= 0.0f)) return CQ_ERR_ARG;
  if (S == 0) return CQ_OK;
  if (x == nullptr || w == nullptr || out == nullptr) return CQ_ERR_ARG;
  if (!aligned(x, 16) || !aligned(w, 16) || !aligned(out, 16) || (rope != nullptr && !aligned(rope, 8)))
    return CQ_ERR_ALIGN;
  if (int dv = check_device()) return dv;
  cq::RmsRopeArgs a{static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w), rope,
                    static_cast<__nv_bfloat16*>(out), S, C, rope != nullptr ? D : 0, eps, 1};
  return cuda_status(cq::launch_rmsnorm_rope_rows(a, static_cast<cudaStream_t>(stream)));
}

int cq_heads_to_rows(const void* o, int64_t S, int Hp, int D, void* const* outs, int n_outs, int64_t col0,
                     int64_t ldo, void* stream) {
  if (S < 0 || S > kMaxRows || Hp < 1 || (D != 64 && D != 128) || Hp * D > 8192) return CQ_ERR_SHAPE;
  if (col0 < 0 || col0 % 8 != 0 || ldo % 8 != 0 || col0 + static_cast<int64_t>(Hp) * D > ldo) return CQ_ERR_SHAPE;
  if (outs == nullptr || n_outs < 1 || n_outs > cq::kMaxOutBuffers) return CQ_ERR_ARG;
  if (S == 0) return CQ_OK;
  if (o == nullptr) return CQ_ERR_ARG;
  if (!aligned(o, 16)) return CQ_ERR_ALIGN;
  cq::HeadsToRowsArgs a{};
  a.src = static_cast<const __nv_bfloat16*>(o);
  for (int i = 0; i < n_outs; ++i) {
    if (outs[i] == nullptr) return CQ_ERR_ARG;
    if (!aligned(outs[i], 16)) return CQ_ERR_ALIGN;
    a.outs[i] = static_cast<__nv_bfloat16*>(outs[i]);
  }
  if (int dv = check_device()) return dv;
  a.n_out = n_outs;
  a.S = S;
  a.Hp = Hp;
  a.D = D;
  a.col0 = col0;
  a.ldo = ldo;
  return cuda_status(cq::launch_heads_to_rows(a, static_cast<cudaStream_t>(stream)));
}

int cq_weight_rotquant(const void* w, int w_is_bf16, int64_t N, int64_t K, int rot_group, int mode, int group,
                       void* q, void* scale, void* zeros, void* stream) {
  if (N < 0 || N > kMaxRows) return CQ_ERR_SHAPE;
  if (K < 256 || K % 256 != 0 || K > kMaxK) return CQ_ERR_SHAPE;
  if (!valid_rot(rot_group)) return CQ_ERR_ARG;
  int kmode;
  switch (mode) {
    case CQ_W_INT4_ROW: kmode = 10; break;
    case CQ_W_INT8_ROW: kmode = 11; break;
    case CQ_W_AFFINE_INT4_GROUP: kmode = 12; break;
    case CQ_W_INT4_GROUP_BF16UP: kmode = 13; break;
    default: return CQ_ERR_ARG;
  }
  const bool grouped = mode == CQ_W_AFFINE_INT4_GROUP || mode == CQ_W_INT4_GROUP_BF16UP;
  if (grouped && group != 64 && group != 128) return CQ_ERR_ARG;
  if (N == 0) return CQ_OK;
  if (w == nullptr || q == nullptr || scale == nullptr || (mode == CQ_W_AFFINE_INT4_GROUP && zeros == nullptr))
    return CQ_ERR_ARG;
  if (!aligned(w, 16) || !aligned(q, 16) || !aligned(scale, 4) || !aligned(zeros, 2)) return CQ_ERR_ALIGN;
  if (int dv = check_device()) return dv;
  cq::RotQuantArgs a{w, N, N, static_cast<int>(K), grouped ? group : 0, 0, 0, q, scale, zeros, nullptr, 0};
  return cuda_status(cq::launch_weight_rotquant(rot_group, w_is_bf16 != 0, kmode, a, static_cast<cudaStream_t>(stream)));
}

int cq_unpack_int4(const void* src, int64_t R, int64_t C, void* dst, void* stream) {
  if (R < 0 || C < 0 || C % 16 != 0) return CQ_ERR_SHAPE;
  if (R == 0 || C == 0) return CQ_OK;
  if (src == nullptr || dst == nullptr) return CQ_ERR_ARG;
  if (!aligned(src, 8) || !aligned(dst, 16)) return CQ_ERR_ALIGN;
  if (int dv = check_device()) return dv;
  return cuda_status(cq::launch_unpack_int4(src, R * C / 2, dst, static_cast<cudaStream_t>(stream)));
}

static int check_gemm(const void* a, const void* b, const void* out, int64_t M, int64_t N, int64_t K) {
  if (M < 0 || N <= 0 || M > kMaxRows || N > kMaxRows) return CQ_ERR_SHAPE;
  if (K < 128 || K % 128 != 0 || K > (int64_t(1) << 17)) return CQ_ERR_SHAPE;
  if (M == 0) return CQ_OK;
  if (a == nullptr || b == nullptr || out == nullptr) return CQ_ERR_ARG;
  if (!aligned(a, 16) || !aligned(b, 16) || !aligned(out, 2)) return CQ_ERR_ALIGN;
  return CQ_OK;
}

static int gemm_rowcol(const int8_t* a, int a_kperm, const float* sa, const void* b, int b_format, const float* sb,
                       const void* bias, void* out, int64_t M, int64_t N, int64_t K, void* stream, bool pdl,
                       const cq::OutOp* op = nullptr);

int cq_gemm_rowcol(const int8_t* a, int a_kperm, const float* sa, const void* b, int b_format, const float* sb,
                   const void* bias, void* out, int64_t M, int64_t N, int64_t K, void* stream) {
  return gemm_rowcol(a, a_kperm, sa, b, b_format, sb, bias, out, M, N, K, stream, false);
}

// pdl: the fused linears launch the GEMM as a programmatic dependent of their activation kernel
static int gemm_rowcol(const int8_t* a, int a_kperm, const float* sa, const void* b, int b_format, const float* sb,
                       const void* bias, void* out, int64_t M, int64_t N, int64_t K, void* stream, bool pdl,
                       const cq::OutOp* op) {
  if (b_format != CQ_B_INT4_SIGNED && b_format != CQ_B_INT8) return CQ_ERR_ARG;
  if (a_kperm != 0 && (a_kperm != 1 || b_format == CQ_B_INT8)) return CQ_ERR_ARG;
  if (int e = check_gemm(a, b, out, M, N, K)) return e;
  if (M == 0) return CQ_OK;
  if (sa == nullptr || sb == nullptr) return CQ_ERR_ARG;
  if (int dv = check_device()) return dv;
  return cq::launch_gemm_rowcol(a, a_kperm, sa, b, b_format, sb, bias, out, static_cast<int>(M), static_cast<int>(N),
                                static_cast<int>(K), static_cast<cudaStream_t>(stream), pdl, op);
}

int cq_gemm_groupwise(const int8_t* a, int a_kperm, const float* sa_g, int64_t sa_ld, const void* b_packed,
                      const float* sb_g, const void* bias, void* out, int64_t M, int64_t N, int64_t K, int group,
                      void* stream) {
  if (group != 128) return CQ_ERR_ARG;
  if (a_kperm != 0 && a_kperm != 1) return CQ_ERR_ARG;
  if (int e = check_gemm(a, b_packed, out, M, N, K)) return e;
  if (M == 0) return CQ_OK;
  if (K > kMaxK) return CQ_ERR_SHAPE;
  if (sa_ld < M || sa_ld % 4 != 0 || sa_ld > kMaxRows) return CQ_ERR_SHAPE;
  if (sa_g == nullptr || sb_g == nullptr) return CQ_ERR_ARG;
  if (!aligned(sa_g, 16) || !aligned(sb_g, 4)) return CQ_ERR_ALIGN;
  if (int dv = check_device()) return dv;
  return cq::launch_gemm_group(a, a_kperm, sa_g, sa_ld, b_packed, sb_g, bias, out, static_cast<int>(M),
                               static_cast<int>(N), static_cast<int>(K), static_cast<cudaStream_t>(stream));
}

int cq_gemm_intratio(const int8_t* a, int a_kperm, const float* sa, const void* b_packed, const float* sb,
                     const void* cw, int cw_u8, int cw_group, const void* bias, void* out, int64_t M, int64_t N,
                     int64_t K, void* stream) {
  if (a_kperm != 0 && a_kperm != 1) return CQ_ERR_ARG;
  if (cw_group != 64 && cw_group != 128) return CQ_ERR_ARG;
  if (cw_u8 != 0 && cw_u8 != 1) return CQ_ERR_ARG;
  if (int e = check_gemm(a, b_packed, out, M, N, K)) return e;
  if (M == 0) return CQ_OK;
  if (K >= 171840) return CQ_ERR_SHAPE;          // the reference's int32 accumulator bound
  if (sa == nullptr || sb == nullptr || cw == nullptr) return CQ_ERR_ARG;
  if (!aligned(cw, cw_u8 ? 1 : 4) || !aligned(sa, 4) || !aligned(sb, 4)) return CQ_ERR_ALIGN;
  if (int dv = check_device()) return dv;
  return cq::launch_gemm_intratio(a, a_kperm, sa, b_packed, sb, cw, cw_u8, cw_group, bias, out, static_cast<int>(M),
                                  static_cast<int>(N), static_cast<int>(K), static_cast<cudaStream_t>(stream));
}

static int gemm_affine(const int8_t* a, int a_kperm, const float* sa, const void* gsplit, const void* b_packed,
                       const void* s_bf16, const void* zt_bf16, const void* bias, const cq_out_op* op, void* out,
                       int64_t M, int64_t N, int64_t K, int group, void* stream, bool pdl, float* partial = nullptr);

int cq_gemm_affine(const int8_t* a, int a_kperm, const float* sa, const void* gsplit, const void* b_packed,
                   const void* s_bf16, const void* zt_bf16, const void* bias, void* out, int64_t M, int64_t N,
                   int64_t K, int group, void* stream) {
  return gemm_affine(a, a_kperm, sa, gsplit, b_packed, s_bf16, zt_bf16, bias, nullptr, out, M, N, K, group, stream,
                     false);
}

// the output operation of cq_gemm_affine_op: a known kind and, for the gated residual, a residual that is either
// the output itself (same rows) or wholly apart from it
static int check_out_op(const cq_out_op* op, const void* out, int64_t M, int64_t N) {
  if (op == nullptr || op->kind == CQ_OUT_PLAIN) return CQ_OK;
  if (op->kind != CQ_OUT_GELU_TANH && op->kind != CQ_OUT_GATED_RESIDUAL) return CQ_ERR_ARG;
  // the operations run in the epilogue's staged (TMA-store) output path
  if (N % 8 != 0) return CQ_ERR_SHAPE;
  if (!aligned(out, 16)) return CQ_ERR_ALIGN;
  if (op->kind == CQ_OUT_GELU_TANH) return CQ_OK;
  if (op->residual == nullptr || op->gate == nullptr) return CQ_ERR_ARG;
  if (op->residual_ld < N || op->residual_ld > (int64_t(1) << 31)) return CQ_ERR_SHAPE;
  if (!aligned(op->residual, 2) || !aligned(op->gate, 2)) return CQ_ERR_ALIGN;
  const uintptr_t r0 = reinterpret_cast<uintptr_t>(op->residual), o0 = reinterpret_cast<uintptr_t>(out);
  if (r0 == o0) return op->residual_ld == N ? CQ_OK : CQ_ERR_ARG;
  const uintptr_t r1 = r0 + static_cast<uintptr_t>(((M - 1) * op->residual_ld + N) * 2);
  const uintptr_t o1 = o0 + static_cast<uintptr_t>(M * N * 2);
  return (r1 <= o0 || o1 <= r0) ? CQ_OK : CQ_ERR_ARG;
}

int cq_gemm_affine_op(const int8_t* a, int a_kperm, const float* sa, const void* gsplit, const void* b_packed,
                      const void* s_bf16, const void* zt_bf16, const void* bias, const cq_out_op* op, void* out,
                      int64_t M, int64_t N, int64_t K, int group, void* stream) {
  return gemm_affine(a, a_kperm, sa, gsplit, b_packed, s_bf16, zt_bf16, bias, op, out, M, N, K, group, stream, false);
}

static int gemm_affine(const int8_t* a, int a_kperm, const float* sa, const void* gsplit, const void* b_packed,
                       const void* s_bf16, const void* zt_bf16, const void* bias, const cq_out_op* op, void* out,
                       int64_t M, int64_t N, int64_t K, int group, void* stream, bool pdl, float* partial) {
  if (group != 128) return CQ_ERR_ARG;
  if (a_kperm != 0 && a_kperm != 1) return CQ_ERR_ARG;
  if (int e = check_gemm(a, b_packed, out, M, N, K)) return e;
  if (M == 0) return CQ_OK;
  if (K > kMaxK) return CQ_ERR_SHAPE;
  if (sa == nullptr || gsplit == nullptr || s_bf16 == nullptr || zt_bf16 == nullptr) return CQ_ERR_ARG;
  if (!aligned(gsplit, 16) || !aligned(zt_bf16, 16)) return CQ_ERR_ALIGN;
  if (int e = check_out_op(op, out, M, N)) return e;
  if (int dv = check_device()) return dv;
  cq::OutOp o{};
  if (op != nullptr) o = cq::OutOp{op->kind, op->residual, op->residual_ld, op->gate};
  return cq::launch_gemm_affine(a, a_kperm, sa, gsplit, b_packed, s_bf16, zt_bf16, bias, out, static_cast<int>(M),
                                static_cast<int>(N), static_cast<int>(K), static_cast<cudaStream_t>(stream), nullptr,
                                0, 0, 0, &o, pdl, partial);
}

// ---------------------------------------------------------------------------------------------
// fused linears: activation stage into the caller's workspace, then the GEMM
// ---------------------------------------------------------------------------------------------
static int64_t ws_mpad(int64_t M) { return round_up(M > 0 ? M : 1, 16); }

int64_t cq_linear_workspace_bytes(int64_t M, int64_t K) {
  if (M < 0 || K <= 0) return -1;
  const int64_t mp = ws_mpad(M);
  return round_up(mp * K, 256) + round_up(mp * 4, 256) + round_up(mp * cq_group_sum_cols(K) * 2, 256);
}

// room for the K-split partial sums of an affine GEMM with too few tiles to fill the SMs (0 when it does not split)
static int64_t splitk_bytes(int64_t M, int64_t K, int64_t N) {
  if (M <= 8 || M > kMaxRows || N <= 0 || N > kMaxRows || K < 128 || K % 128 != 0) return 0;
  const int s = cq::affine_ksplit(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K));
  return s > 1 ? round_up(static_cast<int64_t>(s) * M * N * 4, 256) : 0;
}

int64_t cq_linear_workspace_bytes_n(int64_t M, int64_t K, int64_t N) {
  const int64_t base = cq_linear_workspace_bytes(M, K);
  if (base < 0) return base;
  return base + splitk_bytes(M, K, N);
}

// the partial-sum region of a workspace given with room for it, else null (the GEMM then runs unsplit)
static float* splitk_region(void* ws, int64_t ws_bytes, int64_t M, int64_t K, int64_t N) {
  const int64_t extra = splitk_bytes(M, K, N);
  const int64_t base = cq_linear_workspace_bytes(M, K);
  if (extra == 0 || ws_bytes < base + extra) return nullptr;
  return reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + base);
}

struct Workspace {
  int8_t* xq;
  float* sx;
  __nv_bfloat16* gsplit;
  int64_t mpad;
};

static int carve(void* ws, int64_t ws_bytes, int64_t M, int64_t K, Workspace* w) {
  const int64_t need = cq_linear_workspace_bytes(M, K);
  if (ws == nullptr || ws_bytes < need) return CQ_ERR_ARG;
  if (!aligned(ws, 256)) return CQ_ERR_ALIGN;
  w->mpad = ws_mpad(M);
  uint8_t* p = static_cast<uint8_t*>(ws);
  w->xq = reinterpret_cast<int8_t*>(p);
  p += round_up(w->mpad * K, 256);
  w->sx = reinterpret_cast<float*>(p);
  p += round_up(w->mpad * 4, 256);
  w->gsplit = reinterpret_cast<__nv_bfloat16*>(p);
  return CQ_OK;
}

int cq_linear_convrot_w4a4(const void* x, int64_t M, int64_t K, int64_t N, int rot_group, int swiglu, int act_bits,
                           const void* qweight, const float* wscale, const void* bias, void* out, void* workspace,
                           int64_t workspace_bytes, void* stream) {
  if (act_bits != 4 && act_bits != 8) return CQ_ERR_ARG;
  if (M == 0) return CQ_OK;
  Workspace w;
  if (int e = carve(workspace, workspace_bytes, M, K, &w)) return e;
  const int mode = act_bits == 4 ? CQ_ACT_INT4_ROW : CQ_ACT_INT8_ROW;
  if (int e = cq_rotquant(x, M, K, rot_group, swiglu, mode, 0, w.mpad, CQ_Q_INT8_CODES | CQ_Q_KPERM, w.xq, w.sx,
                          nullptr, stream))
    return e;
  return gemm_rowcol(w.xq, 1, w.sx, qweight, CQ_B_INT4_SIGNED, wscale, bias, out, M, N, K, stream, true);
}

static int gemm_rowcol_swiglu(const int8_t* a, const float* sa, const void* b_glu, const float* sb, const void* bias,
                              void* out, int64_t M, int64_t N, int64_t K, void* stream, bool pdl);

int cq_gemm_rowcol_swiglu(const int8_t* a, const float* sa, const void* b_glu, const float* sb, const void* bias,
                          void* out, int64_t M, int64_t N, int64_t K, void* stream) {
  return gemm_rowcol_swiglu(a, sa, b_glu, sb, bias, out, M, N, K, stream, false);
}

static int gemm_rowcol_swiglu(const int8_t* a, const float* sa, const void* b_glu, const float* sb, const void* bias,
                              void* out, int64_t M, int64_t N, int64_t K, void* stream, bool pdl) {
  if (N % 128 != 0) return CQ_ERR_SHAPE;            // whole 128-row weight tiles of 16-gate + 16-up row groups
  if (int e = check_gemm(a, b_glu, out, M, N, K)) return e;
  if (M == 0) return CQ_OK;
  if (sa == nullptr || sb == nullptr) return CQ_ERR_ARG;
  if (int dv = check_device()) return dv;
  return cq::launch_gemm_rowcol_glu(a, sa, b_glu, sb, bias, out, static_cast<int>(M), static_cast<int>(N),
                                    static_cast<int>(K), static_cast<cudaStream_t>(stream), pdl);
}

int cq_linear_convrot_w4a4_swiglu(const void* x, int64_t M, int64_t K, int64_t N, int rot_group, int act_bits,
                                  const void* qweight_glu, const float* wscale_glu, const void* bias_glu, void* out,
                                  void* workspace, int64_t workspace_bytes, void* stream) {
  if (act_bits != 4 && act_bits != 8) return CQ_ERR_ARG;
  if (N % 128 != 0) return CQ_ERR_SHAPE;            // checked before the activations are quantized
  if (M == 0) return CQ_OK;
  Workspace w;
  if (int e = carve(workspace, workspace_bytes, M, K, &w)) return e;
  const int mode = act_bits == 4 ? CQ_ACT_INT4_ROW : CQ_ACT_INT8_ROW;
  if (int e = cq_rotquant(x, M, K, rot_group, 0, mode, 0, w.mpad, CQ_Q_INT8_CODES | CQ_Q_KPERM, w.xq, w.sx, nullptr,
                          stream))
    return e;
  return gemm_rowcol_swiglu(w.xq, w.sx, qweight_glu, wscale_glu, bias_glu, out, M, N, K, stream, true);
}

int cq_gemm_affine_peers(const int8_t* a, int a_kperm, const float* sa, const void* gsplit, const void* b_packed,
                         const void* s_bf16, const void* zt_bf16, const void* bias, void* const* outs, int n_outs,
                         int64_t col0, int64_t ldo, int64_t M, int64_t N, int64_t K, int group, void* stream) {
  if (group != 128) return CQ_ERR_ARG;
  if (a_kperm != 0 && a_kperm != 1) return CQ_ERR_ARG;
  if (outs == nullptr || n_outs < 1 || n_outs > cq::kMaxOutBuffers) return CQ_ERR_ARG;
  for (int i = 0; i < n_outs; ++i) {
    if (outs[i] == nullptr) return CQ_ERR_ARG;
    if (!aligned(outs[i], 16)) return CQ_ERR_ALIGN;
  }
  // whole 32-column store boxes of this launch, 16-byte aligned, inside the output rows
  if (N % 32 != 0 || col0 < 0 || col0 % 8 != 0 || ldo % 8 != 0 || col0 + N > ldo || ldo > kMaxRows)
    return CQ_ERR_SHAPE;
  if (int e = check_gemm(a, b_packed, outs[0], M, N, K)) return e;
  if (M == 0) return CQ_OK;
  if (K > kMaxK) return CQ_ERR_SHAPE;
  if (sa == nullptr || gsplit == nullptr || s_bf16 == nullptr || zt_bf16 == nullptr) return CQ_ERR_ARG;
  if (!aligned(gsplit, 16) || !aligned(zt_bf16, 16)) return CQ_ERR_ALIGN;
  if (int dv = check_device()) return dv;
  return cq::launch_gemm_affine(a, a_kperm, sa, gsplit, b_packed, s_bf16, zt_bf16, bias, outs[0], static_cast<int>(M),
                                static_cast<int>(N), static_cast<int>(K), static_cast<cudaStream_t>(stream), outs,
                                n_outs, static_cast<int>(col0), ldo);
}

int cq_linear_w4a8_affine_peers(const void* x, int64_t M, int64_t K, int64_t N, int rot_group, int swiglu,
                                const void* qweight, const void* s_bf16, const void* zt_bf16, int group,
                                const void* bias, void* const* outs, int n_outs, int64_t col0, int64_t ldo,
                                void* workspace, int64_t workspace_bytes, void* stream) {
  if (M == 0) return CQ_OK;
  Workspace w;
  if (int e = carve(workspace, workspace_bytes, M, K, &w)) return e;
  if (int e = cq_rotquant(x, M, K, rot_group, swiglu, CQ_ACT_INT8_ROW, 0, w.mpad, CQ_Q_KPERM, w.xq, w.sx, w.gsplit,
                          stream))
    return e;
  return cq_gemm_affine_peers(w.xq, 1, w.sx, w.gsplit, qweight, s_bf16, zt_bf16, bias, outs, n_outs, col0, ldo, M, N,
                              K, group, stream);
}

int cq_linear_w4a8_affine(const void* x, int64_t M, int64_t K, int64_t N, int rot_group, int swiglu,
                          const void* qweight, const void* s_bf16, const void* zt_bf16, int group, const void* bias,
                          void* out, void* workspace, int64_t workspace_bytes, void* stream) {
  if (M == 0) return CQ_OK;
  Workspace w;
  if (int e = carve(workspace, workspace_bytes, M, K, &w)) return e;
  if (int e = cq_rotquant(x, M, K, rot_group, swiglu, CQ_ACT_INT8_ROW, 0, w.mpad, CQ_Q_KPERM, w.xq, w.sx, w.gsplit,
                          stream))
    return e;
  return gemm_affine(w.xq, 1, w.sx, w.gsplit, qweight, s_bf16, zt_bf16, bias, nullptr, out, M, N, K, group, stream,
                     true, splitk_region(workspace, workspace_bytes, M, K, N));
}

int cq_linear_w4a8_affine_lnmod(const void* x, int64_t M, int64_t K, int64_t N, int rot_group, const void* shift,
                                const void* scale1p, float eps, const void* qweight, const void* s_bf16,
                                const void* zt_bf16, int group, const void* bias, void* out, void* workspace,
                                int64_t workspace_bytes, void* stream) {
  if (M == 0) return CQ_OK;
  Workspace w;
  if (int e = carve(workspace, workspace_bytes, M, K, &w)) return e;
  if (int e = cq_rotquant_lnmod(x, M, K, rot_group, shift, scale1p, eps, w.mpad, CQ_Q_KPERM, w.xq, w.sx, w.gsplit,
                                stream))
    return e;
  return gemm_affine(w.xq, 1, w.sx, w.gsplit, qweight, s_bf16, zt_bf16, bias, nullptr, out, M, N, K, group, stream,
                     true, splitk_region(workspace, workspace_bytes, M, K, N));
}

int cq_linear_w4a8_op(const void* x, int64_t M, int64_t K, int64_t N, int rot_group, const void* shift,
                      const void* mod_scale, float eps, const void* qweight, const void* s_bf16, const void* zt_bf16,
                      int group, const void* bias, const cq_out_op* op, void* out, void* workspace,
                      int64_t workspace_bytes, void* stream) {
  if (M == 0) return CQ_OK;
  if (int e = check_out_op(op, out, M, N)) return e;
  Workspace w;
  if (int e = carve(workspace, workspace_bytes, M, K, &w)) return e;
  const int e = shift != nullptr
                    ? rotquant_lnmod(x, M, K, rot_group, shift, mod_scale, eps, w.mpad, CQ_Q_KPERM, w.xq, w.sx,
                                     w.gsplit, stream, true)
                    : cq_rotquant(x, M, K, rot_group, 0, CQ_ACT_INT8_ROW, 0, w.mpad, CQ_Q_KPERM, w.xq, w.sx, w.gsplit,
                                  stream);
  if (e) return e;
  return gemm_affine(w.xq, 1, w.sx, w.gsplit, qweight, s_bf16, zt_bf16, bias, op, out, M, N, K, group, stream, true,
                     splitk_region(workspace, workspace_bytes, M, K, N));
}

// the library's epilogue operation from the public one (the same kind codes; null: plain output)
static const cq::OutOp* to_out_op(const cq_out_op* op, cq::OutOp* buf) {
  if (op == nullptr || op->kind == CQ_OUT_PLAIN) return nullptr;
  *buf = cq::OutOp{op->kind, op->residual, op->residual_ld, op->gate};
  return buf;
}

// the fused row/col linears with an epilogue operation: activations (optionally of the modulated layer norm), then
// the GEMM as a programmatic dependent with `op` in its epilogue
static int linear_rowcol_op(const void* x, int64_t M, int64_t K, int64_t N, int rot_group, int mode,
                            const void* shift, const void* mod_scale, float eps, const void* weight, int b_format,
                            const float* wscale, const void* bias, const cq_out_op* op, void* out, void* workspace,
                            int64_t workspace_bytes, void* stream) {
  if (M == 0) return CQ_OK;
  if (int e = check_out_op(op, out, M, N)) return e;
  Workspace w;
  if (int e = carve(workspace, workspace_bytes, M, K, &w)) return e;
  const int kperm = b_format == CQ_B_INT4_SIGNED ? CQ_Q_KPERM : 0;
  const int codes = mode == CQ_ACT_INT4_ROW ? CQ_Q_INT8_CODES : 0;
  const int e = shift != nullptr
                    ? rotquant_lnmod(x, M, K, rot_group, shift, mod_scale, eps, w.mpad, kperm, w.xq, w.sx, nullptr,
                                     stream, true, mode)
                    : cq_rotquant(x, M, K, rot_group, 0, mode, 0, w.mpad, codes | kperm, w.xq, w.sx, nullptr, stream);
  if (e) return e;
  cq::OutOp buf;
  return gemm_rowcol(w.xq, kperm ? 1 : 0, w.sx, weight, b_format, wscale, bias, out, M, N, K, stream, true,
                     to_out_op(op, &buf));
}

int cq_linear_convrot_w4a4_op(const void* x, int64_t M, int64_t K, int64_t N, int rot_group, int act_bits,
                              const void* shift, const void* mod_scale, float eps, const void* qweight,
                              const float* wscale, const void* bias, const cq_out_op* op, void* out, void* workspace,
                              int64_t workspace_bytes, void* stream) {
  if (act_bits != 4 && act_bits != 8) return CQ_ERR_ARG;
  return linear_rowcol_op(x, M, K, N, rot_group, act_bits == 4 ? CQ_ACT_INT4_ROW : CQ_ACT_INT8_ROW, shift, mod_scale,
                          eps, qweight, CQ_B_INT4_SIGNED, wscale, bias, op, out, workspace, workspace_bytes, stream);
}

int cq_linear_w8a8_op(const void* x, int64_t M, int64_t K, int64_t N, int rot_group, const void* shift,
                      const void* mod_scale, float eps, const int8_t* weight, const float* wscale, const void* bias,
                      const cq_out_op* op, void* out, void* workspace, int64_t workspace_bytes, void* stream) {
  return linear_rowcol_op(x, M, K, N, rot_group, CQ_ACT_INT8_ROW, shift, mod_scale, eps, weight, CQ_B_INT8, wscale,
                          bias, op, out, workspace, workspace_bytes, stream);
}

int cq_linear_w8a8(const void* x, int64_t M, int64_t K, int64_t N, int rot_group, int swiglu, const int8_t* weight,
                   const float* wscale, const void* bias, void* out, void* workspace, int64_t workspace_bytes,
                   void* stream) {
  if (M == 0) return CQ_OK;
  Workspace w;
  if (int e = carve(workspace, workspace_bytes, M, K, &w)) return e;
  if (int e = cq_rotquant(x, M, K, rot_group, swiglu, CQ_ACT_INT8_ROW, 0, w.mpad, 0, w.xq, w.sx, nullptr, stream))
    return e;
  return gemm_rowcol(w.xq, 0, w.sx, weight, CQ_B_INT8, wscale, bias, out, M, N, K, stream, true);
}

}  // extern "C"
