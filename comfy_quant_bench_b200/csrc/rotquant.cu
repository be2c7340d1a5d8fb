// Rotation + quantization kernels (activations and weights), sm_100a.
//
// One CTA per row.  Each warp owns "pairs" of 256-element blocks (512 elements): lane l holds the 16
// contiguous elements [16l, 16l+16) of its pair in registers (two 16-byte loads of bf16, four of f32).
//
// Rotation (kron^p of the regular order-4 Hadamard, divided by 2^p, p = log4(group)) runs as radix-4 stages
// in the order of the reference quantizer (experiments/qwen21-kernel/kernels/g64_quant.cu:68-85: strides 1, 4,
// 16, 64), each butterfly hs = 0.5*(((x0+x1)+x2)+x3); y_i = hs - x_{3-i} with one rounding per operation
// (explicit _rn intrinsics: no FMA contraction), so codes and scales match the CPU oracle bit for bit:
//   * strides 1 and 4 act on the 16 register-resident elements of a lane;
//   * strides 16 and 64 act across lanes: the warp transposes its 512 values through a swizzled, padded
//     shared-memory tile (conflict-free 16-byte and 4-byte phases), runs the two stages in registers and
//     transposes back.
// Quantization then runs in the load layout, so every store is a contiguous 16-, 8- or 4-byte vector.
#include "kernels.cuh"

namespace cq {

enum : int {
  MODE_ACT_INT8_ROW = 0,
  MODE_ACT_INT4_ROW = 1,
  MODE_ACT_INT4_GROUP = 2,
  MODE_W_INT4_ROW = 10,
  MODE_W_INT8_ROW = 11,
  MODE_W_AFFINE = 12,
  MODE_W_INT4_GROUP_BF16UP = 13,
};

__device__ __forceinline__ void h4r_butterfly(float& x0, float& x1, float& x2, float& x3) {
  const float hs = __fmul_rn(0.5f, __fadd_rn(__fadd_rn(__fadd_rn(x0, x1), x2), x3));
  const float y0 = __fsub_rn(hs, x3), y1 = __fsub_rn(hs, x2), y2 = __fsub_rn(hs, x1), y3 = __fsub_rn(hs, x0);
  x0 = y0; x1 = y1; x2 = y2; x3 = y3;
}

// stride-1 stage (digit 0) then stride-4 stage (digit 1) on 16 register values
__device__ __forceinline__ void stages_1_4(float (&v)[16]) {
#pragma unroll
  for (int a = 0; a < 4; ++a) h4r_butterfly(v[4 * a + 0], v[4 * a + 1], v[4 * a + 2], v[4 * a + 3]);
#pragma unroll
  for (int d = 0; d < 4; ++d) h4r_butterfly(v[d], v[d + 4], v[d + 8], v[d + 12]);
}

// shared-memory index of element r of writer lane wl inside a warp's 528-float transpose tile
__device__ __forceinline__ int tp_index(int wl, int r) {
  const int quad = (r >> 2) ^ ((wl >> 1) & 3);
  return wl * 16 + ((wl >> 4) << 4) + quad * 4 + (r & 3);
}

// strides 16 (and 64 when ROT == 256) across lanes, through the warp's transpose tile
template <int ROT>
__device__ __forceinline__ void stages_cross(float (&v)[16], float* tile, int lane) {
  static_assert(ROT == 64 || ROT == 256, "cross-lane stages only for 64 and 256");
#pragma unroll
  for (int j = 0; j < 4; ++j)
    *reinterpret_cast<float4*>(tile + tp_index(lane, 4 * j)) = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  __syncwarp();
  const int h = lane >> 4, c = lane & 15;
  float u[16];
#pragma unroll
  for (int t = 0; t < 16; ++t) u[t] = tile[tp_index(16 * h + t, c)];
  // digit 2: element stride 16 == consecutive t
#pragma unroll
  for (int a = 0; a < 4; ++a) h4r_butterfly(u[4 * a + 0], u[4 * a + 1], u[4 * a + 2], u[4 * a + 3]);
  if (ROT == 256) {
#pragma unroll
    for (int d = 0; d < 4; ++d) h4r_butterfly(u[d], u[d + 4], u[d + 8], u[d + 12]);
  }
  __syncwarp();
#pragma unroll
  for (int t = 0; t < 16; ++t) tile[tp_index(16 * h + t, c)] = u[t];
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float4 f = *reinterpret_cast<const float4*>(tile + tp_index(lane, 4 * j));
    v[4 * j] = f.x; v[4 * j + 1] = f.y; v[4 * j + 2] = f.z; v[4 * j + 3] = f.w;
  }
  __syncwarp();
}

// silu(g) * u of comfy-kitchen's fused SwiGLU quantizer, rounded once to bf16: g / (1 + exp(-g)) * u with the
// hardware exponential and the approximate division its fast-math build uses (tools/ck_swiglu/swiglu_quant.cu:65)
__device__ __forceinline__ float swiglu_fused(float g, float u) {
  return bf16_round(__fmul_rn(__fdividef(g, __fadd_rn(1.0f, __expf(-g))), u));
}

__device__ __forceinline__ void load_bf16x16(const __nv_bfloat16* p, float (&v)[16]) {
  const uint4 a = *reinterpret_cast<const uint4*>(p);
  const uint4 b = *reinterpret_cast<const uint4*>(p + 8);
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[2 * i] = bf16_bits_to_f32(w[i] & 0xFFFFu);
    v[2 * i + 1] = bf16_bits_to_f32(w[i] >> 16);
  }
}

__device__ __forceinline__ void load_f32x16(const float* p, float (&v)[16]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float4 f = *reinterpret_cast<const float4*>(p + 4 * j);
    v[4 * j] = f.x; v[4 * j + 1] = f.y; v[4 * j + 2] = f.z; v[4 * j + 3] = f.w;
  }
}

template <int LANES>
__device__ __forceinline__ float group_max(float v) {
#pragma unroll
  for (int o = 1; o < LANES; o <<= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
template <int LANES>
__device__ __forceinline__ float group_min(float v) {
#pragma unroll
  for (int o = 1; o < LANES; o <<= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
template <int LANES>
__device__ __forceinline__ int group_sum(int v) {
#pragma unroll
  for (int o = 1; o < LANES; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// store 16 signed codes (values fit in 4 or 8 bits) at element offset e of the row
template <bool PACK4>
__device__ __forceinline__ void store_codes(void* qrow, int e, const int (&c)[16], bool unsigned4 = false) {
  if (PACK4) {
    uint32_t w0 = 0, w1 = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) w0 |= (static_cast<uint32_t>(c[i]) & 0xFu) << (4 * i);
#pragma unroll
    for (int i = 0; i < 8; ++i) w1 |= (static_cast<uint32_t>(c[8 + i]) & 0xFu) << (4 * i);
    (void)unsigned4;
    *reinterpret_cast<uint2*>(static_cast<uint8_t*>(qrow) + e / 2) = make_uint2(w0, w1);
  } else {
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      w[j] = (static_cast<uint32_t>(c[4 * j]) & 0xFFu) | ((static_cast<uint32_t>(c[4 * j + 1]) & 0xFFu) << 8) |
             ((static_cast<uint32_t>(c[4 * j + 2]) & 0xFFu) << 16) | ((static_cast<uint32_t>(c[4 * j + 3]) & 0xFFu) << 24);
    *reinterpret_cast<uint4*>(static_cast<int8_t*>(qrow) + e) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

constexpr int kMaxWarps = 32;

template <typename IN_T, int ROT, bool SWIGLU, int MODE, int PPW>
__global__ void __launch_bounds__(1024) rotquant_kernel(const RotQuantArgs args) {
  constexpr bool ROWWISE = MODE == MODE_ACT_INT8_ROW || MODE == MODE_ACT_INT4_ROW || MODE == MODE_W_INT4_ROW ||
                           MODE == MODE_W_INT8_ROW;
  extern __shared__ float smem_tiles[];
  __shared__ float red[kMaxWarps];

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  const int K = args.K;
  const int64_t row = blockIdx.x;
  const bool live_row = row < args.rows;
  const int npairs = (K + 511) >> 9;
  float* tile = smem_tiles + warp * 528;

  float v[PPW][16];
  bool valid[PPW];
#pragma unroll
  for (int s = 0; s < PPW; ++s) {
    const int p = warp + s * nwarps;
    const int e = p * 512 + lane * 16;
    valid[s] = (p < npairs) && (e < K);
#pragma unroll
    for (int i = 0; i < 16; ++i) v[s][i] = 0.0f;
    if (valid[s] && live_row) {
      if constexpr (SWIGLU) {
        const __nv_bfloat16* hrow = static_cast<const __nv_bfloat16*>(args.x) + row * (2 * static_cast<int64_t>(K));
        float g[16], u[16];
        load_bf16x16(hrow + e, g);
        load_bf16x16(hrow + K + e, u);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          // comfy-kitchen's fused per-token quantizer rounds the product once to bf16; the per-group quantizer
          // keeps fp32.  Both take the hardware exponential; the fused one is built with fast-math division
          // (tools/ck_swiglu/swiglu_quant.cu:65 with --use_fast_math), the per-group one divides exactly
          // (experiments/qwen21-kernel/kernels/g64_quant.cu:47-48)
          v[s][i] = (MODE == MODE_ACT_INT4_GROUP) ? __fmul_rn(__fdiv_rn(g[i], __fadd_rn(1.0f, __expf(-g[i]))), u[i])
                                                  : swiglu_fused(g[i], u[i]);
        }
      } else if constexpr (sizeof(IN_T) == 2) {
        load_bf16x16(static_cast<const __nv_bfloat16*>(args.x) + row * static_cast<int64_t>(K) + e, v[s]);
      } else {
        load_f32x16(static_cast<const float*>(args.x) + row * static_cast<int64_t>(K) + e, v[s]);
      }
    }
  }

  // ---- rotation ----
  if constexpr (ROT >= 16) {
#pragma unroll
    for (int s = 0; s < PPW; ++s) stages_1_4(v[s]);
  }
  if constexpr (ROT >= 64) {
#pragma unroll
    for (int s = 0; s < PPW; ++s) {
      const int p = warp + s * nwarps;
      if (p < npairs) stages_cross<ROT>(v[s], tile, lane);   // warp-uniform condition
    }
  }

  // ---- quantization ----
  float row_scale = 0.0f, row_inv = 0.0f;
  if constexpr (ROWWISE) {
    float am = 0.0f;
#pragma unroll
    for (int s = 0; s < PPW; ++s)
#pragma unroll
      for (int i = 0; i < 16; ++i) am = fmaxf(am, fabsf(v[s][i]));
    am = group_max<32>(am);
    if (lane == 0) red[warp] = am;
    __syncthreads();
    if (warp == 0) {
      float a = lane < nwarps ? red[lane] : 0.0f;
      a = group_max<32>(a);
      if (lane == 0) red[0] = a;
    }
    __syncthreads();
    am = red[0];
    if constexpr (MODE == MODE_ACT_INT8_ROW) {
      row_scale = fmaxf(__fmul_rn(am, 1.0f / 127.0f), 1e-10f);
      row_inv = __frcp_rn(row_scale);
    } else if constexpr (MODE == MODE_ACT_INT4_ROW) {
      row_scale = fmaxf(__fmul_rn(am, 1.0f / 7.0f), 1e-10f);
      row_inv = __frcp_rn(row_scale);
    } else if constexpr (MODE == MODE_W_INT4_ROW) {
      row_scale = fmaxf(__fdiv_rn(am, 7.0f), 1e-12f);
    } else {
      row_scale = fmaxf(__fdiv_rn(am, 127.0f), 1e-12f);
    }
    if (threadIdx.x == 0) {
      static_cast<float*>(args.scale)[row] = live_row ? row_scale : 0.0f;
    }
  }

  const int64_t ld = args.rows_pad;
  if (args.rsplit != nullptr) {
    const int G = K >> 7;
    for (int j = 2 * G + threadIdx.x; j < args.rs_cols; j += blockDim.x)
      args.rsplit[row * args.rs_cols + j] = __float2bfloat16_rn(0.0f);
  }
  const bool pack4 = !(MODE == MODE_ACT_INT8_ROW || MODE == MODE_W_INT8_ROW) && !args.int4_as_int8;
#pragma unroll
  for (int s = 0; s < PPW; ++s) {
    const int p = warp + s * nwarps;
    if (p >= npairs) continue;                      // warp-uniform
    const int e = p * 512 + lane * 16;
    int c[16];
    if constexpr (ROWWISE) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        int qi;
        if constexpr (MODE == MODE_ACT_INT8_ROW || MODE == MODE_ACT_INT4_ROW) qi = __float2int_rn(__fmul_rn(v[s][i], row_inv));
        else qi = __float2int_rn(__fdiv_rn(v[s][i], row_scale));
        const int lim = (MODE == MODE_ACT_INT8_ROW || MODE == MODE_W_INT8_ROW) ? 127 : 7;
        c[i] = live_row ? max(-lim, min(lim, qi)) : 0;
      }
    } else if constexpr (MODE == MODE_ACT_INT4_GROUP) {
      float am = 0.0f;
#pragma unroll
      for (int i = 0; i < 16; ++i) am = fmaxf(am, fabsf(v[s][i]));
      am = (args.act_group == 64) ? group_max<4>(am) : group_max<8>(am);
      const float sc = (am > 0.0f && live_row) ? bf16_up(__fdiv_rn(am, 7.0f)) : 0.0f;
      const float inv = sc > 0.0f ? __frcp_rn(sc) : 0.0f;
#pragma unroll
      for (int i = 0; i < 16; ++i) c[i] = max(-7, min(7, __float2int_rn(__fmul_rn(v[s][i], inv))));
      const int lpg = args.act_group / 16;
      if (valid[s] && (lane % lpg) == 0) static_cast<float*>(args.scale)[(e / args.act_group) * ld + row] = sc;
    } else if constexpr (MODE == MODE_W_INT4_GROUP_BF16UP) {
      float am = 0.0f;
#pragma unroll
      for (int i = 0; i < 16; ++i) am = fmaxf(am, fabsf(v[s][i]));
      am = (args.act_group == 64) ? group_max<4>(am) : group_max<8>(am);
      const float sc = bf16_up(fmaxf(__fdiv_rn(am, 7.0f), 1e-30f));
#pragma unroll
      for (int i = 0; i < 16; ++i) c[i] = max(-7, min(7, __float2int_rn(__fdiv_rn(v[s][i], sc))));
      const int lpg = args.act_group / 16;
      if (valid[s] && (lane % lpg) == 0 && live_row) static_cast<float*>(args.scale)[(e / args.act_group) * ld + row] = sc;
    } else {  // MODE_W_AFFINE
      float lo = 3.4e38f, hi = -3.4e38f;
#pragma unroll
      for (int i = 0; i < 16; ++i) { lo = fminf(lo, v[s][i]); hi = fmaxf(hi, v[s][i]); }
      if (args.act_group == 64) { lo = group_min<4>(lo); hi = group_max<4>(hi); }
      else { lo = group_min<8>(lo); hi = group_max<8>(hi); }
      const float sc = bf16_round(fmaxf(__fdiv_rn(__fsub_rn(hi, lo), 15.0f), 1e-8f));
      const float zf = bf16_round(__fadd_rn(lo, __fmul_rn(8.0f, sc)));
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float t = rintf(__fdiv_rn(__fsub_rn(v[s][i], zf), sc));
        c[i] = max(0, min(15, static_cast<int>(t) + 8));
      }
      const int lpg = args.act_group / 16;
      if (valid[s] && (lane % lpg) == 0 && live_row) {
        const int64_t o = (e / args.act_group) * ld + row;
        static_cast<__nv_bfloat16*>(args.scale)[o] = __float2bfloat16_rn(sc);
        static_cast<__nv_bfloat16*>(args.zeros)[o] = __float2bfloat16_rn(zf);
      }
    }
    if (!live_row) {
#pragma unroll
      for (int i = 0; i < 16; ++i) c[i] = 0;
    }
    if (valid[s]) {
      if (pack4) {
        store_codes<true>(static_cast<uint8_t*>(args.q) + row * (static_cast<int64_t>(K) / 2), e, c);
      } else if (args.kperm) {
        int cp[16];
#pragma unroll
        for (int b = 0; b < 2; ++b)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            cp[8 * b + j] = c[8 * b + 2 * j];
            cp[8 * b + 4 + j] = c[8 * b + 2 * j + 1];
          }
        store_codes<false>(static_cast<int8_t*>(args.q) + row * static_cast<int64_t>(K), e, cp);
      } else {
        store_codes<false>(static_cast<int8_t*>(args.q) + row * static_cast<int64_t>(K), e, c);
      }
    }
    if (args.rsplit != nullptr) {
      int sum = 0;
#pragma unroll
      for (int i = 0; i < 16; ++i) sum += c[i];
      sum = group_sum<8>(sum);
      if (valid[s] && (lane & 7) == 0) {
        const int g = e >> 7, G = K >> 7;
        const int hi = (sum >= 0 ? sum : sum - 127) / 128 * 128;   // 128 * floor(sum / 128)
        __nv_bfloat16* rrow = args.rsplit + row * args.rs_cols;
        rrow[g] = __float2bfloat16_rn(static_cast<float>(hi));
        rrow[G + g] = __float2bfloat16_rn(static_cast<float>(sum - hi));
      }
    }  }
}

// ---------------------------------------------------------------------------------------------------------
// Per-token int8 activations (the W4A8 / W8A8 activation kernel, and per-token int4 values held in int8 codes
// for the W4A4 GEMM): two rows per CTA, packed f32x2 arithmetic.
//
// A CTA of W warps ("team") owns rows 2b and 2b+1.  Every register holds a float2 (row A value, row B value) of
// the same column, so each butterfly, scale multiply and rounding step is one f32x2 instruction for two tokens,
// with exactly the per-element rounding of the scalar kernel above (same operations, same order).  Warp w of the
// team owns the 512-column chunks j = w, w + W, w + 2W; lane (h, c) holds columns 512j + 256h + 16c + [0, 16).
//   * strides 1 and 4 run in registers; the lane's 16 float2 then go through a padded shared-memory tile (row
//     stride 144 B: conflict-free 16-byte writes and 8-byte reads, immediate offsets only) so that lane (h, c)
//     holds columns 512j + 256h + 16t + c, t = 0..15, for strides 16 and 64;
//   * the codes are formed in that layout: fp32(q * (1 / scale)) + 1.5 * 2^23 (round to nearest even) leaves
//     the int8 code in the low byte; the two tokens' bytes go to a shared staging block as one 16-bit store at
//     the column's (K-permuted) position, and each lane reads back 16 contiguous columns of both rows (row
//     stride 48 B: conflict-free 16-byte reads), splits them with one byte permute per word and stores 16 bytes
//     a row;
//   * the absolute maximum propagates NaN, so a token with a NaN or infinite value is seen before rounding and
//     takes the scalar kernel's semantics (NaN ignored by the maximum, NaN products give code 0).
// Group sums for the affine GEMM come from dp4a over the stored words and three xor-shuffles.
// Instructions: about 13 thread-instructions per element, against 28 for the scalar kernel (ncu counters).
namespace act8 {
constexpr int kMaxPasses = 3;           // 512-column chunks per warp: 48 float2 registers per lane
constexpr int kTileRow = 144;           // bytes per transpose-tile row (16 float2 + 16 B pad)
constexpr int kTileBytes = 32 * kTileRow;
constexpr int kStageRow = 48;           // bytes per staged 16-column chunk (32 B of codes + 16 B pad)
constexpr int kStageBlock = 16 * kStageRow + 32;   // second 256-column block: banks shifted by 8
constexpr int kMaxTeamWarps = 16;
constexpr float kRound = 12582912.0f;   // 1.5 * 2^23
}  // namespace act8

__device__ __forceinline__ float2 f2_add(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 f2_sub(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "sub.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 f2_mul(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float max3_nan(float a, float b, float c) {
  float d;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float max_nan(float a, float b) {
  float d;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}

__device__ __forceinline__ void h4r_butterfly2(float2& x0, float2& x1, float2& x2, float2& x3) {
  const float2 hs = f2_mul(make_float2(0.5f, 0.5f), f2_add(f2_add(f2_add(x0, x1), x2), x3));
  const float2 y0 = f2_sub(hs, x3), y1 = f2_sub(hs, x2), y2 = f2_sub(hs, x1), y3 = f2_sub(hs, x0);
  x0 = y0; x1 = y1; x2 = y2; x3 = y3;
}

// strides 1 and 4 on the 16 register columns of a lane
__device__ __forceinline__ void stages_1_4_x2(float2 (&v)[16]) {
#pragma unroll
  for (int a = 0; a < 4; ++a) h4r_butterfly2(v[4 * a + 0], v[4 * a + 1], v[4 * a + 2], v[4 * a + 3]);
#pragma unroll
  for (int d = 0; d < 4; ++d) h4r_butterfly2(v[d], v[d + 4], v[d + 8], v[d + 12]);
}

// Lane (h, c) holds columns 16c + i (i = 0..15) of block h on entry and columns 16t + c (t = 0..15) on exit;
// then stride 16 (t digit 0) and, for ROT 256, stride 64 (t digit 1).
template <int ROT>
__device__ __forceinline__ void stages_cross_x2(float2 (&v)[16], unsigned char* tile, int lane) {
  unsigned char* wr = tile + lane * act8::kTileRow;
#pragma unroll
  for (int k = 0; k < 8; ++k)
    *reinterpret_cast<float4*>(wr + 16 * k) = make_float4(v[2 * k].x, v[2 * k].y, v[2 * k + 1].x, v[2 * k + 1].y);
  __syncwarp();
  const unsigned char* rd = tile + (lane >> 4) * 16 * act8::kTileRow + (lane & 15) * 8;
#pragma unroll
  for (int t = 0; t < 16; ++t) v[t] = *reinterpret_cast<const float2*>(rd + t * act8::kTileRow);
  __syncwarp();
#pragma unroll
  for (int a = 0; a < 4; ++a) h4r_butterfly2(v[4 * a + 0], v[4 * a + 1], v[4 * a + 2], v[4 * a + 3]);
  if (ROT == 256) {
#pragma unroll
    for (int d = 0; d < 4; ++d) h4r_butterfly2(v[d], v[d + 4], v[d + 8], v[d + 12]);
  }
}

// low bytes of four words, in order
__device__ __forceinline__ uint32_t pack_low_bytes(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  return prmt(prmt(a, b, 0x0040u), prmt(c, d, 0x0040u), 0x5410u);
}

// eight int4 codes (bytes of w0, w1 in column order) as packed nibbles, the low nibble the even column
__device__ __forceinline__ uint32_t pack_nibbles(uint32_t w0, uint32_t w1) {
  uint32_t x0 = w0 & 0x0F0F0F0Fu, x1 = w1 & 0x0F0F0F0Fu;
  x0 |= x0 >> 4;                               // bytes 0 and 2: (column 2i) | (column 2i + 1) << 4
  x1 |= x1 >> 4;
  return prmt(x0, x1, 0x6420u);
}

// One lane's 16 stored columns (512j + 256h + 16c + [0, 16)) of both rows: codes (int8 bytes, or packed int4
// nibbles with `pack`), group sums.
__device__ __forceinline__ void act8_emit(const RotQuantArgs& args, int64_t rA, bool storeB, int j, int lane,
                                          bool valid, bool pack, const uint32_t (&wa)[4], const uint32_t (&wb)[4]) {
  const int K = args.K;
  const int e0 = 512 * j + 16 * lane;          // 256h + 16c == 16 * lane
  int8_t* q = static_cast<int8_t*>(args.q);
  if (valid && pack) {
    const int64_t kh = K >> 1;
    *reinterpret_cast<uint2*>(q + rA * kh + (e0 >> 1)) = make_uint2(pack_nibbles(wa[0], wa[1]), pack_nibbles(wa[2], wa[3]));
    if (storeB)
      *reinterpret_cast<uint2*>(q + (rA + 1) * kh + (e0 >> 1)) = make_uint2(pack_nibbles(wb[0], wb[1]), pack_nibbles(wb[2], wb[3]));
  } else if (valid) {
    *reinterpret_cast<uint4*>(q + rA * K + e0) = make_uint4(wa[0], wa[1], wa[2], wa[3]);
    if (storeB) *reinterpret_cast<uint4*>(q + (rA + 1) * K + e0) = make_uint4(wb[0], wb[1], wb[2], wb[3]);
  }
  if (args.rsplit != nullptr) {
    int sa = 0, sb = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) { sa = __dp4a(static_cast<int>(wa[k]), 0x01010101, sa); sb = __dp4a(static_cast<int>(wb[k]), 0x01010101, sb); }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
      sa += __shfl_xor_sync(0xffffffffu, sa, o);
      sb += __shfl_xor_sync(0xffffffffu, sb, o);
    }
    if (valid && (lane & 7) == 0) {
      const int g = e0 >> 7, G = K >> 7;
      __nv_bfloat16* ra = args.rsplit + rA * args.rs_cols;
      const int ha = (sa >= 0 ? sa : sa - 127) / 128 * 128;   // 128 * floor(sum / 128)
      ra[g] = __float2bfloat16_rn(static_cast<float>(ha));
      ra[G + g] = __float2bfloat16_rn(static_cast<float>(sa - ha));
      if (storeB) {
        __nv_bfloat16* rb = ra + args.rs_cols;
        const int hb = (sb >= 0 ? sb : sb - 127) / 128 * 128;
        rb[g] = __float2bfloat16_rn(static_cast<float>(hb));
        rb[G + g] = __float2bfloat16_rn(static_cast<float>(sb - hb));
      }
    }
  }
}

__device__ __forceinline__ float2 f2_fma(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

// codes of one float2: round-to-nearest-even integer of the rounded product in the low byte of each word (SAFE:
// a NaN product, which only a token flagged non-finite can produce, gives code 0).  The product must be rounded
// to fp32 before the integer rounding (the reference rounds v * (1/s) first): a multiply followed by an add of
// 1.5 * 2^23 was measured to come out as one fused operation (a product just inside a half-integer then rounds
// the other way), so the add is written as an fma whose multiplier, 1.0, is a value the compiler cannot see
// (`one`, computed at run time from the kernel arguments).
template <bool SAFE>
__device__ __forceinline__ uint2 act8_code(float2 v, float2 inv, float one) {
  float2 r = f2_fma(f2_mul(v, inv), make_float2(one, one), make_float2(act8::kRound, act8::kRound));
  if (SAFE) {
    if (r.x != r.x) r.x = act8::kRound;
    if (r.y != r.y) r.y = act8::kRound;
  }
  return make_uint2(__float_as_uint(r.x), __float_as_uint(r.y));
}

template <int ROT, int PASSES, bool SAFE>
__device__ __forceinline__ void act8_quant_store(const RotQuantArgs& args, float2 (&v)[PASSES][16],
                                                 float2 inv, int64_t rA, bool storeB, int warp, int nwarps,
                                                 int nchunks, int lane, unsigned char* tile, bool pack) {
  const int K = args.K;
  const int h = lane >> 4, c = lane & 15;
  const float one = args.rows_pad > 0 ? 1.0f : 2.0f;   // 1.0 whenever the kernel runs (rows_pad > 0)
  // K-permuted position of this lane's column inside its 8-column block (0,2,4,6,1,3,5,7 order)
  const int c7 = c & 7;
  const int ip = args.kperm ? ((c7 & 1) ? 4 + (c7 >> 1) : (c7 >> 1)) : c7;
  unsigned char* st_wr = tile + h * act8::kStageBlock + 2 * ((c & 8) + ip);
  const unsigned char* st_rd = tile + h * act8::kStageBlock + c * act8::kStageRow;
#pragma unroll
  for (int s = 0; s < PASSES; ++s) {
    const int j = warp + s * nwarps;
    if (j >= nchunks) break;                                   // warp-uniform
    const bool valid = 512 * j + 256 * h < K;
    uint32_t wa[4], wb[4];
    if constexpr (ROT >= 64) {
      __syncwarp();
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        const uint2 b = act8_code<SAFE>(v[s][t], inv, one);
        const uint32_t pair = prmt(b.x, b.y, 0x0040u);         // byte 0: row A code, byte 1: row B code
        asm volatile("st.shared.b16 [%0], %1;" ::"r"(smem_u32(st_wr + t * act8::kStageRow)), "h"(static_cast<unsigned short>(pair & 0xFFFFu)) : "memory");
      }
      __syncwarp();
      const uint4 lo = *reinterpret_cast<const uint4*>(st_rd);
      const uint4 hi = *reinterpret_cast<const uint4*>(st_rd + 16);
      const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        wa[k] = prmt(w[2 * k], w[2 * k + 1], 0x6420u);
        wb[k] = prmt(w[2 * k], w[2 * k + 1], 0x7531u);
      }
    } else {
      uint32_t ca[16], cb[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) { const uint2 b = act8_code<SAFE>(v[s][i], inv, one); ca[i] = b.x; cb[i] = b.y; }
      if (args.kperm) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int o = 8 * (k >> 1) + (k & 1);
          wa[k] = pack_low_bytes(ca[o], ca[o + 2], ca[o + 4], ca[o + 6]);
          wb[k] = pack_low_bytes(cb[o], cb[o + 2], cb[o + 4], cb[o + 6]);
        }
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          wa[k] = pack_low_bytes(ca[4 * k], ca[4 * k + 1], ca[4 * k + 2], ca[4 * k + 3]);
          wb[k] = pack_low_bytes(cb[4 * k], cb[4 * k + 1], cb[4 * k + 2], cb[4 * k + 3]);
        }
      }
    }
    act8_emit(args, rA, storeB, j, lane, valid, pack, wa, wb);
  }
}

// Sum of both tokens' values over the team: warp shuffles, then one slot per warp in `slots` (2 x kMaxTeamWarps
// floats) and a CTA barrier.  `slots` must not be read by any warp still using it from an earlier call.
__device__ __forceinline__ float2 act8_team_sum(float2 t, float* slots, int lane, int warp, int nwarps) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    t.x += __shfl_xor_sync(0xffffffffu, t.x, o);
    t.y += __shfl_xor_sync(0xffffffffu, t.y, o);
  }
  if (nwarps > 1) {
    if (lane == 0) { slots[warp] = t.x; slots[act8::kMaxTeamWarps + warp] = t.y; }
    __syncthreads();
    t = make_float2(slots[0], slots[act8::kMaxTeamWarps]);
    for (int w = 1; w < nwarps; ++w) { t.x += slots[w]; t.y += slots[act8::kMaxTeamWarps + w]; }
  }
  return t;
}

__device__ __forceinline__ float2 bf16x2_round(float2 v) {
  const __nv_bfloat162 b = __floats2bfloat162_rn(v.x, v.y);
  const uint32_t u = *reinterpret_cast<const uint32_t*>(&b);
  return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xFFFF0000u));
}

template <int ROT, int PASSES, bool LNMOD, int QMAX, bool SWIGLU>
__global__ void __launch_bounds__(act8::kMaxTeamWarps * 32) act8_kernel(const RotQuantArgs args) {
  static_assert(!(LNMOD && SWIGLU), "one prologue at a time");
  // the GEMM that consumes these codes may be scheduled as soon as every CTA of this grid runs (its prologue then
  // overlaps this kernel's tail; it waits for this grid's completion before reading anything)
  grid_dep_launch();
  extern __shared__ __align__(16) unsigned char act8_smem[];
  __shared__ float red[2][act8::kMaxTeamWarps];
  __shared__ float red_ln[2][2][act8::kMaxTeamWarps];   // layer-norm prologue: sums, then centered squares
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int K = args.K;
  const int nchunks = (K + 511) >> 9;
  const int64_t rA = 2 * static_cast<int64_t>(blockIdx.x);
  const bool liveA = rA < args.rows, liveB = rA + 1 < args.rows, storeB = rA + 1 < args.rows_pad;
  unsigned char* tile = act8_smem + warp * act8::kTileBytes;
  const int h = lane >> 4;

  float2 v[PASSES][16];
  const int64_t ld = SWIGLU ? 2 * static_cast<int64_t>(K) : K;   // SwiGLU rows are [gate | up], 2K wide
  const __nv_bfloat16* xa = static_cast<const __nv_bfloat16*>(args.x) + rA * ld;
  const __nv_bfloat16* xb = xa + ld;
#pragma unroll
  for (int s = 0; s < PASSES; ++s) {
    const int j = warp + s * nwarps;
    const int e = 512 * j + 16 * lane;
    const bool valid = j < nchunks && 512 * j + 256 * h < K;
    if constexpr (SWIGLU) {
      // silu(gate) * up in fp32, rounded once to bf16 (comfy-kitchen's fused form, as in the scalar kernel)
      uint4 r[8];                                          // gate A, up A, gate B, up B: 16 bf16 each
#pragma unroll
      for (int i = 0; i < 8; ++i) r[i] = make_uint4(0, 0, 0, 0);
      if (valid && liveA) {
        r[0] = __ldg(reinterpret_cast<const uint4*>(xa + e)); r[1] = __ldg(reinterpret_cast<const uint4*>(xa + e + 8));
        r[2] = __ldg(reinterpret_cast<const uint4*>(xa + K + e)); r[3] = __ldg(reinterpret_cast<const uint4*>(xa + K + e + 8));
      }
      if (valid && liveB) {
        r[4] = __ldg(reinterpret_cast<const uint4*>(xb + e)); r[5] = __ldg(reinterpret_cast<const uint4*>(xb + e + 8));
        r[6] = __ldg(reinterpret_cast<const uint4*>(xb + K + e)); r[7] = __ldg(reinterpret_cast<const uint4*>(xb + K + e + 8));
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int q = (i >> 3), w = (i >> 1) & 3;          // uint4 and word holding column i
        auto word = [&](int k) {
          const uint4 t = r[k + q];
          return w == 0 ? t.x : (w == 1 ? t.y : (w == 2 ? t.z : t.w));
        };
        auto col = [&](uint32_t u) { return __uint_as_float((i & 1) ? (u & 0xFFFF0000u) : (u << 16)); };
        const float ga = col(word(0)), ua = col(word(2)), gb = col(word(4)), ub = col(word(6));
        v[s][i] = make_float2(swiglu_fused(ga, ua), swiglu_fused(gb, ub));
      }
      continue;
    }
    uint4 a0 = make_uint4(0, 0, 0, 0), a1 = a0, b0 = a0, b1 = a0;
    if (valid && liveA) { a0 = __ldg(reinterpret_cast<const uint4*>(xa + e)); a1 = __ldg(reinterpret_cast<const uint4*>(xa + e + 8)); }
    if (valid && liveB) { b0 = __ldg(reinterpret_cast<const uint4*>(xb + e)); b1 = __ldg(reinterpret_cast<const uint4*>(xb + e + 8)); }
    const uint32_t wa[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    const uint32_t wb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      v[s][2 * k] = make_float2(__uint_as_float(wa[k] << 16), __uint_as_float(wb[k] << 16));
      v[s][2 * k + 1] = make_float2(__uint_as_float(wa[k] & 0xFFFF0000u), __uint_as_float(wb[k] & 0xFFFF0000u));
    }
  }

  if constexpr (LNMOD) {
    // layer norm over the K columns of each token (two passes over the registers: mean, then centered squares),
    // rounded to bf16, then the modulation shift + ln * (1 + scale) rounded to bf16 (torch's layer_norm and
    // addcmul on bf16 tensors); padding tokens and columns past K stay 0
    const float inv_k = 1.0f / static_cast<float>(K);
    float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
    for (int s = 0; s < PASSES; ++s)
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[i & 3] = f2_add(acc[i & 3], v[s][i]);
    float2 sum = act8_team_sum(f2_add(f2_add(acc[0], acc[1]), f2_add(acc[2], acc[3])), &red_ln[0][0][0], lane, warp,
                               nwarps);
    const float2 mean = make_float2(sum.x * inv_k, sum.y * inv_k);
#pragma unroll
    for (int a = 0; a < 4; ++a) acc[a] = make_float2(0.f, 0.f);
#pragma unroll
    for (int s = 0; s < PASSES; ++s) {
      const int j = warp + s * nwarps;
      const bool valid = j < nchunks && 512 * j + 256 * h < K;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        v[s][i] = valid ? f2_sub(v[s][i], mean) : make_float2(0.f, 0.f);
        acc[i & 3] = f2_fma(v[s][i], v[s][i], acc[i & 3]);
      }
    }
    const float2 ssq = act8_team_sum(f2_add(f2_add(acc[0], acc[1]), f2_add(acc[2], acc[3])), &red_ln[1][0][0], lane,
                                     warp, nwarps);
    const float2 rstd = make_float2(rsqrtf(ssq.x * inv_k + args.ln_eps), rsqrtf(ssq.y * inv_k + args.ln_eps));
#pragma unroll
    for (int s = 0; s < PASSES; ++s) {
      const int j = warp + s * nwarps;
      const bool valid = j < nchunks && 512 * j + 256 * h < K;
      const int e = 512 * j + 16 * lane;
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        uint4 sh = make_uint4(0, 0, 0, 0), sc = sh;
        if (valid) {
          sh = __ldg(reinterpret_cast<const uint4*>(args.ln_shift + e + 8 * k));
          sc = __ldg(reinterpret_cast<const uint4*>(args.ln_scale1p + e + 8 * k));
        }
        const uint32_t shw[4] = {sh.x, sh.y, sh.z, sh.w}, scw[4] = {sc.x, sc.y, sc.z, sc.w};
#pragma unroll
        for (int i2 = 0; i2 < 8; ++i2) {
          const int i = 8 * k + i2;
          const uint32_t shb = (i2 & 1) ? (shw[i2 >> 1] & 0xFFFF0000u) : (shw[i2 >> 1] << 16);
          uint32_t scb = (i2 & 1) ? (scw[i2 >> 1] & 0xFFFF0000u) : (scw[i2 >> 1] << 16);
          if (args.ln_scale_plus_one)   // bf16(1 + scale): torch's `1 + scale` on a bf16 tensor
            scb = __float_as_uint(bf16_round(__fadd_rn(1.0f, __uint_as_float(scb))));
          const float2 ln = bf16x2_round(f2_mul(v[s][i], rstd));
          float2 xn = bf16x2_round(f2_fma(ln, make_float2(__uint_as_float(scb), __uint_as_float(scb)),
                                          make_float2(__uint_as_float(shb), __uint_as_float(shb))));
          if (!valid || !liveA) xn.x = 0.0f;
          if (!valid || !liveB) xn.y = 0.0f;
          v[s][i] = xn;
        }
      }
    }
  }

  if constexpr (ROT >= 16) {
#pragma unroll
    for (int s = 0; s < PASSES; ++s) stages_1_4_x2(v[s]);
  }
  if constexpr (ROT >= 64) {
#pragma unroll
    for (int s = 0; s < PASSES; ++s)
      if (warp + s * nwarps < nchunks) stages_cross_x2<ROT>(v[s], tile, lane);   // warp-uniform
  }

  // the scalar kernel's maximum: fmaxf ignores NaN; an infinity gives scale inf and reciprocal 0
  auto nan_ignoring_max = [&](float& ma, float& mb) {
    ma = 0.0f; mb = 0.0f;
#pragma unroll
    for (int s = 0; s < PASSES; ++s)
#pragma unroll
      for (int i = 0; i < 16; ++i) { ma = fmaxf(ma, fabsf(v[s][i].x)); mb = fmaxf(mb, fabsf(v[s][i].y)); }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ma = fmaxf(ma, __shfl_xor_sync(0xffffffffu, ma, o));
      mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, o));
    }
    if (nwarps > 1) {
      __syncthreads();                              // every warp has read red[] from an earlier use
      if (lane == 0) { red[0][warp] = ma; red[1][warp] = mb; }
      __syncthreads();
      ma = red[0][0]; mb = red[1][0];
      for (int w = 1; w < nwarps; ++w) { ma = fmaxf(ma, red[0][w]); mb = fmaxf(mb, red[1][w]); }
    }
  };
  float ma, mb;
  bool finite;
  if (args.amax_in != nullptr) {
    // the row's maximum and NaN flag, combined over the ranks that hold its columns
    ma = args.amax_in[rA];
    mb = storeB ? args.amax_in[rA + 1] : 0.0f;
    const bool nan_seen = args.amax_in[args.rows_pad + rA] != 0.0f || (storeB && args.amax_in[args.rows_pad + rA + 1] != 0.0f);
    finite = !nan_seen && ma <= 3.402823466e38f && mb <= 3.402823466e38f;
  } else {
    // per-token absolute maximum (NaN-propagating: a NaN or infinity anywhere makes it non-finite)
    float pa[4] = {0.0f, 0.0f, 0.0f, 0.0f}, pb[4] = {0.0f, 0.0f, 0.0f, 0.0f};   // four chains per token
#pragma unroll
    for (int s = 0; s < PASSES; ++s)
#pragma unroll
      for (int i = 0; i < 16; i += 2) {
        const int a = (i >> 1) & 3;
        pa[a] = max3_nan(pa[a], fabsf(v[s][i].x), fabsf(v[s][i + 1].x));
        pb[a] = max3_nan(pb[a], fabsf(v[s][i].y), fabsf(v[s][i + 1].y));
      }
    ma = max_nan(max3_nan(pa[0], pa[1], pa[2]), pa[3]);
    mb = max_nan(max3_nan(pb[0], pb[1], pb[2]), pb[3]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ma = max_nan(ma, __shfl_xor_sync(0xffffffffu, ma, o));
      mb = max_nan(mb, __shfl_xor_sync(0xffffffffu, mb, o));
    }
    if (nwarps > 1) {
      if (lane == 0) { red[0][warp] = ma; red[1][warp] = mb; }
      __syncthreads();
      ma = red[0][0]; mb = red[1][0];
      for (int w = 1; w < nwarps; ++w) { ma = max_nan(ma, red[0][w]); mb = max_nan(mb, red[1][w]); }
    }
    finite = ma <= 3.402823466e38f && mb <= 3.402823466e38f;   // false for NaN and infinity
    if (args.amax_out != nullptr) {
      // one rank's columns of the rows: the NaN-ignoring maximum and a NaN flag, for a maximum over the ranks
      const bool nan_a = ma != ma, nan_b = mb != mb;
      if (!finite) nan_ignoring_max(ma, mb);
      if (threadIdx.x == 0) {
        args.amax_out[rA] = liveA ? ma : 0.0f;
        args.amax_out[args.rows_pad + rA] = (liveA && nan_a) ? 1.0f : 0.0f;
        if (storeB) {
          args.amax_out[rA + 1] = liveB ? mb : 0.0f;
          args.amax_out[args.rows_pad + rA + 1] = (liveB && nan_b) ? 1.0f : 0.0f;
        }
      }
      return;
    }
    if (!finite) nan_ignoring_max(ma, mb);
  }
  // per-token scale max(absmax / QMAX, 1e-10) (QMAX 127: int8 codes; 7: int4 values held in int8 codes)
  constexpr float kInvQ = 1.0f / static_cast<float>(QMAX);
  const float sa = fmaxf(__fmul_rn(ma, kInvQ), 1e-10f), sb = fmaxf(__fmul_rn(mb, kInvQ), 1e-10f);
  const float2 inv = make_float2(__frcp_rn(sa), __frcp_rn(sb));
  if (threadIdx.x == 0) {
    float* scale = static_cast<float*>(args.scale);
    scale[rA] = liveA ? sa : 0.0f;
    if (storeB) scale[rA + 1] = liveB ? sb : 0.0f;
  }
  if (args.rsplit != nullptr) {
    const int G = K >> 7;
    for (int jj = 2 * G + threadIdx.x; jj < args.rs_cols; jj += blockDim.x) {
      args.rsplit[rA * args.rs_cols + jj] = __float2bfloat16_rn(0.0f);
      if (storeB) args.rsplit[(rA + 1) * args.rs_cols + jj] = __float2bfloat16_rn(0.0f);
    }
  }
  const bool pack = QMAX == 7 && !args.int4_as_int8;   // int4 codes as packed nibbles [rows_pad, K/2]
  if (finite) act8_quant_store<ROT, PASSES, false>(args, v, inv, rA, storeB, warp, nwarps, nchunks, lane, tile, pack);
  else act8_quant_store<ROT, PASSES, true>(args, v, inv, rA, storeB, warp, nwarps, nchunks, lane, tile, pack);
}

template <int ROT, bool LNMOD = false, int QMAX = 127, bool SWIGLU = false>
static cudaError_t launch_act8(const RotQuantArgs& a, cudaStream_t st) {
  // Three chunks per warp.  Measured on B200 at K = 3072 and 12288, M = 4096-65536: one or two chunks per warp
  // (more, smaller warps) were slower or equal, and so was a persistent variant that prefetched the next token
  // pair into shared memory (cp.async) while working on the current one.
  constexpr int kPasses = 3;
  const int nchunks = (a.K + 511) / 512;
  const int warps = (nchunks + kPasses - 1) / kPasses;
  const size_t smem = static_cast<size_t>(warps) * act8::kTileBytes;
  auto k = act8_kernel<ROT, kPasses, LNMOD, QMAX, SWIGLU>;
  if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  k<<<static_cast<unsigned>((a.rows_pad + 1) / 2), warps * 32, smem, st>>>(a);
  return cudaGetLastError();
}

static bool act8_fits(const RotQuantArgs& a) {
  return a.K % 256 == 0 && (a.K + 511) / 512 <= act8::kMaxPasses * act8::kMaxTeamWarps;
}

template <typename IN_T, int ROT, bool SWIGLU, int MODE>
static cudaError_t launch_rq(const RotQuantArgs& a, cudaStream_t st) {
  const int npairs = (a.K + 511) / 512;
  const int ppw = npairs <= kMaxWarps ? 1 : 2;
  const int warps = (npairs + ppw - 1) / ppw;
  const size_t smem = static_cast<size_t>(warps) * 528 * sizeof(float);
  if (a.rows_pad == 0) return cudaSuccess;
  if (ppw == 1) {
    auto k = rotquant_kernel<IN_T, ROT, SWIGLU, MODE, 1>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    k<<<static_cast<unsigned>(a.rows_pad), warps * 32, smem, st>>>(a);
  } else {
    auto k = rotquant_kernel<IN_T, ROT, SWIGLU, MODE, 2>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    k<<<static_cast<unsigned>(a.rows_pad), warps * 32, smem, st>>>(a);
  }
  return cudaGetLastError();
}

template <typename IN_T, bool SWIGLU, int MODE>
static cudaError_t launch_rq_rot(int rot, const RotQuantArgs& a, cudaStream_t st) {
  switch (rot) {
    case 0: return launch_rq<IN_T, 0, SWIGLU, MODE>(a, st);
    case 16: return launch_rq<IN_T, 16, SWIGLU, MODE>(a, st);
    case 64: return launch_rq<IN_T, 64, SWIGLU, MODE>(a, st);
    default: return launch_rq<IN_T, 256, SWIGLU, MODE>(a, st);
  }
}

template <int QMAX, bool SWIGLU>
static cudaError_t launch_act8_rot(int rot, const RotQuantArgs& a, cudaStream_t st) {
  switch (rot) {
    case 0: return launch_act8<0, false, QMAX, SWIGLU>(a, st);
    case 16: return launch_act8<16, false, QMAX, SWIGLU>(a, st);
    case 64: return launch_act8<64, false, QMAX, SWIGLU>(a, st);
    default: return launch_act8<256, false, QMAX, SWIGLU>(a, st);
  }
}

cudaError_t launch_act_rotquant(int rot, bool swiglu, int mode, const RotQuantArgs& a, cudaStream_t st) {
  if (swiglu) {
    // per-token modes on the two-token kernel; the per-group mode (fp32 product) stays on the scalar kernel
    if ((mode == MODE_ACT_INT8_ROW || mode == MODE_ACT_INT4_ROW) && act8_fits(a)) {
      if (a.rows_pad == 0) return cudaSuccess;
      return mode == MODE_ACT_INT8_ROW ? launch_act8_rot<127, true>(rot, a, st) : launch_act8_rot<7, true>(rot, a, st);
    }
    if (mode == MODE_ACT_INT8_ROW) return launch_rq_rot<__nv_bfloat16, true, MODE_ACT_INT8_ROW>(rot, a, st);
    if (mode == MODE_ACT_INT4_ROW) return launch_rq_rot<__nv_bfloat16, true, MODE_ACT_INT4_ROW>(rot, a, st);
    return launch_rq_rot<__nv_bfloat16, true, MODE_ACT_INT4_GROUP>(rot, a, st);
  }
  if (mode == MODE_ACT_INT8_ROW) {
    if (a.rows_pad == 0) return cudaSuccess;
    if (a.ln_shift != nullptr) {                    // modulated layer norm prologue (callers check act8_fits)
      if (!act8_fits(a)) return cudaErrorInvalidValue;
      switch (rot) {
        case 0: return launch_act8<0, true>(a, st);
        case 16: return launch_act8<16, true>(a, st);
        case 64: return launch_act8<64, true>(a, st);
        default: return launch_act8<256, true>(a, st);
      }
    }
    if (act8_fits(a)) return launch_act8_rot<127, false>(rot, a, st);
    return launch_rq_rot<__nv_bfloat16, false, MODE_ACT_INT8_ROW>(rot, a, st);
  }
  if (mode == MODE_ACT_INT4_ROW) {
    if (a.rows_pad == 0) return cudaSuccess;
    if (a.ln_shift != nullptr) {                    // modulated layer norm prologue (callers check act8_fits)
      if (!act8_fits(a)) return cudaErrorInvalidValue;
      switch (rot) {
        case 0: return launch_act8<0, true, 7>(a, st);
        case 16: return launch_act8<16, true, 7>(a, st);
        case 64: return launch_act8<64, true, 7>(a, st);
        default: return launch_act8<256, true, 7>(a, st);
      }
    }
    // int4 values as int8 codes (the W4A4 GEMM's operand) or as packed nibbles (the reference's format)
    if (act8_fits(a)) return launch_act8_rot<7, false>(rot, a, st);
    return launch_rq_rot<__nv_bfloat16, false, MODE_ACT_INT4_ROW>(rot, a, st);
  }
  return launch_rq_rot<__nv_bfloat16, false, MODE_ACT_INT4_GROUP>(rot, a, st);
}

template <typename IN_T>
static cudaError_t launch_w(int rot, int mode, const RotQuantArgs& a, cudaStream_t st) {
  switch (mode) {
    case MODE_W_INT4_ROW: return launch_rq_rot<IN_T, false, MODE_W_INT4_ROW>(rot, a, st);
    case MODE_W_INT8_ROW: return launch_rq_rot<IN_T, false, MODE_W_INT8_ROW>(rot, a, st);
    case MODE_W_AFFINE: return launch_rq_rot<IN_T, false, MODE_W_AFFINE>(rot, a, st);
    default: return launch_rq_rot<IN_T, false, MODE_W_INT4_GROUP_BF16UP>(rot, a, st);
  }
}

cudaError_t launch_weight_rotquant(int rot, bool w_bf16, int mode, const RotQuantArgs& a, cudaStream_t st) {
  return w_bf16 ? launch_w<__nv_bfloat16>(rot, mode, a, st) : launch_w<float>(rot, mode, a, st);
}

// ---- int4 -> int8 unpack (signed nibbles, low nibble = even column) ----
__global__ void unpack_int4_kernel(const uint8_t* __restrict__ src, int8_t* __restrict__ dst, int64_t n_bytes) {
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  if (i >= n_bytes) return;
  const uint2 w = *reinterpret_cast<const uint2*>(src + i);
  const uint32_t ws[2] = {w.x, w.y};
  uint32_t o[4];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    // nibble -> byte holding 16*v, then an arithmetic shift back per byte
    const uint32_t lo = (ws[h] << 4) & 0xF0F0F0F0u;
    const uint32_t hi = ws[h] & 0xF0F0F0F0u;
    const uint32_t a = prmt(lo, hi, 0x5140u), b = prmt(lo, hi, 0x7362u);
    uint32_t ra = 0, rb = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      ra |= (static_cast<uint32_t>(static_cast<int8_t>((a >> (8 * k)) & 0xFFu) >> 4) & 0xFFu) << (8 * k);
      rb |= (static_cast<uint32_t>(static_cast<int8_t>((b >> (8 * k)) & 0xFFu) >> 4) & 0xFFu) << (8 * k);
    }
    o[2 * h] = ra; o[2 * h + 1] = rb;
  }
  *reinterpret_cast<uint4*>(dst + 2 * i) = make_uint4(o[0], o[1], o[2], o[3]);
}

cudaError_t launch_unpack_int4(const void* src, int64_t n_bytes, void* dst, cudaStream_t st) {
  if (n_bytes == 0) return cudaSuccess;
  const int64_t threads = (n_bytes + 7) / 8;
  unpack_int4_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, st>>>(
      static_cast<const uint8_t*>(src), static_cast<int8_t*>(dst), n_bytes);
  return cudaGetLastError();
}

}  // namespace cq
