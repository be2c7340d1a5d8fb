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
  constexpr bool IS_WEIGHT = MODE >= 10;
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
          const float sv = __fmul_rn(__fdiv_rn(g[i], __fadd_rn(1.0f, expf(-g[i]))), u[i]);
          // comfy-kitchen's fused quantizer rounds the product once to bf16; the per-group quantizer keeps fp32
          v[s][i] = (MODE == MODE_ACT_INT4_GROUP) ? sv : bf16_round(sv);
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

cudaError_t launch_act_rotquant(int rot, bool swiglu, int mode, const RotQuantArgs& a, cudaStream_t st) {
  if (swiglu) {
    if (mode == MODE_ACT_INT8_ROW) return launch_rq_rot<__nv_bfloat16, true, MODE_ACT_INT8_ROW>(rot, a, st);
    if (mode == MODE_ACT_INT4_ROW) return launch_rq_rot<__nv_bfloat16, true, MODE_ACT_INT4_ROW>(rot, a, st);
    return launch_rq_rot<__nv_bfloat16, true, MODE_ACT_INT4_GROUP>(rot, a, st);
  }
  if (mode == MODE_ACT_INT8_ROW) return launch_rq_rot<__nv_bfloat16, false, MODE_ACT_INT8_ROW>(rot, a, st);
  if (mode == MODE_ACT_INT4_ROW) return launch_rq_rot<__nv_bfloat16, false, MODE_ACT_INT4_ROW>(rot, a, st);
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
