// DiT-step glue kernels, sm_100a: the work between the quantized linears of a dual-stream MMDiT block that would
// otherwise run as several torch kernels with bf16 round trips through HBM.
//
// qkv_rmsnorm_rope_kernel: one token's QKV linear output y [3, H, D] (bf16) ->
//   q = rope(rmsnorm(y[0]) * w_q), k = rope(rmsnorm(y[1]) * w_k), v = y[2], each written at token s0 + s of the
//   joint attention layout, head-major [H, S_all, D] or token-major [S_all, H, D] (batch 1; the token-major form is
//   the [tokens, hidden] layout an attention kernel given strided views reads and writes back in place).  RMSNorm per head in fp32 (x * rsqrt(mean(x^2) + eps) * w,
//   rounded once to bf16, as torch's fused rms_norm does); the rotary rotation acts on interleaved pairs
//   (x[2p], x[2p+1]) with (cos, sin) of the token's position, in fp32 on the bf16 normalized values, rounded to
//   bf16.  It replaces, per stream and block, rms_norm + float copy + complex multiply + bf16 copy + the
//   transposing copies of q, k and v.
#include "kernels.cuh"

namespace cq {

template <int D>
__global__ void __launch_bounds__(256) qkv_rmsnorm_rope_kernel(const QkvRopeArgs a) {
  constexpr int E = D / 32;                       // elements per lane: 2 or 4 (whole rotary pairs)
  static_assert(E == 2 || E == 4, "head dim 64 or 128");
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int64_t s = blockIdx.x;
  const int part = blockIdx.y;                    // 0: q, 1: k, 2: v
  const int H = a.H;
  const __nv_bfloat16* src = a.y + (s * 3 + part) * static_cast<int64_t>(H) * D + lane * E;
  __nv_bfloat16* dst = (part == 0 ? a.q : part == 1 ? a.k : a.v) + (a.s0 + s) * a.tok_stride + lane * E;
  const int64_t head_stride = a.head_stride;

  float w[E], cs[E / 2], sn[E / 2];
  if (part < 2) {
    const __nv_bfloat16* wp = (part == 0 ? a.qw : a.kw) + lane * E;
#pragma unroll
    for (int i = 0; i < E; ++i) w[i] = __bfloat162float(wp[i]);
    const float* rp = a.rope + (s * (D / 2) + lane * (E / 2)) * 2;
#pragma unroll
    for (int p = 0; p < E / 2; ++p) { cs[p] = rp[2 * p]; sn[p] = rp[2 * p + 1]; }
  }
  for (int h = warp; h < H; h += nwarps) {
    const __nv_bfloat16* xp = src + static_cast<int64_t>(h) * D;
    uint32_t raw[E / 2];
    if constexpr (E == 4) {
      const uint2 r = *reinterpret_cast<const uint2*>(xp);
      raw[0] = r.x; raw[1] = r.y;
    } else {
      raw[0] = *reinterpret_cast<const uint32_t*>(xp);
    }
    __nv_bfloat16* op = dst + h * head_stride;
    if (part == 2) {
      if constexpr (E == 4) *reinterpret_cast<uint2*>(op) = make_uint2(raw[0], raw[1]);
      else *reinterpret_cast<uint32_t*>(op) = raw[0];
      continue;
    }
    float x[E];
#pragma unroll
    for (int p = 0; p < E / 2; ++p) { x[2 * p] = bf16_bits_to_f32(raw[p] & 0xFFFFu); x[2 * p + 1] = bf16_bits_to_f32(raw[p] >> 16); }
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < E; ++i) ss = fmaf(x[i], x[i], ss);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float r = rsqrtf(ss / static_cast<float>(D) + a.eps);
    uint32_t out[E / 2];
#pragma unroll
    for (int p = 0; p < E / 2; ++p) {
      const float x0 = bf16_round(x[2 * p] * r * w[2 * p]), x1 = bf16_round(x[2 * p + 1] * r * w[2 * p + 1]);
      const float y0 = x0 * cs[p] - x1 * sn[p], y1 = x0 * sn[p] + x1 * cs[p];
      const __nv_bfloat162 b = __floats2bfloat162_rn(y0, y1);
      out[p] = *reinterpret_cast<const uint32_t*>(&b);
    }
    if constexpr (E == 4) *reinterpret_cast<uint2*>(op) = make_uint2(out[0], out[1]);
    else *reinterpret_cast<uint32_t*>(op) = out[0];
  }
}

cudaError_t launch_qkv_rmsnorm_rope(const QkvRopeArgs& a, cudaStream_t st) {
  if (a.S == 0) return cudaSuccess;
  const dim3 grid(static_cast<unsigned>(a.S), 3);
  const int threads = 32 * (a.H < 8 ? a.H : 8);
  if (a.D == 128) qkv_rmsnorm_rope_kernel<128><<<grid, threads, 0, st>>>(a);
  else qkv_rmsnorm_rope_kernel<64><<<grid, threads, 0, st>>>(a);
  return cudaGetLastError();
}

// heads_to_rows_kernel: attention output o [Hp, S, D] (this rank's Hp heads, bf16) -> rows of [S, ldo] at columns
// col0 + h*D + [0, D), written into every buffer of outs (the head-parallel attention's gather: peer buffers of a
// symmetric allocation, or one local buffer, where it replaces the transposing copy to the [tokens, hidden] layout).
// One CTA per token, 16 bytes per thread, plain stores.
__global__ void __launch_bounds__(1024) heads_to_rows_kernel(const HeadsToRowsArgs a) {
  const int64_t s = blockIdx.x;
  const int per_head = a.D / 8;
  const int h = threadIdx.x / per_head, c8 = threadIdx.x - h * per_head;
  const uint4 v = *reinterpret_cast<const uint4*>(a.src + (static_cast<int64_t>(h) * a.S + s) * a.D + 8 * c8);
  const int64_t off = s * a.ldo + a.col0 + static_cast<int64_t>(h) * a.D + 8 * c8;
  for (int i = 0; i < a.n_out; ++i) *reinterpret_cast<uint4*>(a.outs[i] + off) = v;
}

cudaError_t launch_heads_to_rows(const HeadsToRowsArgs& a, cudaStream_t st) {
  if (a.S == 0) return cudaSuccess;
  heads_to_rows_kernel<<<static_cast<unsigned>(a.S), a.Hp * a.D / 8, 0, st>>>(a);
  return cudaGetLastError();
}

// rmsnorm_rope_rows_kernel: one token's row x [C] (bf16) -> out = rope(bf16(x * rsqrt(mean(x^2) + eps) * w)), the
// RMSNorm over the whole row in fp32 with one bf16 rounding (torch's fused rms_norm on a bf16 row), then, with a
// rope table, each D-wide head's interleaved pairs (x[2p], x[2p+1]) rotated by (cos, sin) of the token's position in
// fp32 and rounded to bf16 (the float copy + complex multiply + bf16 copy it replaces).  One CTA per token; each
// thread holds `chunks` 16-byte chunks of the row in registers across the CTA's sum, so out may be x.
__global__ void __launch_bounds__(512) rmsnorm_rope_rows_kernel(const RmsRopeArgs a) {
  constexpr int kMaxChunks = 4;
  __shared__ float red[16];
  const int64_t s = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = (blockDim.x + 31) >> 5;
  const int nchunk = a.C >> 3;
  const __nv_bfloat16* xr = a.x + s * a.C;
  uint4 raw[kMaxChunks];
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < kMaxChunks; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    raw[i] = make_uint4(0, 0, 0, 0);
    if (i < a.chunks && c < nchunk) raw[i] = *reinterpret_cast<const uint4*>(xr + 8 * c);
    const uint32_t wv[4] = {raw[i].x, raw[i].y, raw[i].z, raw[i].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float lo = bf16_bits_to_f32(wv[j] & 0xFFFFu), hi = bf16_bits_to_f32(wv[j] >> 16);
      ss = fmaf(lo, lo, ss);
      ss = fmaf(hi, hi, ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = 0.0f;
  for (int w = 0; w < nwarps; ++w) tot += red[w];
  const float r = rsqrtf(tot / static_cast<float>(a.C) + a.eps);
  const float* rp = a.rope != nullptr ? a.rope + s * (a.D / 2) * 2 : nullptr;
#pragma unroll
  for (int i = 0; i < kMaxChunks; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (i >= a.chunks || c >= nchunk) break;
    const uint4 wq = *reinterpret_cast<const uint4*>(a.w + 8 * c);
    const uint32_t xv[4] = {raw[i].x, raw[i].y, raw[i].z, raw[i].w};
    const uint32_t wv[4] = {wq.x, wq.y, wq.z, wq.w};
    uint32_t ov[4];
    const int p0 = ((8 * c) % a.D) >> 1;   // first rotary pair of the chunk inside its head
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float x0 = bf16_round(bf16_bits_to_f32(xv[j] & 0xFFFFu) * r * bf16_bits_to_f32(wv[j] & 0xFFFFu));
      float x1 = bf16_round(bf16_bits_to_f32(xv[j] >> 16) * r * bf16_bits_to_f32(wv[j] >> 16));
      if (rp != nullptr) {
        const float2 cs = *reinterpret_cast<const float2*>(rp + 2 * (p0 + j));
        const float y0 = x0 * cs.x - x1 * cs.y, y1 = x0 * cs.y + x1 * cs.x;
        x0 = y0;
        x1 = y1;
      }
      const __nv_bfloat162 b2 = __floats2bfloat162_rn(x0, x1);
      ov[j] = *reinterpret_cast<const uint32_t*>(&b2);
    }
    *reinterpret_cast<uint4*>(a.out + s * a.C + 8 * c) = make_uint4(ov[0], ov[1], ov[2], ov[3]);
  }
}

cudaError_t launch_rmsnorm_rope_rows(const RmsRopeArgs& a, cudaStream_t st) {
  if (a.S == 0) return cudaSuccess;
  const int nchunk = a.C / 8;
  RmsRopeArgs b = a;
  b.chunks = (nchunk + 511) / 512;
  const int threads = ((nchunk + b.chunks - 1) / b.chunks + 31) / 32 * 32;
  rmsnorm_rope_rows_kernel<<<static_cast<unsigned>(a.S), threads, 0, st>>>(b);
  return cudaGetLastError();
}

}  // namespace cq
