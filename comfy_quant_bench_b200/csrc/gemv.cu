// Small-M W4A8 affine product: the W4A8 linear for M <= 8 tokens (adaLN modulation and other one-token products).
//
// The tensor-core GEMM runs whole 256-token tiles, so a one-token product pays for 256 tokens of MMA and drain; at
// M <= 8 the product is bound by reading the packed weights once.  One warp per four weight rows: lane l reads the
// rows' 16-byte chunks l, l + 32, ... (32 K columns each, a quarter of a 128-wide group) and every token's 32
// matching int8 codes once for the four rows, in the K-permuted order the activation kernel stores (0,2,4,6,1,3,5,7
// inside each 8-column block), so a packed word's low nibbles meet one activation word and its high nibbles the
// next.
//
// Per token and group: P = sum x (q - 8) = dp4a(q, x) - 8 R with R = sum x (exact int32), then the group adds
// s[g, n] P + z[g, n] R in fp32; the lane partials are summed by a fixed shuffle tree (deterministic), and the
// output is bf16(acc * sx[m] + bias[n]) as in the GEMM's epilogue.  The fp32 summation order differs from the
// tensor-core GEMM's, so the two paths agree to fp32 rounding, not bit for bit.
#include "kernels.cuh"

namespace cq {

namespace gemv {
constexpr int kWarps = 8;
constexpr int kRowsPerWarp = 4;  // rows share each chunk's activation loads and group sums
constexpr int kMaxTokens = 8;
}  // namespace gemv

// sum of the four products of unsigned bytes of a and signed bytes of b, plus c
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

struct GemvArgs {
  const int8_t* a;               // [>= M, K] int8 codes, K-permuted
  const float* sa;               // [M]
  const uint8_t* b;              // [N, K/2] packed uint4, low nibble = even column
  const __nv_bfloat16* s;        // [K/128, N]
  const __nv_bfloat16* zt;       // [N, zt_cols]: zt[n, g] = z[g, n] for g < K/128
  const __nv_bfloat16* bias;     // [N] or null
  __nv_bfloat16* out;            // [M, N]
  int M, N, K, zt_cols;
};

template <int MT>
__global__ void __launch_bounds__(gemv::kWarps * 32) gemv_affine_kernel(const GemvArgs args) {
  constexpr int R = gemv::kRowsPerWarp;
  const int lane = threadIdx.x & 31;
  const int n0 = (blockIdx.x * gemv::kWarps + (threadIdx.x >> 5)) * R;
  if (n0 >= args.N) return;                                  // warp-uniform
  const int K = args.K, M = args.M;
  const int nchunks = K >> 5;                                // 32-column chunks (16 packed bytes)
  const bool leader = (lane & 3) == 0;                       // one lane per group adds the group's terms
  bool row_ok[R];
#pragma unroll
  for (int r = 0; r < R; ++r) row_ok[r] = n0 + r < args.N;
  float part[R][MT];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < MT; ++m) part[r][m] = 0.0f;

  // every lane runs every iteration (the shuffles below name the whole warp); chunks past the row are skipped.
  // nchunks is a multiple of 4, so the four lanes of a group are all inside the row or all past it.
  // one or two tokens: two iterations' weight loads in flight; more tokens need the registers
  constexpr int kUnroll = MT <= 2 ? 2 : 1;
  // the group leaders' weight scales and zeros (raw bf16 bits) are loaded one iteration ahead, so no iteration
  // waits for a dependent load after its shuffles
  unsigned short s_next[R], z_next[R];
  auto load_sz = [&](int c0, unsigned short (&sv)[R], unsigned short (&zv)[R]) {
    const int c = c0 + lane;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      sv[r] = 0;
      zv[r] = 0;
      if (leader && c < nchunks && row_ok[r]) {
        const int g = c >> 2, n = n0 + r;
        sv[r] = __ldg(reinterpret_cast<const unsigned short*>(args.s) + static_cast<int64_t>(g) * args.N + n);
        zv[r] = __ldg(reinterpret_cast<const unsigned short*>(args.zt) + static_cast<int64_t>(n) * args.zt_cols + g);
      }
    }
  };
  // the packed weights are loaded one iteration ahead as well
  uint4 w_next[R];
  auto load_w = [&](int c0, uint4 (&wv)[R]) {
    const int c = c0 + lane;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      wv[r] = make_uint4(0, 0, 0, 0);
      if (c < nchunks && row_ok[r])
        wv[r] = __ldg(reinterpret_cast<const uint4*>(args.b + static_cast<int64_t>(n0 + r) * (K >> 1) +
                                                     16 * static_cast<int64_t>(c)));
    }
  };
  // Weights, scales and zeros are not written by the activation kernel this product follows: their first loads are
  // issued before waiting for it (a programmatic launch of the fused linear), the activation codes only after.
  load_w(0, w_next);
  load_sz(0, s_next, z_next);
  grid_dep_wait();
#pragma unroll kUnroll
  for (int c0 = 0; c0 < nchunks; c0 += 32) {
    const int c = c0 + lane;
    const bool valid = c < nchunks;
    unsigned short s_cur[R], z_cur[R];
    uint4 wq[R];
#pragma unroll
    for (int r = 0; r < R; ++r) { s_cur[r] = s_next[r]; z_cur[r] = z_next[r]; wq[r] = w_next[r]; }
    // one or two tokens: the next iteration's weights in flight during this one (measured faster); more tokens
    // need the registers, so their next weights are loaded after this iteration's products
    constexpr bool kAhead = MT <= 2;
    if (c0 + 32 < nchunks) {
      if (kAhead) load_w(c0 + 32, w_next);
      load_sz(c0 + 32, s_next, z_next);
    }
    int pm[R][MT], rm[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      rm[m] = 0;
#pragma unroll
      for (int r = 0; r < R; ++r) pm[r][m] = 0;
      if (valid && m < M) {
        // this token's 32 codes of the chunk, shared by the warp's R rows
        const int8_t* xr = args.a + static_cast<int64_t>(m) * K + 32 * c;
        const uint4 x0 = __ldg(reinterpret_cast<const uint4*>(xr));
        const uint4 x1 = __ldg(reinterpret_cast<const uint4*>(xr + 16));
        const uint32_t x[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
        int rs = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) rs = __dp4a(static_cast<int>(x[j]), 0x01010101, rs);
        rm[m] = rs;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const uint32_t w[4] = {wq[r].x, wq[r].y, wq[r].z, wq[r].w};
          int p = 0;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            p = dp4a_us(w[k] & 0x0F0F0F0Fu, x[2 * k], p);           // even columns of the 8-column block
            p = dp4a_us((w[k] >> 4) & 0x0F0F0F0Fu, x[2 * k + 1], p);  // odd columns
          }
          pm[r][m] = p - 8 * rs;                             // sum x (q - 8) over the chunk
        }
      }
    }
    if (!kAhead && c0 + 32 < nchunks) load_w(c0 + 32, w_next);
    // the four lanes of a group (chunks 4g .. 4g + 3 sit in lanes 4j .. 4j + 3) sum their chunks
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      rm[m] += __shfl_xor_sync(0xffffffffu, rm[m], 1);
      rm[m] += __shfl_xor_sync(0xffffffffu, rm[m], 2);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        pm[r][m] += __shfl_xor_sync(0xffffffffu, pm[r][m], 1);
        pm[r][m] += __shfl_xor_sync(0xffffffffu, pm[r][m], 2);
      }
    }
    if (leader && valid) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        if (!row_ok[r]) continue;
        const float sg = bf16_bits_to_f32(s_cur[r]);
        const float zg = bf16_bits_to_f32(z_cur[r]);
#pragma unroll
        for (int m = 0; m < MT; ++m)
          part[r][m] = __fmaf_rn(zg, __int2float_rn(rm[m]), __fmaf_rn(sg, __int2float_rn(pm[r][m]), part[r][m]));
      }
    }
  }
  // lane partials -> one sum per row and token (fixed tree: deterministic); lane r * MT + m writes (n0 + r, m)
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < MT; ++m) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) part[r][m] += __shfl_xor_sync(0xffffffffu, part[r][m], o);
      if (lane == (r * MT + m) % 32 && m < M && row_ok[r]) {
        const int n = n0 + r;
        const float bias = args.bias != nullptr ? __bfloat162float(args.bias[n]) : 0.0f;
        args.out[static_cast<int64_t>(m) * args.N + n] = __float2bfloat16_rn(__fmaf_rn(part[r][m], args.sa[m], bias));
      }
    }
}

bool gemv_affine_fits(int M, int a_kperm) { return M >= 1 && M <= gemv::kMaxTokens && a_kperm != 0; }

// pdl: launch as a programmatic dependent of the previous kernel in the stream (the fused linears, whose previous
// kernel is their own activation kernel): the weight stream starts under that kernel's tail
cudaError_t launch_gemv_affine(const int8_t* a, const float* sa, const void* b, const void* s, const void* zt,
                               const void* bias, void* out, int M, int N, int K, cudaStream_t st, bool pdl) {
  const GemvArgs g{a, sa, static_cast<const uint8_t*>(b), static_cast<const __nv_bfloat16*>(s),
                   static_cast<const __nv_bfloat16*>(zt), static_cast<const __nv_bfloat16*>(bias),
                   static_cast<__nv_bfloat16*>(out), M, N, K, rsplit_cols(K)};
  constexpr int kRowsPerCta = gemv::kWarps * gemv::kRowsPerWarp;
  auto kern = M <= 1 ? gemv_affine_kernel<1> : M <= 2 ? gemv_affine_kernel<2> : M <= 4 ? gemv_affine_kernel<4>
                                                                                          : gemv_affine_kernel<8>;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(static_cast<unsigned>((N + kRowsPerCta - 1) / kRowsPerCta));
  cfg.blockDim = dim3(gemv::kWarps * 32);
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (cudaLaunchKernelEx(&cfg, kern, g) != cudaSuccess) return cudaErrorLaunchFailure;
  return cudaGetLastError();
}

}  // namespace cq
