// Packed-int4-weight x int8-activation GEMM with fused dequant epilogue, sm_100a (tcgen05 kind::i8).
//
// Orientation: the MMA computes D[n, m] = sum_k W[n, k] * X[m, k] with the WEIGHT tile on the tensor core's
// M side (128 weight rows = the 128 TMEM lanes) and 256 tokens on its N side (TMEM columns).  Each epilogue
// thread therefore owns one weight row n: the per-group weight scale s[g, n] and zero z[g, n] are per-thread
// scalars, and only the per-token terms (activation scale, code sums) are broadcast loads.
//
// Per CTA (persistent, one per SM, 512 threads):
//   warp 0      TMA producer: activation tile [256 tokens x 128 B] (128-byte swizzle) and the packed weight
//               tile [128 rows x 64 B] per 128-wide K block, into a 4-stage ring;
//   warps 2-7   converters: unpack int4 -> int8 from the TMA ring into a 3-stage ring laid out as the tensor
//               core's K-major 128-byte-swizzled operand (nibble v becomes the byte 16*v, the 1/16 is folded
//               into the weight scale; with K-permuted activations each 32-bit word unpacks with one shift and
//               two masks, no byte shuffles), 16 packed bytes per item, then fence.proxy.async and arrive.
//               Each pair of converter warps owns one converter stage and takes every third K block, so three
//               blocks are converted at once;
//   warp 1      MMA issuer: 4 x tcgen05.mma (128 x 256 x 32) per K block into a double-buffered TMEM
//               accumulator (2 x 256 columns); tcgen05.commit releases both rings and hands buffers over;
//   warps 8-15  epilogue: tcgen05.ld the int32 partial sums.  Affine weights (per 128-group scale/zero) drain
//               every group into fp32 registers, acc += s[g,n] * float(P_g) (the exact int32 -> fp32 conversion
//               runs on the integer pipe, the packed f32x2 FMA on the FMA pipe, side by side), starting from the
//               zero-point term sum_g z[g,n] * R[g,m] that the tensor core computes first (kind::f16: the bf16
//               zeros, built by the converters, times the tokens' code sums split exactly into bf16 hi/lo parts);
//               each group's first MMA overwrites the buffer, so the drain only reads TMEM (no re-seeding
//               stores), and a buffer goes back to the MMA as soon as its last chunk is in registers.
//               Row/col weights drain once per tile.  Output bf16 [M, N] row-major.
// int8 weights (W8A8) skip the converters: TMA loads them straight into the operand layout.
// Every mbarrier wait is bounded (see cq_common.cuh).  No cluster launch, no multicast.
#include <cstdio>
#include <type_traits>
#include <cstring>

#include "kernels.cuh"

namespace cq {

constexpr int kBW = 128;       // weight rows per tile (MMA M, TMEM lanes)
constexpr int kBT = 256;       // tokens per tile (MMA N, TMEM columns per accumulator buffer; 128 also builds and
                               // passes the tests, but measured ~40 % slower)
constexpr int kNumBufs = 512 / kBT;    // accumulator buffers in the 512 TMEM columns
constexpr int kWarpTok = kBT / 2;      // tokens per epilogue warp (two warps per TMEM lane quadrant)
constexpr int kChunks = kWarpTok / 32; // 32-column TMEM loads per epilogue warp per drain
constexpr int kBK = 128;       // K elements (bytes of int8) per stage
constexpr int kConvStages = 3;
constexpr int kThreads = 512;
constexpr int kConvWarps = 6;          // warps 2..7, one pair per converter stage
static_assert(kConvWarps == 2 * kConvStages, "one pair of converter warps per converter stage");
constexpr int kEpiWarp0 = 8;           // warps 8..15
constexpr int kMaxOutMaps = kMaxOutBuffers;   // affine: output buffers one launch writes (column-parallel)
constexpr int kXBytes = kBT * kBK;          // 32 KB
constexpr int kWuBytes = kBW * kBK;         // 16 KB (unpacked int4, or TMA-loaded int8 weights)
constexpr int kWpBytes = kBW * kBK / 2;     //  8 KB (packed int4)
constexpr int kProducerRegs = 40;    // warps 0-7 (producer, MMA, converters)
constexpr int kEpilogueRegs = 216;   // warps 8-15; 256*40 + 256*216 = 128*512, the launch allocation

// ROWCOL: per-token x per-row scales once per tile (the reference's policy 0); AFFINE: per-group weight scale and
// zero, per-token activation scale; GROUP: per-group scales on both sides (the reference's policy 4, CTA-pair kernel);
// INTRATIO: integer weight ratios per 64- or 128-wide group summed in int32, then per-token x per-row scales (the
// reference's policies 5/7/15/17, CTA-pair kernel)
enum : int { EPI_ROWCOL = 0, EPI_AFFINE = 1, EPI_GROUP = 2, EPI_INTRATIO = 3 };
enum : int { BF_S4 = 0, BF_U4 = 1, BF_S8 = 2 };

// shared-memory plan per epilogue and weight format.  The affine kernel trades one TMA stage for the output
// staging buffers of its asynchronous (TMA) output stores.
template <int EPI, int BFMT, bool GLU = false>
struct SmemPlan {
  // TMA ring depth
  static constexpr int kStages = (EPI == EPI_AFFINE) ? (kBT == 256 ? 3 : 4) : (kBT == 256 ? 4 : 6);
  static constexpr int kWStageBytes = (BFMT == BF_S8) ? kWuBytes : kWpBytes;   // weight bytes in the TMA ring
  static constexpr int kTmaStageBytes = kXBytes + kWStageBytes;
  static constexpr int kConvBytes = (BFMT == BF_S8) ? 0 : kConvStages * kWuBytes;
  static constexpr int kData = kStages * kTmaStageBytes + kConvBytes;
  static constexpr int kSaStage = kData + 512;                    // after the barriers: per-token scales
  static constexpr int kSaBytes = 8 * kWarpTok * 4;               // kWarpTok fp32 per epilogue warp
  static constexpr int kOutStage = kSaStage + kSaBytes;           // output staging: 64 tokens x 32 columns bf16
  static constexpr int kOutWarpBytes = 64 * 32 * 2;               //   per epilogue warp (affine only)
  static constexpr int kOutBytes = (EPI == EPI_AFFINE) ? 8 * kOutWarpBytes : 0;
  static constexpr int kBytes = kOutStage + kOutBytes + 1024 /*align slack*/;
};

// Output tensor maps of the affine epilogue: map i covers buffer i ([M, ldo] bf16); every staged output box is
// stored to each of the first n_out maps at column out_col0 + its tile column.
struct OutMaps {
  CUtensorMap m[kMaxOutMaps];
};

struct GemmArgs {
  const float* sa;       // [M] activation scale (rowcol, affine)
  const float* sbg;      // [K/128, N] f32 per-group weight scale (group)
  int64_t sag_ld;        // group: row stride (elements) of the tokens' per-group scales [K/128, sag_ld] f32
  const float* sb;       // [N] weight scale (rowcol)
  const __nv_bfloat16* ws;  // [K/128, N] bf16 (affine)
  const __nv_bfloat16* zt;  // [N, 64*nz] bf16 (affine): Zt[n, j] = z[j mod G, n] for j < 2G, else 0
  const __nv_bfloat16* bias;  // [N] or null
  __nv_bfloat16* out;    // [M, N]
  int M, N, K;
  int nz;                // affine: zero-point pseudo blocks per tile (64 bf16 columns of the split sums each)
  int tma_out;           // affine: outputs leave through the TMA store maps (N % 8 == 0, 16-byte aligned out)
  int n_out;             // affine with tma_out: number of output maps (1, or the ranks of a column-parallel layer)
  int out_col0;          // affine with tma_out: column of the output maps where this launch's N columns start
  int split;             // row/col epilogue: the last `split` tiles of the tile order run as two 128-token half
                         // tiles each (a partial last wave of at most half the CTAs finishes in half a tile's time)
  int out_w64;           // affine with tma_out: two epilogue warps (adjacent lane quadrants) share one 64-column
                         // box per pass (128-byte rows) instead of one 32-column box each (N % 64 == 0)
  int out_op;            // affine: OUT_PLAIN / OUT_GELU / OUT_GATED, applied to the bf16 result before the store
  int64_t res_ld;        // OUT_GATED: row stride (elements) of res
  const __nv_bfloat16* res;   // OUT_GATED: residual [M, res_ld] (may be `out` itself)
  const __nv_bfloat16* gate;  // OUT_GATED: per-column gate [N]
  const void* cw;        // intratio: integer weight ratios [K/cw_group, N], int32 or uint8
  int cw_u8;             // intratio: cw holds uint8 (policies 15/17) instead of int32 (5/7)
  int cw_group;          // intratio: 64 or 128 K columns per ratio
  int ksplit;            // affine, one-SM kernel: K blocks of every tile split over this many CTAs (1: none); each
                         // writes its fp32 partial sums to `partial`, and splitk_finalize_kernel adds them
  float* partial;        // ksplit > 1: fp32 [ksplit, M, N] partial sums (zero-point term in split 0)
  int pdl;               // host: launch with programmatic stream serialization (the kernel's prologue - barrier
                         // set-up, TMEM allocation, descriptor prefetch - overlaps the tail of the previous kernel;
                         // every thread waits for that kernel's completion before its first read of any input)
};

// Output operations of the affine epilogue (values of cq_out_kind)
enum : int { OUT_PLAIN = 0, OUT_GELU = 1, OUT_GATED = 2 };
constexpr int kResBatch = 8;   // gated residual: rows per batch of residual loads
constexpr int kResAhead = 2;   //   batches in flight ahead of the one in use

__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProducerRegs));
}
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kEpilogueRegs));
}

// d = a * b + c on two fp32 lanes at once (sm_100 packed FMA)
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

// d = a * b on two fp32 lanes at once
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// d = a + b on two fp32 lanes at once
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// The output operation (plain or GELU) on two fp32 linear outputs u (bias included) of one column; the caller
// rounds the results to bf16.  GELU acts on y = bf16(u), the value the plain epilogue stores:
//   gelu_tanh(y) = 0.5 y (1 + tanh(w)), w = sqrt(2/pi) (y + 0.044715 y^3), in its logistic form
//   y / (1 + 2^(-y (kA + kB y^2))), kA = 2 sqrt(2/pi) log2(e), kB = 0.044715 kA,
// which has no cancellation near 1 + tanh(w) = 0; the hardware base-2 exponential and reciprocal (for large
// negative y the exponential overflows to inf and the reciprocal gives 0).  The fp32 arithmetic runs in packed f32x2
// instructions: the store pass is bound by the epilogue warps' instruction issue (a variant that replaced the
// reciprocal by Newton steps on the FMA pipe measured slower, and so did the scalar form of this one).
template <int OP>
__device__ __forceinline__ float2 out_apply2(float2 u) {
  if constexpr (OP == OUT_PLAIN) {
    return u;
  } else {
    uint32_t b;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(b) : "f"(u.y), "f"(u.x));
    const float2 y = make_float2(__uint_as_float(b << 16), __uint_as_float(b & 0xFFFF0000u));
    // t = -y (kA + kB y^2) with the constants negated, then y / (1 + 2^t)
    const float2 p = ffma2(make_float2(-0.10294324f, -0.10294324f), fmul2(y, y), make_float2(-2.3022082f, -2.3022082f));
    const float2 t = fmul2(y, p);
    float2 e, r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e.x) : "f"(t.x));
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e.y) : "f"(t.y));
    const float2 d = fadd2(e, make_float2(1.0f, 1.0f));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r.x) : "f"(d.x));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r.y) : "f"(d.y));
    return fmul2(y, r);
  }
}

// Row/col epilogue with an output operation: one 32-token chunk (tokens m_c + [0, 32)) of column n from the chunk's
// int32 sums r.  v = fma(float(P) * sb, sa[m], bias), the plain epilogue's value; then GELU-tanh of bf16(v), or the
// gated residual bf16(res[m, n] + gate[n] * bf16(v)) in one packed bf16 fma (gate2: the gate's bits in both halves);
// stored as bf16.  Rows past M are neither read nor written.  Each (m, n) is read and written by one thread, so the
// residual may be the output itself.
template <int OP>
__device__ __forceinline__ void rowcol_op_chunk(const GemmArgs& args, const uint32_t (&r)[32], const float* sa_c,
                                                float sb, float bias, int m_c, int n, uint32_t gate2) {
  const int N = args.N;
  const int rows = min(32, args.M - m_c);
  uint32_t res[OP == OUT_GATED ? 32 : 1];
  if constexpr (OP == OUT_GATED) {
    const unsigned short* rp =
        reinterpret_cast<const unsigned short*>(args.res) + static_cast<int64_t>(m_c) * args.res_ld + n;
#pragma unroll
    for (int t = 0; t < 32; ++t) res[t] = t < rows ? __ldg(rp + static_cast<int64_t>(t) * args.res_ld) : 0u;
  }
  __nv_bfloat16* orow = args.out + static_cast<int64_t>(m_c) * N + n;
#pragma unroll
  for (int t = 0; t < 32; t += 2) {
    const float2 c = *reinterpret_cast<const float2*>(sa_c + t);
    const float v0 = __fmaf_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[t])), sb), c.x, bias);
    const float v1 = __fmaf_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[t + 1])), sb), c.y, bias);
    uint32_t o;
    if constexpr (OP == OUT_GATED) {
      o = gated_pair_bits(v0, v1, gate2, res[t], res[t + 1]);
    } else {
      const float2 g = out_apply2<OP>(make_float2(v0, v1));
      o = bf16_pair_bits(g.x, g.y);
    }
    if (t < rows) *reinterpret_cast<unsigned short*>(orow) = static_cast<unsigned short>(o & 0xFFFFu);
    if (t + 1 < rows) *reinterpret_cast<unsigned short*>(orow + N) = static_cast<unsigned short>(o >> 16);
    orow += 2 * static_cast<int64_t>(N);
  }
}

// the gate of column n in both halves of a word (gated residual output), else 0
template <int OP>
__device__ __forceinline__ uint32_t load_gate2(const GemmArgs& args, int n, bool n_ok) {
  if constexpr (OP != OUT_GATED) return 0u;
  const uint32_t g = n_ok ? static_cast<uint32_t>(__ldg(reinterpret_cast<const unsigned short*>(args.gate) + n)) : 0u;
  return g | (g << 16);
}

// Tile order.  Tiles are visited in groups of up to kRasterGroup token tiles: inside a group the token tile varies
// fastest and the weight tile next, so one wave of CTAs (consecutive tile indices) covers a few token tiles by many
// weight tiles.  Both operands of a wave then stay in L2, where a plain token-fastest order would stream a
// different activation tile into every CTA of the wave and re-read all activations from HBM for every weight
// tile once they outgrow L2.
constexpr int kRasterGroup = 8;
__device__ __forceinline__ void tile_coords(int tile, int m_tiles, int n_tiles, int& mt, int& nt) {
  const int per_group = kRasterGroup * n_tiles;
  const int g = tile / per_group;
  const int t = tile - g * per_group;
  const int rows = min(kRasterGroup, m_tiles - g * kRasterGroup);   // token tiles in this (possibly last) group
  mt = g * kRasterGroup + t % rows;
  nt = t / rows;
}

// Work item -> tile and token range.  Items [0, num_tiles - split) are whole tiles in raster order; each of the last
// `split` tiles becomes two items, the two halves of its tokens.  t0: first token of the item in its tile; width:
// kBT (whole) or kBT / 2 (half).
__device__ __forceinline__ void item_coords(int item, int num_tiles, int split, int m_tiles, int n_tiles, int& mt,
                                            int& nt, int& t0, int& width) {
  const int whole = num_tiles - split;
  int tile = item;
  t0 = 0;
  width = kBT;
  if (item >= whole) {
    const int h = item - whole;
    tile = whole + (h >> 1);
    t0 = (kBT / 2) * (h & 1);
    width = kBT / 2;
  }
  tile_coords(tile, m_tiles, n_tiles, mt, nt);
}

// 8 packed bytes (16 nibbles, low nibble = even column) -> 16 bytes holding 16*v per column.
//   KPERM: the activations' K order inside each 8-column block is 0,2,4,6,1,3,5,7, so the low nibbles of a
//          word (even columns) and its high nibbles (odd columns) are already in place.
//   else:  natural K order, interleaved with byte permutes.
template <int BFMT, bool KPERM>
__device__ __forceinline__ uint4 unpack16(uint2 p) {
  const uint32_t flip = (BFMT == BF_U4) ? 0x80808080u : 0u;   // uint4 q -> signed (q - 8): flip the top bit
  const uint32_t lo0 = ((p.x << 4) & 0xF0F0F0F0u) ^ flip, hi0 = (p.x & 0xF0F0F0F0u) ^ flip;
  const uint32_t lo1 = ((p.y << 4) & 0xF0F0F0F0u) ^ flip, hi1 = (p.y & 0xF0F0F0F0u) ^ flip;
  if (KPERM) return make_uint4(lo0, hi0, lo1, hi1);
  return make_uint4(prmt(lo0, hi0, 0x5140u), prmt(lo0, hi0, 0x7362u), prmt(lo1, hi1, 0x5140u),
                    prmt(lo1, hi1, 0x7362u));
}

template <int EPI, int BFMT, bool KPERM, bool GLU = false, int OP = OUT_PLAIN>
__global__ void __launch_bounds__(kThreads, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
            const __grid_constant__ CUtensorMap tm_r, const __grid_constant__ CUtensorMap tm_z,
            const __grid_constant__ OutMaps tm_out, const GemmArgs args) {
  using P = SmemPlan<EPI, BFMT, GLU>;
  static_assert(!GLU || (EPI == EPI_ROWCOL && BFMT == BF_S4), "the SwiGLU output is a row/col W4A4 epilogue");
  static_assert(OP == OUT_PLAIN || EPI == EPI_AFFINE || (EPI == EPI_ROWCOL && !GLU),
                "output operations are affine or plain row/col epilogue variants");
  constexpr int kTmaStages = P::kStages;
  constexpr bool kConv = BFMT != BF_S8;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // TMA ring: [stage][X 32 KB | W 8/16 KB]; converter ring after it
  uint8_t* sm_tma = smem;
  uint8_t* sm_conv = smem + kTmaStages * P::kTmaStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P::kData);
  uint64_t* full_tma = bars;
  uint64_t* empty_tma = bars + kTmaStages;
  uint64_t* full_conv = bars + 2 * kTmaStages;
  uint64_t* empty_conv = full_conv + kConvStages;
  uint64_t* tmem_full = empty_conv + kConvStages;
  uint64_t* tmem_empty = tmem_full + kNumBufs;
  uint64_t* zt_full = tmem_empty + kNumBufs;   // affine: per converter pair, the TMA load of its zero-point operand
  uint64_t* box_free = zt_full + kConvStages;   // affine, 64-column boxes: per epilogue warp pair, staging free
  uint64_t* box_full = box_free + 4;            //   and both halves of the box written
  uint64_t* mma_done = box_full + 4;            // every MMA this CTA issued has completed (before the TMEM release)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mma_done + 1);
  static_assert((2 * kTmaStages + 3 * kConvStages + 2 * kNumBufs + 9) * 8 + 8 <= P::kSaStage - P::kData,
                "the barriers, the TMEM address and the abort flag fit the region before the scale staging");
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int M = args.M, N = args.N, K = args.K;
  const int kblocks = K / kBK;
  const int m_tiles = (M + kBT - 1) / kBT;
  const int n_tiles = (N + kBW - 1) / kBW;
  const int num_tiles = m_tiles * n_tiles;
  // Half tiles only for the row/col epilogue, which drains once per tile: the affine epilogue drains every group
  // in each warp's own 128 token columns, so a half tile would take a whole tile's drain time (measured: no gain,
  // and the extra control flow spills registers in the affine epilogue).
  constexpr bool kSplit = (EPI == EPI_ROWCOL);
  const int split = kSplit ? args.split : 0;
  // split K (affine, few tiles): item = tile * ksplit + r sums K blocks [r kps, (r + 1) kps) of the tile
  const int ksplit = (EPI == EPI_AFFINE && args.ksplit > 1) ? args.ksplit : 1;
  const int kps = kblocks / ksplit;
  const int num_items = num_tiles * ksplit + split;
  auto coords = [&](int item, int& mt, int& nt, int& t0, int& width) {
    if constexpr (kSplit) {
      item_coords(item, num_tiles, split, m_tiles, n_tiles, mt, nt, t0, width);
    } else {
      tile_coords(item / ksplit, m_tiles, n_tiles, mt, nt);
      t0 = 0;
      width = kBT;
    }
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTmaStages; ++s) {
      mbar_init(&full_tma[s], 1);
      mbar_init(&empty_tma[s], 1);
    }
    for (int s = 0; s < kConvStages; ++s) {
      mbar_init(&full_conv[s], kConvWarps / kConvStages);   // the pair of converter warps that owns the stage
      mbar_init(&empty_conv[s], 1);
      mbar_init(&zt_full[s], 1);
    }
    for (int b = 0; b < kNumBufs; ++b) {
      mbar_init(&tmem_full[b], 1);
      mbar_init(&tmem_empty[b], 8);
    }
    for (int p = 0; p < 4; ++p) {
      mbar_init(&box_free[p], 1);
      mbar_init(&box_full[p], 2);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tensormap(&tm_x);
    prefetch_tensormap(&tm_w);
    if (EPI == EPI_AFFINE) prefetch_tensormap(&tm_r);
    if (EPI == EPI_AFFINE) prefetch_tensormap(&tm_z);
    if (EPI == EPI_AFFINE && args.tma_out)
      for (int i = 0; i < args.n_out; ++i) prefetch_tensormap(&tm_out.m[i]);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  grid_dep_wait();   // inputs written by the previous kernel (programmatic launch) are visible from here on

  if (warp < kEpiWarp0) {
    setmaxnreg_dec();
    if (warp == 0 && lane == 0) {
      // ------------------------------ TMA producer ------------------------------
      int stage = 0;
      uint32_t phase = 0, issued = 0;
      for (int item = blockIdx.x; item < num_items && !*abort_flag; item += gridDim.x) {
        int mt, nt, t0, width;
        coords(item, mt, nt, t0, width);
        const int m0 = mt * kBT + t0;    // a half tile loads 256 rows from its first token; the MMA reads 128
        const int n0 = nt * kBW;
        const int r_split = item % ksplit;
        if (EPI == EPI_AFFINE) {
          // zero-point operand: the tokens' split group sums (bf16, 64 columns per block) into the X slot.  Only
          // the first K split adds the zero-point term: the others load rows past M, which the copy fills with 0.
          for (int p = 0; p < args.nz; ++p) {
            if (!mbar_wait(&empty_tma[stage], phase ^ 1u, abort_flag, 10)) break;
            uint8_t* st = sm_tma + stage * P::kTmaStageBytes;
            mbar_arrive_expect_tx(&full_tma[stage], kXBytes);
            tma_load_2d(st, &tm_r, &full_tma[stage], p * 128, r_split == 0 ? m0 : M);
            ++issued;
            if (++stage == kTmaStages) { stage = 0; phase ^= 1u; }
          }
        }
        for (int kb = r_split * kps; kb < (r_split + 1) * kps; ++kb) {
          if (!mbar_wait(&empty_tma[stage], phase ^ 1u, abort_flag, 1)) break;
          uint8_t* st = sm_tma + stage * P::kTmaStageBytes;
          mbar_arrive_expect_tx(&full_tma[stage], P::kTmaStageBytes);
          tma_load_2d(st, &tm_x, &full_tma[stage], kb * kBK, m0);
          if (BFMT == BF_S8) tma_load_2d(st + kXBytes, &tm_w, &full_tma[stage], kb * kBK, n0);
          else tma_load_2d(st + kXBytes, &tm_w, &full_tma[stage], kb * (kBK / 2), n0);
          ++issued;
          if (++stage == kTmaStages) { stage = 0; phase ^= 1u; }
        }
      }
      // every load issued has landed before the CTA's shared memory can be released (at once on a normal end)
      drain_ring(full_tma, kTmaStages, issued, 50000000ull);
    } else if (warp == 1 && lane == 0) {
      // ------------------------------ MMA issuer ------------------------------
      int stage = 0, cstage = 0;
      uint32_t phase = 0, cphase = 0;
      int buf = 0;
      uint32_t buf_phase = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < num_items && ok; item += gridDim.x) {
        int mt, nt, t0, width;
        coords(item, mt, nt, t0, width);
        const uint32_t idesc = width == kBT ? idesc_i8(kBW, kBT) : idesc_i8(kBW, kBT / 2);
        if (EPI == EPI_ROWCOL) {
          if (!(ok = mbar_wait(&tmem_empty[buf], buf_phase, abort_flag, 2))) break;
          tc_fence_after();
        }
        if (EPI == EPI_AFFINE) {
          // D = sum_j Zt[n, j] * Rsplit[m, j] in fp32: the zero-point term, the accumulator's starting value
          if (!(ok = mbar_wait(&tmem_empty[buf], buf_phase, abort_flag, 11))) break;
          tc_fence_after();
          const uint32_t idesc_z = width == kBT ? idesc_bf16(kBW, kBT) : idesc_bf16(kBW, kBT / 2);
          for (int p = 0; p < args.nz && ok; ++p) {
            if (!(ok = mbar_wait(&full_tma[stage], phase, abort_flag, 12))) break;
            if (!(ok = mbar_wait(&full_conv[cstage], cphase, abort_flag, 13))) break;
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * kBT);
            const uint32_t a_base = smem_u32(sm_conv + cstage * kWuBytes);
            const uint32_t b_base = smem_u32(sm_tma + stage * P::kTmaStageBytes);
#pragma unroll
            for (int k = 0; k < 4; ++k)   // 64 bf16 = 4 x K16
              mma_bf16(d_tmem, smem_desc_k_sw128(a_base + 32 * k), smem_desc_k_sw128(b_base + 32 * k), idesc_z,
                       (p > 0 || k > 0) ? 1u : 0u);
            tc_commit(&empty_tma[stage]);
            tc_commit(&empty_conv[cstage]);
            if (++stage == kTmaStages) { stage = 0; phase ^= 1u; }
            if (++cstage == kConvStages) { cstage = 0; cphase ^= 1u; }
          }
          if (!ok) break;
          tc_commit(&tmem_full[buf]);
          if (width != kBT) mbar_arrive_cnt(&tmem_empty[buf], 4);   // the idle second-half epilogue warps
          if (++buf == kNumBufs) { buf = 0; buf_phase ^= 1u; }
        }
        for (int kb = 0; kb < kps && ok; ++kb) {
          if (EPI == EPI_AFFINE) {
            if (!(ok = mbar_wait(&tmem_empty[buf], buf_phase, abort_flag, 3))) break;
            tc_fence_after();
          }
          // int4 weights: the converters waited on full_tma before they arrived on full_conv, so full_conv alone
          // orders both the activation tile and the converted weights before these MMAs
          if (!kConv && !(ok = mbar_wait(&full_tma[stage], phase, abort_flag, 4))) break;
          if (kConv && !(ok = mbar_wait(&full_conv[cstage], cphase, abort_flag, 5))) break;
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * kBT);
          uint8_t* st = sm_tma + stage * P::kTmaStageBytes;
          const uint32_t a_base = smem_u32(kConv ? sm_conv + cstage * kWuBytes : st + kXBytes);
          const uint32_t b_base = smem_u32(st);
#pragma unroll
          for (int k = 0; k < kBK / 32; ++k) {
            // affine: every 128-wide group starts its own int32 sum
            const uint32_t acc = (EPI == EPI_AFFINE) ? (k > 0) : (kb > 0 || k > 0);
            mma_i8(d_tmem, smem_desc_k_sw128(a_base + 32 * k), smem_desc_k_sw128(b_base + 32 * k), idesc, acc);
          }
          tc_commit(&empty_tma[stage]);
          if (kConv) tc_commit(&empty_conv[cstage]);
          if (EPI == EPI_AFFINE) {
            tc_commit(&tmem_full[buf]);
            if (width != kBT) mbar_arrive_cnt(&tmem_empty[buf], 4);
            if (++buf == kNumBufs) { buf = 0; buf_phase ^= 1u; }
          }
          if (++stage == kTmaStages) { stage = 0; phase ^= 1u; }
          if (kConv && ++cstage == kConvStages) { cstage = 0; cphase ^= 1u; }
        }
        if (EPI == EPI_ROWCOL && ok) {
          tc_commit(&tmem_full[buf]);
          if (width != kBT) mbar_arrive_cnt(&tmem_empty[buf], 4);
          if (++buf == kNumBufs) { buf = 0; buf_phase ^= 1u; }
        }
      }
      // completes when every MMA issued above has completed; the TMEM release waits for it
      tc_commit(mma_done);
    } else if (warp >= 2 && kConv) {
      // ------------------------------ int4 -> int8 converters ------------------------------
      // Three pairs of warps take this CTA's operand blocks round-robin: pair c converts blocks c, c + 3, c + 6, ...
      // (block j = the j-th K block of the CTA's tile sequence, zero-point pseudo blocks included) into converter
      // stage c, so three blocks are in conversion at once instead of one block at a time.
      const int pair = (warp - 2) >> 1;               // 0..kConvStages-1: this pair's converter stage
      const int pt = threadIdx.x - 64 * (1 + pair);   // 0..63
      const int nzb = (EPI == EPI_AFFINE) ? args.nz : 0;
      const int bpt = nzb + kps;                      // operand blocks per item (tile, or K split of a tile)
      uint8_t* dst = sm_conv + pair * kWuBytes;
      // the thread's items are it = pt + 64 i (i = 0..7): row (pt >> 2) + 16 i, 16-byte column c4 = pt & 3.  Row
      // steps of 16 keep (row & 7), so both swizzled destination chunks sit at fixed offsets from the row start
      // and every address below is a per-thread base plus an immediate.
      const int rr = pt >> 2, c4 = pt & 3;
      const uint32_t src_off = static_cast<uint32_t>(rr * 64 + c4 * 16);
      uint8_t* const drow0 = dst + rr * 128;
      const uint32_t dlo = static_cast<uint32_t>(((2 * c4) ^ (rr & 7)) << 4), dhi = static_cast<uint32_t>(((2 * c4 + 1) ^ (rr & 7)) << 4);
      // block j = pair + 3 i: its tile, its index b inside the tile and its TMA stage advance incrementally
      int item = blockIdx.x, b = pair, stage = pair;
      uint32_t phase = 0, cphase = 0, zphase = 0;
      while (b >= bpt) { b -= bpt; item += gridDim.x; }
      for (; item < num_items; cphase ^= 1u) {
        if (!mbar_wait(&empty_conv[pair], cphase ^ 1u, abort_flag, 9)) break;
        if (EPI == EPI_AFFINE && b < nzb) {
          // zero-point weight operand: rows n0..n0+127 of the prepared Zt, 64 bf16 columns per pseudo block, one TMA
          // load straight into this stage in the operand layout (rows past N read as zeros).  The matching TMA
          // stage carries the activation-side operand.
          if (warp == 2 + 2 * pair && lane == 0) {
            mbar_arrive_expect_tx(&zt_full[pair], kWuBytes);
            int mt, nt, t0, width;
            coords(item, mt, nt, t0, width);
            tma_load_2d(dst, &tm_z, &zt_full[pair], 128 * b, nt * kBW);
          }
          if (!mbar_wait(&zt_full[pair], zphase, abort_flag, 16)) break;
          zphase ^= 1u;
        } else {
          if (!mbar_wait(&full_tma[stage], phase, abort_flag, 6)) break;
          const uint8_t* src = sm_tma + stage * P::kTmaStageBytes + kXBytes + src_off;
          // item i: 16 packed bytes (32 K columns) of row rr + 16 i -> output chunks 2*c4 and 2*c4 + 1 of that row
#pragma unroll 4
          for (int i = 0; i < kBW / 16; ++i) {
            const uint4 p = *reinterpret_cast<const uint4*>(src + i * 1024);
            *reinterpret_cast<uint4*>(drow0 + i * 2048 + dlo) = unpack16<BFMT, KPERM>(make_uint2(p.x, p.y));
            *reinterpret_cast<uint4*>(drow0 + i * 2048 + dhi) = unpack16<BFMT, KPERM>(make_uint2(p.z, p.w));
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full_conv[pair]);
        b += kConvStages;
        while (b >= bpt) { b -= bpt; item += gridDim.x; }
        stage += kConvStages;
        if (stage >= kTmaStages) { stage -= kTmaStages; phase ^= 1u; }
      }
    }
  } else {
    // ------------------------------ epilogue (warps 8..15) ------------------------------
    setmaxnreg_inc();
    const int e = warp - kEpiWarp0;
    const int quad = warp & 3;            // TMEM lane quadrant this warp may access
    const int half = e >> 2;              // token half of the tile: columns [128*half, 128*half + 128)
    const uint32_t lane_addr = static_cast<uint32_t>(32 * quad) << 16;
    // the int4 unpack stores 16*v; fold the 1/16 into the weight scale (exact)
    const float wscale_fold = (BFMT == BF_S8) ? 1.0f : 0.0625f;
    // this warp's 128 token scales for the store phase (read back as broadcast float4 loads)
    float* sa_stage = reinterpret_cast<float*>(smem + P::kSaStage) + e * kWarpTok;
    uint32_t box_pass = 0;                // output store passes so far (phase of this warp pair's box barriers)
    int buf = 0;
    uint32_t buf_phase = 0;
    bool ok = true;
    // hand both accumulator buffers to the MMA issuer
    for (int b = 0; b < kNumBufs; ++b) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tmem_empty[b]);
    }
    for (int item = blockIdx.x; item < num_items && ok; item += gridDim.x) {
      int mt, nt, t0, width;
      coords(item, mt, nt, t0, width);
      if (half * kWarpTok >= width) {
        // a half tile holds tokens for the first half's warps only; the MMA issuer arrives on this warp's behalf on
        // each of the item's accumulator buffers, so the warp only steps its buffer position past the item
        const int uses = (EPI == EPI_AFFINE) ? 1 + kps : 1;
        for (int u = 0; u < uses; ++u)
          if (++buf == kNumBufs) { buf = 0; buf_phase ^= 1u; }
        continue;
      }
      const int m0 = mt * kBT + t0 + half * kWarpTok;
      const int n = nt * kBW + quad * 32 + lane;
      const bool n_ok = n < N;
      const bool m_full = m0 + kWarpTok <= M;   // every token of the warp exists: no per-element checks
      const float bias = (args.bias != nullptr && n_ok) ? __bfloat162float(args.bias[n]) : 0.0f;
      if constexpr (OP == OUT_GATED) {
        // the warp's residual box (its 128 tokens x 32 columns) into L2 now, a whole tile of group drains before
        // the store passes read it
        const int c0 = n - lane;
        if (c0 < N)
          for (int r = lane; r < kWarpTok && m0 + r < M; r += 32)
            prefetch_l2(args.res + static_cast<int64_t>(m0 + r) * args.res_ld + c0);
      }
      // the tokens' activation scales, one per lane and 32-token chunk, loaded when the tile starts so that their
      // latency hides behind the tile's MMAs (indices past the last token clamp to it; those rows are not stored)
      float sa_pre[kChunks];
#pragma unroll
      for (int c = 0; c < kChunks; ++c) sa_pre[c] = __ldg(args.sa + min(m0 + 32 * c + lane, M - 1));
      auto stage_sa = [&]() {
        __syncwarp();
#pragma unroll
        for (int c = 0; c < kChunks; ++c) sa_stage[32 * c + lane] = sa_pre[c];
        __syncwarp();
      };
      if (EPI == EPI_AFFINE) {
        float2 acc[kWarpTok / 2];
        {
          // starting value: the zero-point term sum_g z[g, n] * R[g, m], accumulated in fp32 by the tensor core
          if (!(ok = mbar_wait(&tmem_full[buf], buf_phase, abort_flag, 15))) break;
          tc_fence_after();
          const uint32_t taddr = tmem_base + lane_addr + static_cast<uint32_t>(buf * kBT + half * kWarpTok);
#pragma unroll
          for (int ch = 0; ch < kChunks; ++ch) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(taddr + 32 * ch, r);
            tmem_wait_ld_dep(r);
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[16 * ch + j] = make_float2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tmem_empty[buf]);
          if (++buf == kNumBufs) { buf = 0; buf_phase ^= 1u; }
        }
        // the weight scale of the next group is loaded one group ahead as raw bf16 bits and converted only when it
        // is used, so its latency hides behind a drain instead of stalling the warp at the load
        const int r_split = item % ksplit;
        const unsigned short* ws_bits =
            reinterpret_cast<const unsigned short*>(args.ws) + static_cast<int64_t>(r_split * kps) * N + n;
        unsigned short s_bits_next = n_ok ? __ldg(ws_bits) : static_cast<unsigned short>(0);
        for (int g = 0; g < kps; ++g) {
          const unsigned short s_bits = s_bits_next;
          if (g + 1 < kps && n_ok) s_bits_next = __ldg(ws_bits + static_cast<int64_t>(g + 1) * N);
          if (!(ok = mbar_wait(&tmem_full[buf], buf_phase, abort_flag, 7))) break;
          tc_fence_after();
          const float s = bf16_bits_to_f32(s_bits) * wscale_fold;
          const float2 s2 = make_float2(s, s);
          const uint32_t taddr = tmem_base + lane_addr + static_cast<uint32_t>(buf * kBT + half * kWarpTok);
          // software-pipelined drain: chunk c+1 is in flight while chunk c is scaled, and the buffer goes back to
          // the MMA as soon as the last chunk is in registers
          uint32_t ra[32], rb[32];
          auto scale_chunk = [&](const uint32_t (&r)[32], int ch) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              // |P| < 2^22, so the int32 -> fp32 conversion is exact (it runs on the integer pipe, beside the FMAs)
              const float2 p = make_float2(__int2float_rn(static_cast<int>(r[2 * j])), __int2float_rn(static_cast<int>(r[2 * j + 1])));
              acc[16 * ch + j] = ffma2(s2, p, acc[16 * ch + j]);
            }
          };
          if constexpr (kChunks == 4) {
            tmem_ld_32x32b_x32(taddr, ra);
            tmem_wait_ld_dep(ra);
            tmem_ld_32x32b_x32(taddr + 32, rb);
            scale_chunk(ra, 0);
            tmem_wait_ld_dep(rb);
            tmem_ld_32x32b_x32(taddr + 64, ra);
            scale_chunk(rb, 1);
            tmem_wait_ld_dep(ra);
            tmem_ld_32x32b_x32(taddr + 96, rb);
            scale_chunk(ra, 2);
            tmem_wait_ld_dep(rb);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tmem_empty[buf]);
            scale_chunk(rb, 3);
          } else {
            // two chunks: both loads in flight together, the buffer back to the MMA before the math
            tmem_ld_32x32b_x32(taddr, ra);
            tmem_ld_32x32b_x32(taddr + 32, rb);
            tmem_wait_ld_dep(ra);
            tmem_wait_ld_dep(rb);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tmem_empty[buf]);
            scale_chunk(ra, 0);
            scale_chunk(rb, 1);
          }
          if (++buf == kNumBufs) { buf = 0; buf_phase ^= 1u; }
        }
        if (!ok) break;
        if (ksplit > 1) {
          // one K split of the tile: its fp32 sums (the zero-point term in split 0) into the partial array, 32
          // consecutive columns per token row; splitk_finalize_kernel adds the splits in order and applies the token
          // scale, the bias and the output operation
          if (n_ok) {
            float* prow = args.partial + (static_cast<int64_t>(r_split) * M + m0) * N + n;
#pragma unroll
            for (int j = 0; j < kWarpTok / 2; ++j) {
              if (m_full || m0 + 2 * j < M) prow[static_cast<int64_t>(2 * j) * N] = acc[j].x;
              if (m_full || m0 + 2 * j + 1 < M) prow[static_cast<int64_t>(2 * j + 1) * N] = acc[j].y;
            }
          }
          continue;
        }
        stage_sa();
        if (args.tma_out) {
          // two passes of 64 tokens: bf16 results into a staging buffer ([token][columns]), then one TMA tensor store
          // per pass and output buffer.  The store drains in the background while the warp moves on; rows past M
          // and columns past N are clipped by the tensor map.  With out_w64 the warps of quadrants 2k and 2k+1 (same
          // token half) fill the two halves of a 64-column box in their joint 8 KB buffer, synchronized by a named
          // barrier, and the even warp issues the stores: each box row is 128 contiguous bytes, which a remote
          // (NVLink) write moves more efficiently than 64-byte rows.
          auto store_passes = [&](auto row_bytes_c, auto op_c) -> bool {
            constexpr uint32_t kRow = decltype(row_bytes_c)::value;
            constexpr int kOp = decltype(op_c)::value;
            constexpr bool kPair = kRow == 128;
            const int owner = kPair ? (e & ~1) : e;
            unsigned short* ost = reinterpret_cast<unsigned short*>(smem + P::kOutStage + owner * P::kOutWarpBytes);
            const uint32_t ost_lane = smem_u32(ost) + (kPair ? 64u * (e & 1) : 0u) + 2u * lane;
            // plain and GELU outputs leave as 32-bit stores of two adjacent columns: lanes 2i and 2i + 1 swap one
            // packed token pair, then the even lane writes both columns of the first token and the odd lane both
            // columns of the second (half the shared-memory store instructions of one 16-bit store per element)
            const uint32_t odd = lane & 1u;
            const uint32_t pair_sel = odd ? 0x3276u : 0x5410u;
            const uint32_t ost_pair = ost_lane - 2u * odd + odd * kRow;
            const bool issuer = !kPair || (e & 1) == 0;
            const int x0 = nt * kBW + (kPair ? (quad & 2) : quad) * 32;
            const int pr = e >> 1;
#pragma unroll
            for (int pass = 0; pass < kWarpTok / 64; ++pass, ++box_pass) {
              const uint32_t par = box_pass & 1u;
              if (issuer) {
                if (lane == 0) {
                  bulk_wait_group_read0();            // the previous store has finished reading the buffer
                  if (kPair) mbar_arrive(&box_free[pr]);
                }
                __syncwarp();
              } else if (!mbar_wait(&box_free[pr], par, abort_flag, 17)) {
                return false;
              }
              // gated residual: this lane's column of the pass's 64 residual rows, in batches of kResBatch rows issued
              // kResAhead batches ahead of their use
              // (one pointer walked down the rows; lanes past N read column N - 1 and rows past M repeat the last
              // row, neither of which is stored)
              uint32_t rres[kOp == OUT_GATED ? 64 : 1];
              // the column's gate, loaded here rather than with the bias so that no register holds it across the
              // tile's group drains
              const uint32_t gate_bits =
                  (kOp == OUT_GATED && n_ok) ? static_cast<uint32_t>(__ldg(reinterpret_cast<const unsigned short*>(args.gate) + n)) : 0u;
              const uint32_t gate2 = gate_bits | (gate_bits << 16);
              const unsigned short* rp = nullptr;
              int rows_left = 0;
              if constexpr (kOp == OUT_GATED) {
                rows_left = M - (m0 + 64 * pass);
                rp = reinterpret_cast<const unsigned short*>(args.res) + min(n, N - 1) +
                     static_cast<int64_t>(m0 + 64 * pass) * args.res_ld;
              }
              auto load_res = [&](int b) {
                if constexpr (kOp == OUT_GATED) {
#pragma unroll
                  for (int i = 0; i < kResBatch; ++i) {
                    rres[kResBatch * b + i] = __ldg(rp);
                    if (kResBatch * b + i + 1 < rows_left) rp += args.res_ld;
                  }
                }
              };
#pragma unroll
              for (int b = 0; b < kResAhead; ++b) load_res(b);
#pragma unroll
              for (int j4 = 0; j4 < 16; ++j4) {
                if (j4 % (kResBatch / 4) == 0 && j4 / (kResBatch / 4) + kResAhead < 64 / kResBatch) load_res(j4 / (kResBatch / 4) + kResAhead);
                const int t = 64 * pass + 4 * j4;
                const int r = kOp == OUT_GATED ? 4 * j4 : 0;
                const float4 c = *reinterpret_cast<const float4*>(sa_stage + t);
                // the linear's fp32 outputs of tokens t..t+3, two per packed fma (the same roundings as scalar fmas)
                const float2 u01 = ffma2(acc[t / 2], make_float2(c.x, c.y), make_float2(bias, bias));
                const float2 u23 = ffma2(acc[t / 2 + 1], make_float2(c.z, c.w), make_float2(bias, bias));
                if constexpr (kOp == OUT_GATED) {
                  sts_gated_pair(ost_lane + (4 * j4) * kRow, ost_lane + (4 * j4 + 1) * kRow, u01.x, u01.y, gate2,
                                 rres[r], rres[r + 1]);
                  sts_gated_pair(ost_lane + (4 * j4 + 2) * kRow, ost_lane + (4 * j4 + 3) * kRow, u23.x, u23.y, gate2,
                                 rres[r + 2], rres[r + 3]);
                } else {
                  const float2 v01 = out_apply2<kOp>(u01), v23 = out_apply2<kOp>(u23);
                  const uint32_t b01 = bf16x2_bits(v01.x, v01.y), b23 = bf16x2_bits(v23.x, v23.y);
                  const uint32_t r01 = __shfl_xor_sync(0xffffffffu, b01, 1), r23 = __shfl_xor_sync(0xffffffffu, b23, 1);
                  sts_b32(ost_pair + (4 * j4) * kRow, prmt(b01, r01, pair_sel));
                  sts_b32(ost_pair + (4 * j4 + 2) * kRow, prmt(b23, r23, pair_sel));
                }
              }
              fence_proxy_async_smem();
              __syncwarp();
              if (kPair && lane == 0) mbar_arrive(&box_full[pr]);
              if (issuer && lane == 0) {
                if (kPair && !mbar_wait(&box_full[pr], par, abort_flag, 18)) return false;
                if (x0 < N && m0 + 64 * pass < M) {   // boxes wholly past the edge are not issued
                  // one store per output buffer (column-parallel layers: this rank's columns into every rank's output)
                  for (int i = 0; i < args.n_out; ++i) tma_store_2d(&tm_out.m[i], ost, args.out_col0 + x0, m0 + 64 * pass);
                  bulk_commit_group();
                }
              }
            }
            return true;
          };
          // the output operation is a template parameter: the plain kernel carries none of its code
          using Op = std::integral_constant<int, OP>;
          const bool stored = args.out_w64 ? store_passes(std::integral_constant<uint32_t, 128>{}, Op{})
                                           : store_passes(std::integral_constant<uint32_t, 64>{}, Op{});
          if (!__all_sync(0xffffffffu, stored)) { ok = false; break; }
        } else if (n_ok) {
          // column n of the output for tokens m0..m0+127: one pointer walked down the rows
          __nv_bfloat16* orow = args.out + static_cast<int64_t>(m0) * N + n;
#pragma unroll
          for (int j4 = 0; j4 < kWarpTok / 4; ++j4) {
            const float4 c = *reinterpret_cast<const float4*>(sa_stage + 4 * j4);
            const int m = m0 + 4 * j4;
            const float v0 = __fmaf_rn(acc[2 * j4].x, c.x, bias), v1 = __fmaf_rn(acc[2 * j4].y, c.y, bias);
            const float v2 = __fmaf_rn(acc[2 * j4 + 1].x, c.z, bias), v3 = __fmaf_rn(acc[2 * j4 + 1].y, c.w, bias);
            if (m_full || m + 3 < M) {
              st_bf16_pair_ordered(orow, orow + N, v0, v1);
              st_bf16_pair_ordered(orow + 2 * static_cast<int64_t>(N), orow + 3 * static_cast<int64_t>(N), v2, v3);
            } else {
              // partial tile: rows at or past M are not stored (the paired form writes both rows)
              __nv_bfloat16* rows[4] = {orow, orow + N, orow + 2 * static_cast<int64_t>(N), orow + 3 * static_cast<int64_t>(N)};
              const float vs[4] = {v0, v1, v2, v3};
#pragma unroll
              for (int t = 0; t < 4; ++t)
                if (m + t < M) *rows[t] = __float2bfloat16_rn(vs[t]);
            }
            orow += 4 * static_cast<int64_t>(N);
          }
        }
      } else {
        if (!(ok = mbar_wait(&tmem_full[buf], buf_phase, abort_flag, 8))) break;
        tc_fence_after();
        const float sb = n_ok ? args.sb[n] * wscale_fold : 0.0f;
        const uint32_t taddr = tmem_base + lane_addr + static_cast<uint32_t>(buf * kBT + half * kWarpTok);
        if constexpr (GLU) {
          // SwiGLU output: each 32-row lane quadrant holds 16 gate rows (lanes 0-15, of y[:, :N/2]) and their 16
          // up rows (lanes 16-31, of y[:, N/2:]), so lanes l and l ^ 16 carry the two halves of one output
          // column.  out[m, c] = bf16(bf16(silu(gate)) * up) with gate and up the bf16-rounded linear outputs,
          // the roundings of torch's silu and mul on the bf16 linear output.  Per 32-token chunk, lanes 0-15
          // write tokens 0-15 and lanes 16-31 tokens 16-31: one shuffle per token pair hands each lane the
          // other half it needs.
          stage_sa();
          const bool gate = lane < 16;
          const int ncols = N / 2;
          const int j = nt * (kBW / 2) + quad * 16 + (lane & 15);   // output column of this lane's row pair
          const int tb = gate ? 0 : 16;                              // first token of this lane's 16
#pragma unroll 1
          for (int ch = 0; ch < kChunks; ++ch) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(taddr + 32 * ch, r);
            tmem_wait_ld_dep(r);
            float v[32];
#pragma unroll
            for (int t = 0; t < 32; ++t)
              v[t] = bf16_round(__fmaf_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[t])), sb), sa_stage[32 * ch + t],
                                          bias));
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              // gate lanes send token 16 + k (the up lane's) and receive the up value of token k; up lanes
              // send token k and receive the gate value of token 16 + k
              const float other = __shfl_xor_sync(0xffffffffu, gate ? v[16 + k] : v[k], 16);
              const float g = gate ? v[k] : other;
              const float u = gate ? other : v[16 + k];
              // silu with the hardware exponential and an approximate divide: a few fp32 ulp from torch's
              // expf/IEEE-divide form, which the bf16 rounding that follows hides except at rare rounding ties
              const float silu = bf16_round(__fdividef(g, 1.0f + __expf(-g)));
              const int m = m0 + 32 * ch + tb + k;
              if (m < M) args.out[static_cast<int64_t>(m) * ncols + j] = __float2bfloat16_rn(__fmul_rn(silu, u));
            }
          }
        } else if constexpr (OP != OUT_PLAIN) {
          stage_sa();
          const uint32_t gate2 = load_gate2<OP>(args, n, n_ok);
#pragma unroll 1
          for (int ch = 0; ch < kChunks; ++ch) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(taddr + 32 * ch, r);
            tmem_wait_ld_dep(r);
            if (n_ok && m0 + 32 * ch < M) rowcol_op_chunk<OP>(args, r, sa_stage + 32 * ch, sb, bias, m0 + 32 * ch, n, gate2);
          }
        } else {
        __nv_bfloat16* orow = args.out + static_cast<int64_t>(m0) * N + n;
        stage_sa();
#pragma unroll 1
        for (int ch = 0; ch < kChunks; ++ch) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(taddr + 32 * ch, r);
          tmem_wait_ld_dep(r);
          if (n_ok) {
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4) {
              const float4 c = *reinterpret_cast<const float4*>(sa_stage + 32 * ch + 4 * j4);
              const float cv[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
              for (int t = 0; t < 4; t += 2) {
                const int mm = 32 * ch + 4 * j4 + t;
                const float v0 = __fmaf_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[4 * j4 + t])), sb), cv[t], bias);
                const float v1 = __fmaf_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[4 * j4 + t + 1])), sb), cv[t + 1], bias);
                if (m_full || m0 + mm + 1 < M) {
                  st_bf16_pair_ordered(orow, orow + N, v0, v1);
                } else if (m0 + mm < M) {
                  *orow = __float2bfloat16_rn(v0);
                }
                orow += 2 * static_cast<int64_t>(N);
              }
            }
          }
        }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tmem_empty[buf]);
        if (++buf == kNumBufs) { buf = 0; buf_phase ^= 1u; }
      }
    }
  }

  // outstanding TMA output stores of this thread complete before the CTA exits
  if (EPI == EPI_AFFINE && warp >= kEpiWarp0 && lane == 0) bulk_wait_group0();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    // no MMA still in flight writes the accumulators (on an abort the issuer may have left some behind)
    mbar_wait_drain(mma_done, 0, 50000000ull);
    tc_fence_after();
    __syncwarp();
    tmem_dealloc(tmem_base, 512);
  }
}

// The K splits of the affine GEMM added up: out[m, n0..n0+7] = op(bf16(fma(sum_r partial[r, m, n], sa[m], bias[n])))
// with the splits summed in order r = 0, 1, ... (deterministic), and the output operation as in the GEMM's epilogue.
// One thread per 8 consecutive columns of a row (N % 8 == 0).
template <int OP>
__global__ void splitk_finalize_kernel(const GemmArgs args) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int N = args.N, M = args.M;
  const int n8 = N / 8;
  if (i >= static_cast<int64_t>(M) * n8) return;
  const int m = static_cast<int>(i / n8), n0 = 8 * static_cast<int>(i % n8);
  float v[8];
  const float* p = args.partial + static_cast<int64_t>(m) * N + n0;
  {
    const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
  for (int r = 1; r < args.ksplit; ++r) {
    const float* q = p + static_cast<int64_t>(r) * M * N;
    const float4 a = *reinterpret_cast<const float4*>(q), b = *reinterpret_cast<const float4*>(q + 4);
    v[0] += a.x; v[1] += a.y; v[2] += a.z; v[3] += a.w; v[4] += b.x; v[5] += b.y; v[6] += b.z; v[7] += b.w;
  }
  const float sa = args.sa[m];
  uint32_t w[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float b0 = args.bias != nullptr ? __bfloat162float(args.bias[n0 + 2 * k]) : 0.0f;
    const float b1 = args.bias != nullptr ? __bfloat162float(args.bias[n0 + 2 * k + 1]) : 0.0f;
    const float2 u = make_float2(__fmaf_rn(v[2 * k], sa, b0), __fmaf_rn(v[2 * k + 1], sa, b1));
    if constexpr (OP == OUT_GATED) {
      // one bf16x2 fused multiply-add: res + gate * bf16(u), as the epilogue's gated store
      const uint32_t g2 = *reinterpret_cast<const uint32_t*>(args.gate + n0 + 2 * k);
      const uint32_t r2 = *reinterpret_cast<const uint32_t*>(args.res + static_cast<int64_t>(m) * args.res_ld + n0 + 2 * k);
      uint32_t y, o;
      asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(y) : "f"(u.y), "f"(u.x));
      asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(o) : "r"(g2), "r"(y), "r"(r2));
      w[k] = o;
    } else {
      const float2 o = out_apply2<OP>(u);
      asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(w[k]) : "f"(o.y), "f"(o.x));
    }
  }
  *reinterpret_cast<uint4*>(args.out + static_cast<int64_t>(m) * N + n0) = make_uint4(w[0], w[1], w[2], w[3]);
}

// Zt[n, j] = z[j mod G, n] for j < 2G, 0 for 2G <= j < cols (the affine GEMM's zero-point weight operand)
__global__ void prep_zt_kernel(const __nv_bfloat16* __restrict__ z, __nv_bfloat16* __restrict__ zt, int N, int G,
                               int cols) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<int64_t>(N) * cols) return;
  const int n = static_cast<int>(i / cols), j = static_cast<int>(i % cols);
  const int g = j < G ? j : (j < 2 * G ? j - G : -1);
  zt[i] = g >= 0 ? z[static_cast<int64_t>(g) * N + n] : __float2bfloat16_rn(0.0f);
}

cudaError_t launch_prep_zt(const void* z, int N, int K, void* zt, cudaStream_t st) {
  const int cols = rsplit_cols(K);
  const int64_t total = static_cast<int64_t>(N) * cols;
  if (total == 0) return cudaSuccess;
  prep_zt_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, st>>>(
      static_cast<const __nv_bfloat16*>(z), static_cast<__nv_bfloat16*>(zt), N, K / kBK, cols);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D uint8 tensor map: rows x cols bytes (row stride = cols), box box_cols x box_rows.
static bool make_map_u8(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int box_cols, int box_rows,
                        bool swizzle128) {
  EncodeTiledFn fn = get_encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 2-D bf16 tensor map over the [rows, cols] output (row stride cols), box box_cols x box_rows, no swizzle.
static bool make_map_bf16(CUtensorMap* map, void* base, int64_t rows, int64_t cols, int box_cols, int box_rows) {
  EncodeTiledFn fn = get_encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 2-D f32 tensor map over [rows, cols] (row stride cols * 4 bytes, a multiple of 16), box box_cols x box_rows.
static bool make_map_f32(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int box_cols, int box_rows) {
  EncodeTiledFn fn = get_encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 4};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

static int g_num_sms = 0;

// the current device's SM count (queried once)
static int num_sms() {
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
  }
  return g_num_sms;
}

// Output destinations of an affine launch: n buffers of [M, ldo] bf16, this launch's columns starting at col0.
struct OutSpec {
  void* const* ptrs;
  int n;
  int col0;
  int64_t ldo;
};

template <int EPI, int BFMT, bool KPERM, bool GLU = false, int OP = OUT_PLAIN>
static int launch_gemm_t(const int8_t* a, const void* b, const void* rsplit, const GemmArgs& args, cudaStream_t st,
                         const OutSpec* outs = nullptr) {
  auto kern = gemm_kernel<EPI, BFMT, KPERM, GLU, OP>;
  constexpr int smem_bytes = SmemPlan<EPI, BFMT, GLU>::kBytes;
  static bool configured = false;
  static bool regs_ok = false;
  if (!configured) {
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess) return CQ_ERR_CUDA;
    // setmaxnreg redistributes the registers the CTA was launched with: refuse to launch when the launch
    // allocation could not cover the producer/epilogue split (the .inc would otherwise wait forever)
    regs_ok = fa.numRegs * kThreads >= 256 * kProducerRegs + 256 * kEpilogueRegs;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes) != cudaSuccess)
      return CQ_ERR_CUDA;
    configured = true;
  }
  if (!regs_ok) return CQ_ERR_CUDA;
  if (num_sms() <= 0) return CQ_ERR_CUDA;
  CUtensorMap tm_x, tm_w, tm_r, tm_z;
  OutMaps tm_out;
  if (!make_map_u8(&tm_x, a, args.M, args.K, kBK, kBT, true)) return CQ_ERR_CUDA;
  if (EPI == EPI_AFFINE) {
    if (!make_map_u8(&tm_r, rsplit, args.M, 2 * rsplit_cols(args.K), 128, kBT, true)) return CQ_ERR_CUDA;
    // prepared zeros Zt [N, 64 * nz] bf16 as bytes: 128-byte column blocks, 128 weight rows, operand swizzle
    if (!make_map_u8(&tm_z, args.zt, args.N, 128 * static_cast<int64_t>(args.nz), 128, kBW, true)) return CQ_ERR_CUDA;
  } else {
    tm_r = tm_x;   // unused
    tm_z = tm_x;
  }
  if (BFMT == BF_S8) {
    if (!make_map_u8(&tm_w, b, args.N, args.K, kBK, kBW, true)) return CQ_ERR_CUDA;
  } else {
    if (!make_map_u8(&tm_w, b, args.N, args.K / 2, kBK / 2, kBW, false)) return CQ_ERR_CUDA;
  }
  GemmArgs ga = args;
  ga.tma_out = 0;
  ga.n_out = 0;
  ga.out_col0 = 0;
  std::memset(&tm_out, 0, sizeof(tm_out));
  // box = one store pass: 64 tokens x 32 columns (one epilogue warp).  Column-parallel launches, whose boxes also
  // cross NVLink, use 64 x 64 boxes (128-byte rows, two epilogue warps) when their N is a multiple of 64 (a box
  // never reaches into another rank's columns).  Measured for the local output: the pairing costs ~10 %.
  ga.out_w64 = (outs != nullptr && args.N % 64 == 0) ? 1 : 0;
  const int box_cols = ga.out_w64 ? 64 : 32;
  if (EPI == EPI_AFFINE && outs != nullptr) {
    for (int i = 0; i < outs->n; ++i)
      if (!make_map_bf16(&tm_out.m[i], outs->ptrs[i], args.M, outs->ldo, box_cols, 64)) return CQ_ERR_CUDA;
    ga.tma_out = 1;
    ga.n_out = outs->n;
    ga.out_col0 = outs->col0;
  } else if (EPI == EPI_AFFINE && args.N % 8 == 0 && (reinterpret_cast<uintptr_t>(args.out) & 15u) == 0) {
    if (!make_map_bf16(&tm_out.m[0], args.out, args.M, args.N, box_cols, 64)) return CQ_ERR_CUDA;
    ga.tma_out = 1;
    ga.n_out = 1;
  }
  const int tiles = ((args.M + kBT - 1) / kBT) * ((args.N + kBW - 1) / kBW);
  // Half tiles for a partial last wave: with R = tiles mod SMs whole tiles left after the full waves, running them
  // as 2R half tiles ends the launch half a tile earlier whenever 2R <= SMs (R > SMs / 2 gains nothing at half-tile
  // granularity).  With fewer tiles than SMs, all tiles split when that at most fills the SMs.
  int split = 0;
  if (EPI == EPI_ROWCOL) {
    if (tiles < g_num_sms) split = 2 * tiles <= g_num_sms ? tiles : 0;
    else if (2 * (tiles % g_num_sms) <= g_num_sms) split = tiles % g_num_sms;
  }
  ga.split = split;
  if (EPI != EPI_AFFINE) ga.ksplit = 1;
  const int items = tiles * (ga.ksplit > 1 ? ga.ksplit : 1) + split;
  const int grid = items < g_num_sms ? items : g_num_sms;
  if (grid == 0) return CQ_OK;
  if (ga.pdl) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem_bytes;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, tm_x, tm_w, tm_r, tm_z, tm_out, ga) != cudaSuccess) return CQ_ERR_CUDA;
  } else {
    kern<<<grid, kThreads, smem_bytes, st>>>(tm_x, tm_w, tm_r, tm_z, tm_out, ga);
  }
  if (EPI == EPI_AFFINE && ga.ksplit > 1) {
    const int64_t threads = static_cast<int64_t>(ga.M) * (ga.N / 8);
    splitk_finalize_kernel<OP><<<static_cast<unsigned>((threads + 255) / 256), 256, 0, st>>>(ga);
  }
  return cudaGetLastError() == cudaSuccess ? CQ_OK : CQ_ERR_CUDA;
}

}  // namespace cq
