// Packed-int4-weight x int8-activation GEMM with fused dequant epilogue, sm_100a (tcgen05 kind::i8).
//
// Orientation: the MMA computes D[n, m] = sum_k W[n, k] * X[m, k] with the WEIGHT tile on the tensor core's
// M side (128 weight rows = the 128 TMEM lanes) and 256 tokens on its N side (TMEM columns).  Each epilogue
// thread therefore owns one weight row n: the per-group weight scale s[g, n] and zero z[g, n] are per-thread
// scalars, and only the per-token terms (activation scale, code sums) are broadcast loads.
//
// Per CTA (persistent, one per SM, 384 threads):
//   warp 0      TMA producer: activation tile [256 tokens x 128 B] (128-byte swizzle) and the packed weight
//               tile [128 rows x 64 B] per 128-wide K block, into a 3-stage shared-memory ring;
//   warp 1      MMA issuer: 4 x tcgen05.mma (128 x 256 x 32) per K block into a double-buffered TMEM
//               accumulator (2 x 256 columns); tcgen05.commit releases the stage and hands buffers over;
//   warps 2-3   converters: unpack int4 -> int8 in shared memory into the tensor core's K-major 128-byte
//               swizzled layout (nibble v becomes the byte 16*v: one shift/mask per word, the 1/16 is folded
//               into the weight scale), then fence.proxy.async and arrive;
//   warps 4-11  epilogue: tcgen05.ld the int32 partial sums.  Affine weights (per 128-group scale/zero) drain
//               every group into fp32 registers: acc += s[g,n] * P_g + z[g,n] * R[g,m]; row/col weights drain
//               once per tile.  Output bf16 [M, N] row-major.
// Every mbarrier wait is bounded (see cq_common.cuh).  No cluster launch, no multicast.
#include <cstdio>
#include <cstring>

#include "kernels.cuh"

namespace cq {

constexpr int kBW = 128;       // weight rows per tile (MMA M, TMEM lanes)
constexpr int kBT = 256;       // tokens per tile (MMA N, TMEM columns per accumulator buffer)
constexpr int kBK = 128;       // K elements (bytes of int8) per stage
constexpr int kStages = 3;
constexpr int kThreads = 384;
constexpr int kXBytes = kBT * kBK;          // 32 KB
constexpr int kWuBytes = kBW * kBK;         // 16 KB
constexpr int kWpBytes = kBW * kBK / 2;     //  8 KB
constexpr int kSmemData = kStages * (kXBytes + kWuBytes + kWpBytes);
constexpr int kSmemBytes = kSmemData + 1024 /*align slack*/ + 256 /*barriers*/;
constexpr int kProducerRegs = 80;
constexpr int kEpilogueRegs = 208;

enum : int { EPI_ROWCOL = 0, EPI_AFFINE = 1 };
enum : int { BF_S4 = 0, BF_U4 = 1, BF_S8 = 2 };

struct GemmArgs {
  const float* sa;       // [M] activation scale
  const float* gsum;     // [K/128, gsum_ld] code sums (affine)
  int64_t gsum_ld;
  const float* sb;       // [N] weight scale (rowcol)
  const __nv_bfloat16* ws;  // [K/128, N] bf16 (affine)
  const __nv_bfloat16* wz;  // [K/128, N] bf16 (affine)
  const __nv_bfloat16* bias;  // [N] or null
  __nv_bfloat16* out;    // [M, N]
  int M, N, K;
};

__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProducerRegs));
}
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kEpilogueRegs));
}

// 8 packed bytes (16 nibbles, low nibble = even column) -> 16 bytes holding 16*v per column.
template <int BFMT>
__device__ __forceinline__ uint4 unpack16(uint2 p) {
  const uint32_t flip = (BFMT == BF_U4) ? 0x80808080u : 0u;   // uint4 q -> signed (q - 8): flip the top bit
  const uint32_t lo0 = ((p.x << 4) & 0xF0F0F0F0u) ^ flip, hi0 = (p.x & 0xF0F0F0F0u) ^ flip;
  const uint32_t lo1 = ((p.y << 4) & 0xF0F0F0F0u) ^ flip, hi1 = (p.y & 0xF0F0F0F0u) ^ flip;
  return make_uint4(prmt(lo0, hi0, 0x5140u), prmt(lo0, hi0, 0x7362u), prmt(lo1, hi1, 0x5140u),
                    prmt(lo1, hi1, 0x7362u));
}

template <int EPI, int BFMT>
__global__ void __launch_bounds__(kThreads, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w, const GemmArgs args) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sm_x = smem;                                   // [kStages][kXBytes]
  uint8_t* sm_wu = smem + kStages * kXBytes;              // [kStages][kWuBytes]
  uint8_t* sm_wp = sm_wu + kStages * kWuBytes;            // [kStages][kWpBytes]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kSmemData);
  uint64_t* full_tma = bars;
  uint64_t* full_conv = bars + kStages;
  uint64_t* empty = bars + 2 * kStages;
  uint64_t* tmem_full = bars + 3 * kStages;
  uint64_t* tmem_empty = bars + 3 * kStages + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 3 * kStages + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int M = args.M, N = args.N, K = args.K;
  const int kblocks = K / kBK;
  const int m_tiles = (M + kBT - 1) / kBT;
  const int n_tiles = (N + kBW - 1) / kBW;
  const int num_tiles = m_tiles * n_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_tma[s], 1);
      mbar_init(&full_conv[s], 2);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tmem_full[b], 1);
      mbar_init(&tmem_empty[b], 8);
    }
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tensormap(&tm_x);
    prefetch_tensormap(&tm_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp < 4) {
    setmaxnreg_dec();
    if (warp == 0 && lane == 0) {
      // ------------------------------ TMA producer ------------------------------
      int stage = 0;
      uint32_t phase = 0;
      const uint32_t bytes = kXBytes + (BFMT == BF_S8 ? kWuBytes : kWpBytes);
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
        const int m0 = (tile % m_tiles) * kBT;
        const int n0 = (tile / m_tiles) * kBW;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, 1)) break;
          mbar_arrive_expect_tx(&full_tma[stage], bytes);
          tma_load_2d(sm_x + stage * kXBytes, &tm_x, &full_tma[stage], kb * kBK, m0);
          if (BFMT == BF_S8) tma_load_2d(sm_wu + stage * kWuBytes, &tm_w, &full_tma[stage], kb * kBK, n0);
          else tma_load_2d(sm_wp + stage * kWpBytes, &tm_w, &full_tma[stage], kb * (kBK / 2), n0);
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
      }
    } else if (warp == 1 && lane == 0) {
      // ------------------------------ MMA issuer ------------------------------
      constexpr uint32_t idesc = idesc_i8(kBW, kBT);
      int stage = 0;
      uint32_t phase = 0;
      int buf = 0;
      uint32_t buf_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (EPI == EPI_ROWCOL) {
          if (!(ok = mbar_wait(&tmem_empty[buf], buf_phase ^ 1u, abort_flag, 2))) break;
          tc_fence_after();
        }
        for (int kb = 0; kb < kblocks && ok; ++kb) {
          if (EPI == EPI_AFFINE) {
            if (!(ok = mbar_wait(&tmem_empty[buf], buf_phase ^ 1u, abort_flag, 3))) break;
            tc_fence_after();
          }
          if (!(ok = mbar_wait(&full_tma[stage], phase, abort_flag, 4))) break;
          if (BFMT != BF_S8 && !(ok = mbar_wait(&full_conv[stage], phase, abort_flag, 5))) break;
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * kBT);
          const uint32_t a_base = smem_u32(sm_wu + stage * kWuBytes);
          const uint32_t b_base = smem_u32(sm_x + stage * kXBytes);
#pragma unroll
          for (int k = 0; k < kBK / 32; ++k) {
            const uint32_t acc = (EPI == EPI_AFFINE) ? (k > 0) : (kb > 0 || k > 0);
            mma_i8(d_tmem, smem_desc_k_sw128(a_base + 32 * k), smem_desc_k_sw128(b_base + 32 * k), idesc, acc);
          }
          tc_commit(&empty[stage]);
          if (EPI == EPI_AFFINE) {
            tc_commit(&tmem_full[buf]);
            if (++buf == 2) { buf = 0; buf_phase ^= 1u; }
          }
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
        if (EPI == EPI_ROWCOL && ok) {
          tc_commit(&tmem_full[buf]);
          if (++buf == 2) { buf = 0; buf_phase ^= 1u; }
        }
      }
    } else if (warp >= 2 && BFMT != BF_S8) {
      // ------------------------------ int4 -> int8 converters ------------------------------
      const int ct = threadIdx.x - 64;   // 0..63
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!(ok = mbar_wait(&full_tma[stage], phase, abort_flag, 6))) break;
          const uint8_t* src = sm_wp + stage * kWpBytes;
          uint8_t* dst = sm_wu + stage * kWuBytes;
#pragma unroll 4
          for (int it = ct; it < kBW * 8; it += 64) {
            const int r = it >> 3, c = it & 7;
            const uint2 p = *reinterpret_cast<const uint2*>(src + r * 64 + c * 8);
            *reinterpret_cast<uint4*>(dst + r * 128 + ((c ^ (r & 7)) << 4)) = unpack16<BFMT>(p);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&full_conv[stage]);
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
      }
    }
  } else {
    // ------------------------------ epilogue (warps 4..11) ------------------------------
    setmaxnreg_inc();
    const int e = warp - 4;
    const int quad = warp & 3;            // TMEM lane quadrant this warp may access
    const int half = e >> 2;              // token half of the tile: columns [128*half, 128*half + 128)
    const uint32_t lane_addr = static_cast<uint32_t>(32 * quad) << 16;
    // the int4 unpack stores 16*v; fold the 1/16 into the weight scale (exact)
    const float wscale_fold = (BFMT == BF_S8) ? 1.0f : 0.0625f;
    int buf = 0;
    uint32_t buf_phase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      const int m0 = (tile % m_tiles) * kBT + half * 128;
      const int n = (tile / m_tiles) * kBW + quad * 32 + lane;
      const bool n_ok = n < N;
      const float bias = (args.bias != nullptr && n_ok) ? __bfloat162float(args.bias[n]) : 0.0f;
      if (EPI == EPI_AFFINE) {
        float acc[128];
#pragma unroll
        for (int j = 0; j < 128; ++j) acc[j] = 0.0f;
        for (int g = 0; g < kblocks; ++g) {
          if (!(ok = mbar_wait(&tmem_full[buf], buf_phase, abort_flag, 7))) break;
          tc_fence_after();
          const float s = n_ok ? __bfloat162float(args.ws[static_cast<int64_t>(g) * N + n]) * wscale_fold : 0.0f;
          const float z = n_ok ? __bfloat162float(args.wz[static_cast<int64_t>(g) * N + n]) : 0.0f;
          const uint32_t taddr = tmem_base + lane_addr + static_cast<uint32_t>(buf * kBT + half * 128);
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(taddr + 32 * ch, r);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j)
              acc[32 * ch + j] = __fmaf_rn(s, __int2float_rn(static_cast<int>(r[j])), acc[32 * ch + j]);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tmem_empty[buf]);
          if (++buf == 2) { buf = 0; buf_phase ^= 1u; }
          // zero-point term: z[g, n] * (sum of token m's codes over group g)
          const float* gs = args.gsum + static_cast<int64_t>(g) * args.gsum_ld + m0;
#pragma unroll
          for (int j4 = 0; j4 < 32; ++j4) {
            const float4 rs = (m0 + 4 * j4 < M) ? *reinterpret_cast<const float4*>(gs + 4 * j4) : make_float4(0, 0, 0, 0);
            acc[4 * j4 + 0] = __fmaf_rn(z, rs.x, acc[4 * j4 + 0]);
            acc[4 * j4 + 1] = __fmaf_rn(z, rs.y, acc[4 * j4 + 1]);
            acc[4 * j4 + 2] = __fmaf_rn(z, rs.z, acc[4 * j4 + 2]);
            acc[4 * j4 + 3] = __fmaf_rn(z, rs.w, acc[4 * j4 + 3]);
          }
        }
        if (!ok) break;
#pragma unroll
        for (int j = 0; j < 128; ++j) {
          const int m = m0 + j;
          if (m < M && n_ok) {
            const float y = __fmaf_rn(acc[j], args.sa[m], bias);
            args.out[static_cast<int64_t>(m) * N + n] = __float2bfloat16_rn(y);
          }
        }
      } else {
        if (!(ok = mbar_wait(&tmem_full[buf], buf_phase, abort_flag, 8))) break;
        tc_fence_after();
        const float sb = n_ok ? args.sb[n] * wscale_fold : 0.0f;
        const uint32_t taddr = tmem_base + lane_addr + static_cast<uint32_t>(buf * kBT + half * 128);
#pragma unroll 1
        for (int ch = 0; ch < 4; ++ch) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(taddr + 32 * ch, r);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int m = m0 + 32 * ch + j;
            if (m < M && n_ok) {
              const float y = __fmaf_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[j])), sb), args.sa[m], bias);
              args.out[static_cast<int64_t>(m) * N + n] = __float2bfloat16_rn(y);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tmem_empty[buf]);
        if (++buf == 2) { buf = 0; buf_phase ^= 1u; }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem_base, 512);
  }
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

static int g_num_sms = 0;

template <int EPI, int BFMT>
static int launch_gemm_t(const int8_t* a, const void* b, const GemmArgs& args, cudaStream_t st) {
  auto kern = gemm_kernel<EPI, BFMT>;
  static bool configured = false;
  static bool regs_ok = false;
  if (!configured) {
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess) return CQ_ERR_CUDA;
    // setmaxnreg redistributes the registers the CTA was launched with: refuse to launch when the launch
    // allocation could not cover the producer/epilogue split (the .inc would otherwise wait forever)
    regs_ok = fa.numRegs * kThreads >= 128 * kProducerRegs + 256 * kEpilogueRegs;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) != cudaSuccess)
      return CQ_ERR_CUDA;
    configured = true;
  }
  if (!regs_ok) return CQ_ERR_CUDA;
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) return CQ_ERR_CUDA;
  }
  CUtensorMap tm_x, tm_w;
  if (!make_map_u8(&tm_x, a, args.M, args.K, kBK, kBT, true)) return CQ_ERR_CUDA;
  if (BFMT == BF_S8) {
    if (!make_map_u8(&tm_w, b, args.N, args.K, kBK, kBW, true)) return CQ_ERR_CUDA;
  } else {
    if (!make_map_u8(&tm_w, b, args.N, args.K / 2, kBK / 2, kBW, false)) return CQ_ERR_CUDA;
  }
  const int tiles = ((args.M + kBT - 1) / kBT) * ((args.N + kBW - 1) / kBW);
  const int grid = tiles < g_num_sms ? tiles : g_num_sms;
  if (grid == 0) return CQ_OK;
  kern<<<grid, kThreads, kSmemBytes, st>>>(tm_x, tm_w, args);
  return cudaGetLastError() == cudaSuccess ? CQ_OK : CQ_ERR_CUDA;
}

int launch_gemm_rowcol(const int8_t* a, const float* sa, const void* b, int b_format, const float* sb,
                       const void* bias, void* out, int M, int N, int K, cudaStream_t st) {
  GemmArgs g{};
  g.sa = sa;
  g.sb = sb;
  g.bias = static_cast<const __nv_bfloat16*>(bias);
  g.out = static_cast<__nv_bfloat16*>(out);
  g.M = M; g.N = N; g.K = K;
  if (b_format == CQ_B_INT8) return launch_gemm_t<EPI_ROWCOL, BF_S8>(a, b, g, st);
  return launch_gemm_t<EPI_ROWCOL, BF_S4>(a, b, g, st);
}

int launch_gemm_affine(const int8_t* a, const float* sa, const float* gsum, int64_t gsum_ld, const void* b,
                       const void* s, const void* z, const void* bias, void* out, int M, int N, int K,
                       cudaStream_t st) {
  GemmArgs g{};
  g.sa = sa;
  g.gsum = gsum;
  g.gsum_ld = gsum_ld;
  g.ws = static_cast<const __nv_bfloat16*>(s);
  g.wz = static_cast<const __nv_bfloat16*>(z);
  g.bias = static_cast<const __nv_bfloat16*>(bias);
  g.out = static_cast<__nv_bfloat16*>(out);
  g.M = M; g.N = N; g.K = K;
  return launch_gemm_t<EPI_AFFINE, BF_U4>(a, b, g, st);
}

}  // namespace cq
