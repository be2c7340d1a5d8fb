// 2-SM (CTA pair) form of the packed-int4-weight x int8-activation GEMM, sm_100a (tcgen05 cta_group::2).
//
// A cluster of two CTAs computes a 256-weight-row x 256-token tile with one tcgen05.mma.cta_group::2 stream issued
// by the even CTA (the leader).  CTA r holds weight rows [128 r, 128 r + 128) of the tile (its A operand, the M side)
// and loads the activation rows of tokens [128 r, 128 r + 128) (its half of the B operand, the N side); the tensor
// cores of the pair read each B half once and both accumulate all 256 tokens for their own weight rows, so each SM
// reads 32 KB of operands from shared memory per 128-wide K block instead of 48 KB, and its activation stages are
// half as large, which buys a deeper load ring.  Each CTA's TMEM holds its 128 weight rows x 256 tokens in two
// 256-column accumulator buffers, exactly the layout of the one-SM kernel, so the epilogue is the same code.
//
// Per CTA (persistent, one per SM, 512 threads):
//   warp 0      TMA producer: this CTA's packed weight tile [128 rows x 64 B] into a weight ring and its token
//               half [128 tokens x 128 B] into an activation ring (split group sums for the affine zero-point pass
//               ride in the activation ring);
//   warp 1      leader: MMA issuer (two barriers per block: the accumulator buffer and the operands, probed together);
//   warps 2-5   converters: unpack int4 -> int8 from the weight ring into a 4-stage converter ring (one warp per
//               stage, each taking every fourth block; warps 2-5 sit on the four SM sub-partitions, so the integer
//               pipe work of the unpack is spread evenly beside the epilogue's), release the weight stage, wait for
//               the block's activation stage of their own CTA, then arrive on the leader's operand barrier, which
//               thus stands for both halves of B and both CTAs' converted A;
//   warps 6-7   idle (they keep the 512-thread register split of the one-SM kernel);
//   warps 8-15  epilogue, as in the one-SM kernel; buffers are handed back to the leader by remote arrivals.
// The leader's tcgen05.commit goes to both CTAs (multicast commit), so each CTA's producer, converters and
// epilogue wait on their own barriers.  Every wait is bounded; on an abort the producer waits (bounded) for its
// issued loads, the leader for its issued MMAs, and the two CTAs exchange an exit arrival before the collective TMEM
// release, so neither CTA's memory goes away under the other's operations.  Loads are plain per-CTA TMA copies
// (no multicast); only tcgen05.commit uses the cluster multicast form.
#include "kernels.cuh"

namespace cq {
namespace pr {

constexpr int kRowsCta = 128;          // weight rows per CTA (TMEM lanes); the pair covers 256
constexpr int kRowsPair = 2 * kRowsCta;
constexpr int kTok = 256;              // tokens per pair tile (MMA N; TMEM columns per accumulator buffer); 128 (four
                                       // buffers) also builds and passes, but measured 1.5x slower at the T shape
constexpr int kTokCta = kTok / 2;      // tokens whose activation rows one CTA loads
constexpr int kBK = 128;
constexpr int kBufs = 512 / kTok;     // accumulator buffers in the 512 TMEM columns
constexpr int kWarpTok = kTok / 2;     // tokens per epilogue warp (two warps per TMEM lane quadrant)
constexpr int kChunks = kWarpTok / 32;
constexpr int kConvStages = 4;        // one converter warp per stage (warps 2..5)
constexpr int kConvWarp0 = 2;
constexpr int kTmemWarp = 6;           // allocates and releases the pair's TMEM (warps 6-7 have no other role)
constexpr int kRoleWarps = 14;         // warps 0, 1, the 4 converters and the 8 epilogue warps
constexpr int kThreads = 512;
constexpr int kEpiWarp0 = 8;
constexpr int kXBytes = kTokCta * kBK;          // 16 KB
constexpr int kWpBytes = kRowsCta * kBK / 2;    //  8 KB packed int4
constexpr int kWuBytes = kRowsCta * kBK;        // 16 KB unpacked
constexpr int kWStages = 6;
constexpr unsigned long long kDrainNs = 50000000ull;   // per wait while unwinding (50 ms)

// per-group drains (affine and group scales) keep the output staging of the TMA stores
template <int EPI>
constexpr bool kPerGroup = (EPI == EPI_AFFINE || EPI == EPI_GROUP);
// every group's partial sum in its own accumulator buffer (the integer-ratio epilogue too)
template <int EPI>
constexpr bool kDrainPerGroup = kPerGroup<EPI> || EPI == EPI_INTRATIO;
constexpr int kSgStages = 4;                   // group epilogue: ring of per-group token scales
constexpr int kSgBytes = kTok * 4;             //   one stage: the tile's tokens' scales of one group (f32)

template <int EPI>
struct Plan {
  static constexpr int kXStages = kPerGroup<EPI> ? (kTok == 256 ? 4 : 8) : (kTok == 256 ? 6 : 10);
  static constexpr int kX = 0;
  static constexpr int kW = kX + kXStages * kXBytes;
  static constexpr int kConv = kW + kWStages * kWpBytes;
  static constexpr int kBars = kConv + kConvStages * kWuBytes;
  static constexpr int kBarBytes = 1024;
  static constexpr int kSa = kBars + kBarBytes;
  static constexpr int kSaBytes = 8 * kWarpTok * 4;
  static constexpr int kOut = kSa + kSaBytes;
  static constexpr int kOutWarpBytes = 64 * 32 * 2;
  static constexpr int kOutBytes = kPerGroup<EPI> ? 8 * kOutWarpBytes : 0;
  static constexpr int kSg = kOut + kOutBytes;
  static constexpr int kSgRingBytes = (EPI == EPI_GROUP) ? kSgStages * kSgBytes : 0;
  static constexpr int kBytes = kSg + kSgRingBytes + 1024 /*align slack*/;
};


template <int EPI, int BFMT, bool KPERM, bool GLU, int OP>
__global__ void __launch_bounds__(kThreads, 1)
gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                 const __grid_constant__ CUtensorMap tm_r, const __grid_constant__ CUtensorMap tm_z,
                 const __grid_constant__ OutMaps tm_out, const GemmArgs args) {
  using P = Plan<EPI>;
  static_assert(BFMT == BF_U4 || BFMT == BF_S4, "the pair kernel converts packed int4 weights");
  static_assert(!GLU || EPI == EPI_ROWCOL, "the SwiGLU output is a row/col epilogue");
  static_assert(OP == OUT_PLAIN || EPI == EPI_AFFINE || (EPI == EPI_ROWCOL && !GLU),
                "output operations are affine or plain row/col epilogue variants");
  constexpr int kXS = P::kXStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sm_x = smem + P::kX;
  uint8_t* sm_w = smem + P::kW;
  uint8_t* sm_conv = smem + P::kConv;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P::kBars);
  uint64_t* full_x = bars;                        // [kXS] this CTA's activation stage landed (TMA)
  uint64_t* empty_x = full_x + kXS;               // [kXS] the MMAs that read it completed (multicast commit)
  uint64_t* full_w = empty_x + kXS;               // [kWStages] weight stage landed (TMA)
  uint64_t* empty_w = full_w + kWStages;          // [kWStages] converted (the converter warp that read it)
  uint64_t* full_conv = empty_w + kWStages;       // [4] leader only: both CTAs' operands of the block are in place
  uint64_t* empty_conv = full_conv + kConvStages; // [4] the MMAs that read it completed (multicast commit)
  uint64_t* zt_full = empty_conv + kConvStages;   // [4] affine: the zero-point operand landed (TMA)
  uint64_t* tmem_full = zt_full + kConvStages;    // [2] accumulator buffer ready (multicast commit)
  uint64_t* tmem_empty = tmem_full + kBufs;       // [2] leader only: all 16 epilogue warps of the pair drained it
  uint64_t* box_free = tmem_empty + kBufs;        // [4] affine, 64-column boxes (see the one-SM kernel)
  uint64_t* box_full = box_free + 4;              // [4]
  uint64_t* mma_done = box_full + 4;              // [1] the leader's last commit: every MMA of the pair completed
  uint64_t* exit_bar = mma_done + 1;              // [1] the peer CTA finished with the pair's memory
  uint64_t* sg_full = exit_bar + 1;               // [4] group: a group's token scales landed (TMA)
  uint64_t* sg_empty = sg_full + kSgStages;       // [4] group: the 8 epilogue warps used them
  uint64_t* cta_done = sg_empty + kSgStages;      // [1] every role warp of this CTA finished (14 arrivals)
  const float* sm_sg = reinterpret_cast<const float*>(smem + P::kSg);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(cta_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  static_assert((2 * kXS + 2 * kWStages + 3 * kConvStages + 2 * kBufs + 11 + 2 * kSgStages) * 8 + 8 <= P::kBarBytes,
                "barriers, the TMEM address and the abort flag fit their region");

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();      // 0: leader (issues the MMAs), 1: peer
  const int pair_id = static_cast<int>(blockIdx.x >> 1);
  const int num_pairs = static_cast<int>(gridDim.x >> 1);
  const int M = args.M, N = args.N, K = args.K;
  const int kblocks = K / kBK;
  const int m_tiles = (M + kTok - 1) / kTok;
  const int n_tiles = (N + kRowsPair - 1) / kRowsPair;
  const int num_tiles = m_tiles * n_tiles;
  const int nzb = (EPI == EPI_AFFINE) ? args.nz : 0;   // zero-point pseudo blocks per tile

  if (threadIdx.x == 0) {
    for (int s = 0; s < kXS; ++s) {
      mbar_init(&full_x[s], 1);
      mbar_init(&empty_x[s], 1);
    }
    for (int s = 0; s < kWStages; ++s) {
      mbar_init(&full_w[s], 1);
      mbar_init(&empty_w[s], 1);
    }
    for (int c = 0; c < kConvStages; ++c) {
      mbar_init(&full_conv[c], 2);      // the stage's converter warp in each CTA
      mbar_init(&empty_conv[c], 1);
      mbar_init(&zt_full[c], 1);
    }
    for (int b = 0; b < kBufs; ++b) {
      mbar_init(&tmem_full[b], 1);
      mbar_init(&tmem_empty[b], 16);    // 8 epilogue warps x 2 CTAs
    }
    for (int p = 0; p < 4; ++p) {
      mbar_init(&box_free[p], 1);
      mbar_init(&box_full[p], 2);
    }
    mbar_init(mma_done, 1);
    mbar_init(exit_bar, 1);
    mbar_init(cta_done, kRoleWarps);
    for (int q = 0; q < kSgStages; ++q) {
      mbar_init(&sg_full[q], 1);
      mbar_init(&sg_empty[q], 8);
    }
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tensormap(&tm_x);
    prefetch_tensormap(&tm_w);
    if (EPI == EPI_GROUP) prefetch_tensormap(&tm_r);
    if (EPI == EPI_AFFINE) {
      prefetch_tensormap(&tm_r);
      prefetch_tensormap(&tm_z);
      if (args.tma_out)
        for (int i = 0; i < args.n_out; ++i) prefetch_tensormap(&tm_out.m[i]);
    }
  }
  if (warp == kTmemWarp) {
    tmem_alloc_pair(tmem_holder, 512);   // collective: this warp of each CTA of the pair
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  // both CTAs' barriers are initialized before any remote arrival (the two CTAs of a cluster run together)
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  grid_dep_wait();   // inputs written by the previous kernel (programmatic launch) are visible from here on

  if (warp < kEpiWarp0) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProducerRegs));
    // Lanes with no role leave now (the CTA's closing barrier waits only for threads that have not exited): a warp
    // whose lane 0 loops while its other lanes sit at that barrier measurably delayed the epilogue warps of its SM
    // sub-partition.  Warp kTmemWarp stays whole for the collective TMEM release at the end.
    if ((warp <= 1 && lane != 0) || (warp > kConvWarp0 + kConvStages - 1 && warp != kTmemWarp)) return;
    if (warp == 0 && lane == 0) {
      // ------------------------------ TMA producer ------------------------------
      int xs = 0, ws = 0, gs = 0;
      uint32_t xph = 0, wph = 0, gph = 0, x_issued = 0, w_issued = 0, g_issued = 0;
      bool ok = true;
      for (int item = pair_id; item < num_tiles && ok; item += num_pairs) {
        int mt, nt;
        tile_coords(item, m_tiles, n_tiles, mt, nt);
        const int m0 = mt * kTok + static_cast<int>(rank) * kTokCta;       // this CTA's token half
        const int n0 = nt * kRowsPair + static_cast<int>(rank) * kRowsCta;  // this CTA's weight rows
        for (int p = 0; p < nzb && ok; ++p) {
          // zero-point operand: the tokens' split group sums (bf16, 64 columns per block) into the activation ring
          if (!(ok = mbar_wait(&empty_x[xs], xph ^ 1u, abort_flag, 40))) break;
          mbar_arrive_expect_tx(&full_x[xs], kXBytes);
          tma_load_2d(sm_x + xs * kXBytes, &tm_r, &full_x[xs], p * 128, m0);
          ++x_issued;
          if (++xs == kXS) { xs = 0; xph ^= 1u; }
        }
        for (int kb = 0; kb < kblocks && ok; ++kb) {
          if (!(ok = mbar_wait(&empty_w[ws], wph ^ 1u, abort_flag, 41))) break;
          mbar_arrive_expect_tx(&full_w[ws], kWpBytes);
          tma_load_2d(sm_w + ws * kWpBytes, &tm_w, &full_w[ws], kb * (kBK / 2), n0);
          ++w_issued;
          if (++ws == kWStages) { ws = 0; wph ^= 1u; }
          if (!(ok = mbar_wait(&empty_x[xs], xph ^ 1u, abort_flag, 42))) break;
          mbar_arrive_expect_tx(&full_x[xs], kXBytes);
          tma_load_2d(sm_x + xs * kXBytes, &tm_x, &full_x[xs], kb * kBK, m0);
          ++x_issued;
          if (++xs == kXS) { xs = 0; xph ^= 1u; }
          if (EPI == EPI_GROUP) {
            // group kb's scales of the tile's 256 tokens (both CTAs' epilogues cover all of them)
            if (!(ok = mbar_wait(&sg_empty[gs], gph ^ 1u, abort_flag, 43))) break;
            mbar_arrive_expect_tx(&sg_full[gs], kSgBytes);
            tma_load_2d(const_cast<float*>(sm_sg) + gs * kTok, &tm_r, &sg_full[gs], mt * kTok, kb);
            ++g_issued;
            if (++gs == kSgStages) { gs = 0; gph ^= 1u; }
          }
        }
      }
      // every load issued has landed before this CTA's shared memory can be released (a no-op on a normal end)
      drain_ring(full_x, kXS, x_issued, kDrainNs);
      drain_ring(full_w, kWStages, w_issued, kDrainNs);
      if (EPI == EPI_GROUP) drain_ring(sg_full, kSgStages, g_issued, kDrainNs);
    } else if (warp == 1 && lane == 0 && rank == 0) {
      // ------------------------------ MMA issuer (leader) ------------------------------
      const uint32_t idesc = idesc_i8(kRowsPair, kTok);
      const uint32_t idesc_z = idesc_bf16(kRowsPair, kTok);
      int xs = 0, cs = 0, buf = 0;
      uint32_t xph = 0, cph = 0, bph = 0;
      bool ok = true;
      // The accumulator buffer and the block's operands: both ready is the common case, probed in one round trip.
      auto buffer_and_operands_ready = [&](int where) -> bool {
        if (mbar_test_wait2(&tmem_empty[buf], bph, &full_conv[cs], cph)) return true;
        return mbar_wait(&tmem_empty[buf], bph, abort_flag, where) && mbar_wait(&full_conv[cs], cph, abort_flag, where);
      };
      auto operands_ready = [&](int where) -> bool { return mbar_wait(&full_conv[cs], cph, abort_flag, where); };
      auto advance = [&]() {
        if (++xs == kXS) { xs = 0; xph ^= 1u; }
        if (++cs == kConvStages) { cs = 0; cph ^= 1u; }
      };
      for (int item = pair_id; item < num_tiles && ok; item += num_pairs) {
        if (EPI == EPI_AFFINE) {
          // D = sum_j Zt[n, j] * Rsplit[m, j] in fp32: the zero-point term, the accumulator's starting value
          for (int p = 0; p < nzb && ok; ++p) {
            if (!(ok = (p == 0 ? buffer_and_operands_ready(45) : operands_ready(45)))) break;
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * kTok);
            const uint32_t a_base = smem_u32(sm_conv + cs * kWuBytes);
            const uint32_t b_base = smem_u32(sm_x + xs * kXBytes);
#pragma unroll
            for (int k = 0; k < 4; ++k)   // 64 bf16 = 4 x K16
              mma_bf16_pair(d_tmem, smem_desc_k_sw128(a_base + 32 * k), smem_desc_k_sw128(b_base + 32 * k), idesc_z,
                            (p > 0 || k > 0) ? 1u : 0u);
            tc_commit_pair(&empty_x[xs]);
            tc_commit_pair(&empty_conv[cs]);
            advance();
          }
          if (!ok) break;
          tc_commit_pair(&tmem_full[buf]);
          if (++buf == kBufs) { buf = 0; bph ^= 1u; }
        }
        for (int kb = 0; kb < kblocks && ok; ++kb) {
          // affine / group scales / integer ratios: every group has its own accumulator buffer; row/col: one
          // buffer per tile
          const bool new_buf = kDrainPerGroup<EPI> || kb == 0;
          if (!(ok = (new_buf ? buffer_and_operands_ready(46) : operands_ready(47)))) break;
          tc_fence_after();
          const uint32_t a_base = smem_u32(sm_conv + cs * kWuBytes);
          const uint32_t b_base = smem_u32(sm_x + xs * kXBytes);
          if (EPI == EPI_INTRATIO && args.cw_group == 64) {
            // two 64-wide ratio groups per K block, each summed in its own buffer
#pragma unroll
            for (int k = 0; k < kBK / 32; ++k) {
              if (k == 2) {
                tc_commit_pair(&tmem_full[buf]);
                if (++buf == kBufs) { buf = 0; bph ^= 1u; }
                if (!(ok = mbar_wait(&tmem_empty[buf], bph, abort_flag, 49))) break;
                tc_fence_after();
              }
              const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * kTok);
              mma_i8_pair(d_tmem, smem_desc_k_sw128(a_base + 32 * k), smem_desc_k_sw128(b_base + 32 * k), idesc,
                          (k & 1) ? 1u : 0u);
            }
            if (!ok) break;
          } else {
            const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * kTok);
#pragma unroll
            for (int k = 0; k < kBK / 32; ++k) {
              // per-group drains: every 128-wide group starts its own int32 sum
              const uint32_t acc = kDrainPerGroup<EPI> ? (k > 0) : (kb > 0 || k > 0);
              mma_i8_pair(d_tmem, smem_desc_k_sw128(a_base + 32 * k), smem_desc_k_sw128(b_base + 32 * k), idesc, acc);
            }
          }
          tc_commit_pair(&empty_x[xs]);
          tc_commit_pair(&empty_conv[cs]);
          if (kDrainPerGroup<EPI>) {
            tc_commit_pair(&tmem_full[buf]);
            if (++buf == kBufs) { buf = 0; bph ^= 1u; }
          }
          advance();
        }
        if (EPI == EPI_ROWCOL && ok) {
          tc_commit_pair(&tmem_full[buf]);
          if (++buf == kBufs) { buf = 0; bph ^= 1u; }
        }
      }
      // completes when every MMA issued above has completed; both CTAs wait for it before releasing memory
      tc_commit_pair(mma_done);
    } else if (warp >= kConvWarp0 && warp < kConvWarp0 + kConvStages) {
      // ------------------------------ int4 -> int8 converters ------------------------------
      // Warp c converts blocks c, c + 4, c + 8, ... of this CTA's block sequence (per tile: the zero-point pseudo
      // blocks, then the K blocks) into converter stage c.
      const int cw = warp - kConvWarp0;
      const int bpt = nzb + kblocks;
      uint8_t* dst = sm_conv + cw * kWuBytes;
      // item i of a lane: 16 packed bytes (32 K columns) of row (lane >> 2) + 8 i, 16-byte column lane & 3.  Row steps
      // of 8 keep (row & 7), so the swizzled destination chunks sit at fixed offsets from the row start.
      const int rr = lane >> 2, c4 = lane & 3;
      const uint32_t src_off = static_cast<uint32_t>(rr * 64 + c4 * 16);
      uint8_t* const drow0 = dst + rr * 128;
      const uint32_t dlo = static_cast<uint32_t>(((2 * c4) ^ (rr & 7)) << 4);
      const uint32_t dhi = static_cast<uint32_t>(((2 * c4 + 1) ^ (rr & 7)) << 4);
      const uint32_t leader_full_conv = mapa_shared(smem_u32(&full_conv[cw]), 0);
      int item = pair_id, b = cw, t_local = 0;
      uint32_t cph = 0, zph = 0;
      bool ok = true;
      while (b >= bpt) { b -= bpt; item += num_pairs; ++t_local; }
      for (; item < num_tiles && ok; cph ^= 1u) {
        if (!mbar_wait(&empty_conv[cw], cph ^ 1u, abort_flag, 48)) break;
        if (EPI == EPI_AFFINE && b < nzb) {
          // zero-point weight operand: rows of the prepared Zt, 64 bf16 columns per pseudo block, by TMA into the stage
          if (lane == 0) {
            int mt, nt;
            tile_coords(item, m_tiles, n_tiles, mt, nt);
            mbar_arrive_expect_tx(&zt_full[cw], kWuBytes);
            tma_load_2d(dst, &tm_z, &zt_full[cw], 128 * b, nt * kRowsPair + static_cast<int>(rank) * kRowsCta);
          }
          if (!mbar_wait(&zt_full[cw], zph, abort_flag, 49)) {
            if (lane == 0) mbar_wait_drain(&zt_full[cw], zph, kDrainNs);   // the issued load lands first
            break;
          }
          zph ^= 1u;
        } else {
          const int wq = t_local * kblocks + (b - nzb);   // index of this block in the weight ring's sequence
          const int ws = wq % kWStages;
          const uint32_t wph = static_cast<uint32_t>(wq / kWStages) & 1u;
          if (!mbar_wait(&full_w[ws], wph, abort_flag, 50)) break;
          const uint8_t* src = sm_w + ws * kWpBytes + src_off;
#pragma unroll 4
          for (int i = 0; i < kRowsCta / 8; ++i) {
            const uint4 p = *reinterpret_cast<const uint4*>(src + i * 512);
            *reinterpret_cast<uint4*>(drow0 + i * 1024 + dlo) = unpack16<BFMT, KPERM>(make_uint2(p.x, p.y));
            *reinterpret_cast<uint4*>(drow0 + i * 1024 + dhi) = unpack16<BFMT, KPERM>(make_uint2(p.z, p.w));
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty_w[ws]);
        }
        fence_proxy_async_smem();
        // the block's activation stage of this CTA (the B half its tensor core contributes) has landed too
        const int xq = t_local * bpt + b;
        if (lane == 0) ok = mbar_wait(&full_x[xq % kXS], static_cast<uint32_t>(xq / kXS) & 1u, abort_flag, 56);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        if (lane == 0) mbar_arrive_cluster(leader_full_conv);
        b += kConvStages;
        while (b >= bpt) { b -= bpt; item += num_pairs; ++t_local; }
      }
    }
  } else {
    // ------------------------------ epilogue (warps 8..15) ------------------------------
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kEpilogueRegs));
    const int e = warp - kEpiWarp0;
    const int quad = warp & 3;            // TMEM lane quadrant this warp may access
    const int half = e >> 2;              // token half of the tile: columns [128*half, 128*half + 128)
    const uint32_t lane_addr = static_cast<uint32_t>(32 * quad) << 16;
    const uint32_t leader_tmem_empty = mapa_shared(smem_u32(tmem_empty), 0);
    const float wscale_fold = 0.0625f;    // the int4 unpack stores 16*v; fold the 1/16 into the weight scale (exact)
    float* sa_stage = reinterpret_cast<float*>(smem + P::kSa) + e * kWarpTok;
    uint32_t box_pass = 0;
    int buf = 0;
    uint32_t buf_phase = 0;
    int sg_stage = 0;                     // group scales: position in the producer's ring of token-scale stages
    uint32_t sg_phase = 0;
    bool ok = true;
    auto release = [&](int b) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(leader_tmem_empty + 8u * static_cast<uint32_t>(b));
    };
    for (int b = 0; b < kBufs; ++b) release(b);
    for (int item = pair_id; item < num_tiles && ok; item += num_pairs) {
      int mt, nt;
      tile_coords(item, m_tiles, n_tiles, mt, nt);
      const int m0 = mt * kTok + half * kWarpTok;
      const int row0 = nt * kRowsPair + static_cast<int>(rank) * kRowsCta;   // this CTA's first weight row
      const int n = row0 + quad * 32 + lane;
      const bool n_ok = n < N;
      const bool m_full = m0 + kWarpTok <= M;
      const float bias = (args.bias != nullptr && n_ok) ? __bfloat162float(args.bias[n]) : 0.0f;
      if constexpr (OP == OUT_GATED) {
        // the warp's residual box (its 128 tokens x 32 columns) into L2 now, a whole tile of group drains before
        // the store passes read it
        const int c0 = n - lane;
        if (c0 < N)
          for (int r = lane; r < kWarpTok && m0 + r < M; r += 32)
            prefetch_l2(args.res + static_cast<int64_t>(m0 + r) * args.res_ld + c0);
      }
      float sa_pre[kChunks];
#pragma unroll
      for (int c = 0; c < kChunks; ++c)   // group scales carry the tokens' scales per group: the final factor is 1
        sa_pre[c] = (EPI == EPI_GROUP) ? 1.0f : __ldg(args.sa + min(m0 + 32 * c + lane, M - 1));
      auto stage_sa = [&]() {
        __syncwarp();
#pragma unroll
        for (int c = 0; c < kChunks; ++c) sa_stage[32 * c + lane] = sa_pre[c];
        __syncwarp();
      };
      if constexpr (kPerGroup<EPI>) {
        float2 acc[kWarpTok / 2];
        if constexpr (EPI == EPI_GROUP) {
#pragma unroll
          for (int j = 0; j < kWarpTok / 2; ++j) acc[j] = make_float2(0.0f, 0.0f);
        } else {
          // starting value: the zero-point term sum_g z[g, n] * R[g, m], accumulated in fp32 by the tensor core
          if (!(ok = mbar_wait(&tmem_full[buf], buf_phase, abort_flag, 51))) break;
          tc_fence_after();
          const uint32_t taddr = tmem_base + lane_addr + static_cast<uint32_t>(buf * kTok + half * kWarpTok);
#pragma unroll
          for (int ch = 0; ch < kChunks; ++ch) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(taddr + 32 * ch, r);
            tmem_wait_ld_dep(r);
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[16 * ch + j] = make_float2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
          }
          release(buf);
          if (++buf == kBufs) { buf = 0; buf_phase ^= 1u; }
        }
        // the weight scale of the next group is loaded one group ahead as raw bits and converted at use (affine:
        // bf16 [K/128, N]; group scales: f32 [K/128, N])
        auto load_wscale = [&](int gg) -> uint32_t {
          if (!n_ok) return 0u;
          if constexpr (EPI == EPI_GROUP) return __float_as_uint(__ldg(args.sbg + static_cast<int64_t>(gg) * N + n));
          else return __ldg(reinterpret_cast<const unsigned short*>(args.ws) + static_cast<int64_t>(gg) * N + n);
        };
        uint32_t s_bits_next = load_wscale(0);
        for (int g = 0; g < kblocks; ++g) {
          const uint32_t s_bits = s_bits_next;
          if (g + 1 < kblocks) s_bits_next = load_wscale(g + 1);
          if (!(ok = mbar_wait(&tmem_full[buf], buf_phase, abort_flag, 52))) break;
          tc_fence_after();
          const float s = (EPI == EPI_GROUP ? __uint_as_float(s_bits) : bf16_bits_to_f32(s_bits)) * wscale_fold;
          const float2 s2 = make_float2(s, s);
          const uint32_t taddr = tmem_base + lane_addr + static_cast<uint32_t>(buf * kTok + half * kWarpTok);
          // group scales: this group's scales of the warp's 128 tokens, staged by the producer
          const float* sg_tok = sm_sg + sg_stage * kTok + half * kWarpTok;
          if (EPI == EPI_GROUP && !(ok = mbar_wait(&sg_full[sg_stage], sg_phase, abort_flag, 59))) break;
          uint32_t ra[32], rb[32];
          auto scale_chunk = [&](const uint32_t (&r)[32], int ch) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              // |P| < 2^22, so the int32 -> fp32 conversion is exact
              const float2 p = make_float2(__int2float_rn(static_cast<int>(r[2 * j])), __int2float_rn(static_cast<int>(r[2 * j + 1])));
              if constexpr (EPI == EPI_GROUP) {
                // the reference's order: t = P * s_w rounded once, then acc += t * s_a[token] with one rounding; the
                // tokens' group scales are read four at a time (one 16-byte shared load per two steps)
                const float4 a4 = *reinterpret_cast<const float4*>(sg_tok + 32 * ch + 4 * (j >> 1));
                const float2 a = (j & 1) ? make_float2(a4.z, a4.w) : make_float2(a4.x, a4.y);
                const float2 t = fmul2(s2, p);
                acc[16 * ch + j] = ffma2(t, a, acc[16 * ch + j]);
              } else {
                acc[16 * ch + j] = ffma2(s2, p, acc[16 * ch + j]);
              }
            }
          };
          if constexpr (kChunks == 4) {
            // software-pipelined drain: chunk c+1 in flight while chunk c is scaled; the buffer goes back to the
            // leader as soon as the last chunk is in registers (two rounds of two loads measured the same)
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
            release(buf);
            scale_chunk(rb, 3);
          } else {
            // both chunks in flight together; the buffer goes back to the leader one load latency after the group
            // completed, before any of the math
            tmem_ld_32x32b_x32(taddr, ra);
            tmem_ld_32x32b_x32(taddr + 32, rb);
            tmem_wait_ld_dep(ra);
            tmem_wait_ld_dep(rb);
            release(buf);
            scale_chunk(ra, 0);
            scale_chunk(rb, 1);
          }
          if (++buf == kBufs) { buf = 0; buf_phase ^= 1u; }
          if constexpr (EPI == EPI_GROUP) {
            __syncwarp();
            if (lane == 0) mbar_arrive(&sg_empty[sg_stage]);   // this warp is done with the group's token scales
            if (++sg_stage == kSgStages) { sg_stage = 0; sg_phase ^= 1u; }
          }
        }
        if (!ok) break;
        stage_sa();
        if (args.tma_out) {
          // two passes of 64 tokens through a per-warp staging buffer and TMA tensor stores (see the one-SM kernel;
          // with out_w64 two warps share one 64-column box)
          auto store_passes = [&](auto row_bytes_c, auto op_c) -> bool {
            constexpr uint32_t kRow = decltype(row_bytes_c)::value;
            constexpr int kOp = decltype(op_c)::value;
            constexpr bool kPair = kRow == 128;
            const int owner = kPair ? (e & ~1) : e;
            unsigned short* ost = reinterpret_cast<unsigned short*>(smem + P::kOut + owner * P::kOutWarpBytes);
            const uint32_t ost_lane = smem_u32(ost) + (kPair ? 64u * (e & 1) : 0u) + 2u * lane;
            // plain and GELU outputs leave as 32-bit stores of two adjacent columns: lanes 2i and 2i + 1 swap one
            // packed token pair, then the even lane writes both columns of the first token and the odd lane both
            // columns of the second (half the shared-memory store instructions of one 16-bit store per element)
            const uint32_t odd = lane & 1u;
            const uint32_t pair_sel = odd ? 0x3276u : 0x5410u;
            const uint32_t ost_pair = ost_lane - 2u * odd + odd * kRow;
            const bool issuer = !kPair || (e & 1) == 0;
            const int x0 = row0 + (kPair ? (quad & 2) : quad) * 32;
            const int pr = e >> 1;
#pragma unroll
            for (int pass = 0; pass < kWarpTok / 64; ++pass, ++box_pass) {
              const uint32_t par = box_pass & 1u;
              if (issuer) {
                if (lane == 0) {
                  bulk_wait_group_read0();
                  if (kPair) mbar_arrive(&box_free[pr]);
                }
                __syncwarp();
              } else if (!mbar_wait(&box_free[pr], par, abort_flag, 53)) {
                return false;
              }
              // the token scales are read two steps ahead of their use: the stores are ordered asm, so a load
              // written after them would wait for them and expose its whole latency on every step
              const float4* sa4 = reinterpret_cast<const float4*>(sa_stage + 64 * pass);
              float4 c0 = sa4[0], c1 = sa4[1];
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
                const float4 c2 = sa4[j4 + 2 < 16 ? j4 + 2 : 15];
                const int t = 64 * pass + 4 * j4;
                const int r = kOp == OUT_GATED ? 4 * j4 : 0;
                // the linear's fp32 outputs of tokens t..t+3, two per packed fma (the same roundings as scalar fmas)
                const float2 u01 = ffma2(acc[t / 2], make_float2(c0.x, c0.y), make_float2(bias, bias));
                const float2 u23 = ffma2(acc[t / 2 + 1], make_float2(c0.z, c0.w), make_float2(bias, bias));
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
                c0 = c1;
                c1 = c2;
              }
              fence_proxy_async_smem();
              __syncwarp();
              if (kPair && lane == 0) mbar_arrive(&box_full[pr]);
              if (issuer && lane == 0) {
                if (kPair && !mbar_wait(&box_full[pr], par, abort_flag, 54)) return false;
                if (x0 < N && m0 + 64 * pass < M) {
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
              __nv_bfloat16* rows[4] = {orow, orow + N, orow + 2 * static_cast<int64_t>(N), orow + 3 * static_cast<int64_t>(N)};
              const float vs[4] = {v0, v1, v2, v3};
#pragma unroll
              for (int t = 0; t < 4; ++t)
                if (m + t < M) *rows[t] = __float2bfloat16_rn(vs[t]);
            }
            orow += 4 * static_cast<int64_t>(N);
          }
        }
      } else if constexpr (EPI == EPI_INTRATIO) {
        // integer ratios (the reference's policies 5/7/15/17): acc = sum_g P_g * cw[g, n] in int32, exactly as the
        // reference sums it, then bf16(float(acc) * sa[m] * sb[n] + bias) in its order.  The int4 unpack stores
        // 16 * v, so the TMEM sums are 16 P_g: summed as they are while 16 |acc| stays inside int32 (K <= 8192: at
        // most 64 groups of 128, or 128 of 64, of |16 P cw| <= 2^25) and divided by 16 at the end (float(16 acc) / 16
        // = float(acc), a power-of-two scaling), else shifted back to P_g first.
        int acc[kWarpTok];
#pragma unroll
        for (int j = 0; j < kWarpTok; ++j) acc[j] = 0;
        const int ngroups = K / args.cw_group;
        const bool pre_shift = K > 8192;
        auto load_cw = [&](int gg) -> int {
          if (!n_ok) return 0;
          const int64_t i = static_cast<int64_t>(gg) * N + n;
          return args.cw_u8 ? static_cast<int>(__ldg(static_cast<const uint8_t*>(args.cw) + i))
                            : __ldg(static_cast<const int*>(args.cw) + i);
        };
        int cw_next = load_cw(0);
        for (int g = 0; g < ngroups; ++g) {
          const int cwg = cw_next;
          if (g + 1 < ngroups) cw_next = load_cw(g + 1);
          if (!(ok = mbar_wait(&tmem_full[buf], buf_phase, abort_flag, 60))) break;
          tc_fence_after();
          const uint32_t taddr = tmem_base + lane_addr + static_cast<uint32_t>(buf * kTok + half * kWarpTok);
          uint32_t ra[32], rb[32];
          auto add_chunk = [&](const uint32_t (&r)[32], int ch) {
            if (pre_shift) {
#pragma unroll
              for (int j = 0; j < 32; ++j) acc[32 * ch + j] += (static_cast<int>(r[j]) >> 4) * cwg;
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) acc[32 * ch + j] += static_cast<int>(r[j]) * cwg;
            }
          };
          tmem_ld_32x32b_x32(taddr, ra);
          tmem_wait_ld_dep(ra);
          tmem_ld_32x32b_x32(taddr + 32, rb);
          add_chunk(ra, 0);
          tmem_wait_ld_dep(rb);
          tmem_ld_32x32b_x32(taddr + 64, ra);
          add_chunk(rb, 1);
          tmem_wait_ld_dep(ra);
          tmem_ld_32x32b_x32(taddr + 96, rb);
          add_chunk(ra, 2);
          tmem_wait_ld_dep(rb);
          release(buf);
          add_chunk(rb, 3);
          if (++buf == kBufs) { buf = 0; buf_phase ^= 1u; }
        }
        if (!ok) break;
        stage_sa();
        if (n_ok) {
          const float sbn = args.sb[n];
          const float unscale = pre_shift ? 1.0f : 0.0625f;
          __nv_bfloat16* orow = args.out + static_cast<int64_t>(m0) * N + n;
#pragma unroll
          for (int j2 = 0; j2 < kWarpTok / 2; ++j2) {
            const int mm = 2 * j2;
            const float v0 = __fmaf_rn(__fmul_rn(__int2float_rn(acc[mm]) * unscale, sa_stage[mm]), sbn, bias);
            const float v1 = __fmaf_rn(__fmul_rn(__int2float_rn(acc[mm + 1]) * unscale, sa_stage[mm + 1]), sbn, bias);
            if (m_full || m0 + mm + 1 < M) {
              st_bf16_pair_ordered(orow, orow + N, v0, v1);
            } else if (m0 + mm < M) {
              *orow = __float2bfloat16_rn(v0);
            }
            orow += 2 * static_cast<int64_t>(N);
          }
        }
      } else {
        if (!(ok = mbar_wait(&tmem_full[buf], buf_phase, abort_flag, 55))) break;
        tc_fence_after();
        const float sb = n_ok ? args.sb[n] * wscale_fold : 0.0f;
        const uint32_t taddr = tmem_base + lane_addr + static_cast<uint32_t>(buf * kTok + half * kWarpTok);
        stage_sa();
        if constexpr (GLU) {
          // SwiGLU output (see the one-SM kernel): lanes l and l ^ 16 hold the gate and up rows of one output column
          const bool gate = lane < 16;
          const int ncols = N / 2;
          const int j = row0 / 2 + quad * 16 + (lane & 15);
          const int tb = gate ? 0 : 16;
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
              const float other = __shfl_xor_sync(0xffffffffu, gate ? v[16 + k] : v[k], 16);
              const float g = gate ? v[k] : other;
              const float u = gate ? other : v[16 + k];
              const float silu = bf16_round(__fdividef(g, 1.0f + __expf(-g)));
              const int m = m0 + 32 * ch + tb + k;
              if (m < M && j < ncols) args.out[static_cast<int64_t>(m) * ncols + j] = __float2bfloat16_rn(__fmul_rn(silu, u));
            }
          }
        } else if constexpr (OP != OUT_PLAIN) {
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
        release(buf);
        if (++buf == kBufs) { buf = 0; buf_phase ^= 1u; }
      }
    }
  }

  if (kPerGroup<EPI> && warp >= kEpiWarp0 && lane == 0) bulk_wait_group0();
  tc_fence_before();
  if (warp != kTmemWarp) {
    // this warp's role is done (its TMEM reads ordered before by the fence above)
    __syncwarp(__activemask());
    if (lane == 0) mbar_arrive(cta_done);
    return;
  }
  {
    if (lane == 0) {
      // every role warp of this CTA has finished (bounded: an aborted CTA's roles still arrive)
      mbar_wait_drain(cta_done, 0u, kWaitLimitNs);
      // the leader's last commit: every MMA of the pair has completed (bounded: an aborted leader still commits)
      mbar_wait_drain(mma_done, 0u, kDrainNs);
      // tell the other CTA that this one is done with the pair's memory, and wait until it is done too
      mbar_arrive_cluster(mapa_shared(smem_u32(exit_bar), rank ^ 1u));
      mbar_wait_drain(exit_bar, 0u, kDrainNs);
    }
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 512);
  }
}

}  // namespace pr

static int g_pair_clusters = 0;   // CTA pairs that fit on the device at once (cudaOccupancyMaxActiveClusters)

template <int EPI, int BFMT, bool KPERM, bool GLU = false, int OP = OUT_PLAIN>
static int launch_gemm_pair_t(const int8_t* a, const void* b, const void* rsplit, const GemmArgs& args,
                              cudaStream_t st, const OutSpec* outs = nullptr) {
  auto kern = pr::gemm_pair_kernel<EPI, BFMT, KPERM, GLU, OP>;
  constexpr int smem_bytes = pr::Plan<EPI>::kBytes;
  static bool configured = false;
  static bool regs_ok = false;
  static int clusters = 0;
  if (!configured) {
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess) return CQ_ERR_CUDA;
    regs_ok = fa.numRegs * pr::kThreads >= 256 * kProducerRegs + 256 * kEpilogueRegs;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes) != cudaSuccess)
      return CQ_ERR_CUDA;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(pr::kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem_bytes;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess || clusters <= 0) return CQ_ERR_CUDA;
    configured = true;
  }
  if (!regs_ok) return CQ_ERR_CUDA;
  g_pair_clusters = clusters;
  CUtensorMap tm_x, tm_w, tm_r, tm_z;
  OutMaps tm_out;
  if (!make_map_u8(&tm_x, a, args.M, args.K, pr::kBK, pr::kTokCta, true)) return CQ_ERR_CUDA;
  if (EPI == EPI_AFFINE) {
    if (!make_map_u8(&tm_r, rsplit, args.M, 2 * rsplit_cols(args.K), 128, pr::kTokCta, true)) return CQ_ERR_CUDA;
    if (!make_map_u8(&tm_z, args.zt, args.N, 128 * static_cast<int64_t>(args.nz), 128, pr::kRowsCta, true))
      return CQ_ERR_CUDA;
  } else if (EPI == EPI_GROUP) {
    // the tokens' per-group scales [K/128, sag_ld] f32: one box = one group's scales of a tile's 256 tokens
    if (!make_map_f32(&tm_r, rsplit, args.K / 128, args.sag_ld, pr::kTok, 1)) return CQ_ERR_CUDA;
    tm_z = tm_x;
  } else {
    tm_r = tm_x;
    tm_z = tm_x;
  }
  if (!make_map_u8(&tm_w, b, args.N, args.K / 2, pr::kBK / 2, pr::kRowsCta, false)) return CQ_ERR_CUDA;
  GemmArgs ga = args;
  ga.tma_out = 0;
  ga.n_out = 0;
  ga.out_col0 = 0;
  ga.split = 0;
  std::memset(&tm_out, 0, sizeof(tm_out));
  ga.out_w64 = (outs != nullptr && args.N % 64 == 0) ? 1 : 0;
  const int box_cols = ga.out_w64 ? 64 : 32;
  if (pr::kPerGroup<EPI> && outs != nullptr) {
    for (int i = 0; i < outs->n; ++i)
      if (!make_map_bf16(&tm_out.m[i], outs->ptrs[i], args.M, outs->ldo, box_cols, 64)) return CQ_ERR_CUDA;
    ga.tma_out = 1;
    ga.n_out = outs->n;
    ga.out_col0 = outs->col0;
  } else if (pr::kPerGroup<EPI> && args.N % 8 == 0 && (reinterpret_cast<uintptr_t>(args.out) & 15u) == 0) {
    if (!make_map_bf16(&tm_out.m[0], args.out, args.M, args.N, box_cols, 64)) return CQ_ERR_CUDA;
    ga.tma_out = 1;
    ga.n_out = 1;
  }
  const int tiles = ((args.M + pr::kTok - 1) / pr::kTok) * ((args.N + pr::kRowsPair - 1) / pr::kRowsPair);
  const int pairs = tiles < clusters ? tiles : clusters;
  if (pairs == 0) return CQ_OK;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(pr::kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem_bytes;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = ga.pdl ? 2 : 1;
  if (cudaLaunchKernelEx(&cfg, kern, tm_x, tm_w, tm_r, tm_z, tm_out, ga) != cudaSuccess) return CQ_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? CQ_OK : CQ_ERR_CUDA;
}

// ---------------------------------------------------------------------------------------------
// public launchers: one-SM or CTA-pair kernel by shape
// ---------------------------------------------------------------------------------------------

// Kernel choice for the packed-int4-weight GEMMs: CQ_GEMM_AUTO picks by shape, the other values force one form.
static int g_gemm_variant = CQ_GEMM_AUTO;

int set_gemm_variant(int variant) {
  if (variant != CQ_GEMM_AUTO && variant != CQ_GEMM_ONE_SM && variant != CQ_GEMM_PAIR) return CQ_ERR_ARG;
  g_gemm_variant = variant;
  return CQ_OK;
}

// The pair kernel's tile is 256 weight rows x 256 tokens: it pays off once there are enough tiles to fill the CTA pairs
// (small problems keep the finer one-SM tiles, which also split a partial last wave into half tiles).
static bool use_pair_kernel(int M, int N);

// K splits for an affine GEMM on the one-SM kernel with too few tiles to fill the SMs (a DiT's text stream: one
// 256-token tile): the largest S in {8, 6, 4, 3, 2} that divides the K blocks, leaves each split at least two of them
// and keeps tiles x S within the SMs; 1 when the tiles already fill half the SMs
int affine_ksplit(int M, int N, int K) {
  const int tiles = ((M + 255) / 256) * ((N + 127) / 128);
  const int kb = K / 128;
  const int sms = num_sms();
  if (sms <= 0 || 2 * tiles >= sms || N % 8 != 0 || use_pair_kernel(M, N)) return 1;
  for (int s : {8, 6, 4, 3, 2})
    if (kb % s == 0 && kb / s >= 2 && tiles * s <= sms) return s;
  return 1;
}

static bool use_pair_kernel(int M, int N) {
  if (g_gemm_variant == CQ_GEMM_ONE_SM) return false;
  if (g_gemm_variant == CQ_GEMM_PAIR) return true;
  const int64_t pair_tiles = static_cast<int64_t>((M + 255) / 256) * ((N + 255) / 256);
  return M >= 1024 && pair_tiles >= 74;
}

int launch_gemm_rowcol(const int8_t* a, int a_kperm, const float* sa, const void* b, int b_format, const float* sb,
                       const void* bias, void* out, int M, int N, int K, cudaStream_t st, bool pdl, const OutOp* op) {
  GemmArgs g{};
  g.pdl = pdl;
  g.sa = sa;
  g.sb = sb;
  g.bias = static_cast<const __nv_bfloat16*>(bias);
  g.out = static_cast<__nv_bfloat16*>(out);
  g.M = M; g.N = N; g.K = K;
  if (op != nullptr && op->kind != OUT_PLAIN) {
    g.out_op = op->kind;
    g.res = static_cast<const __nv_bfloat16*>(op->res);
    g.res_ld = op->res_ld;
    g.gate = static_cast<const __nv_bfloat16*>(op->gate);
  }
  auto launch = [&](auto op_c) {
    constexpr int kOp = decltype(op_c)::value;
    if (b_format == CQ_B_INT8) return launch_gemm_t<EPI_ROWCOL, BF_S8, false, false, kOp>(a, b, nullptr, g, st);
    if (use_pair_kernel(M, N)) {
      if (a_kperm) return launch_gemm_pair_t<EPI_ROWCOL, BF_S4, true, false, kOp>(a, b, nullptr, g, st);
      return launch_gemm_pair_t<EPI_ROWCOL, BF_S4, false, false, kOp>(a, b, nullptr, g, st);
    }
    if (a_kperm) return launch_gemm_t<EPI_ROWCOL, BF_S4, true, false, kOp>(a, b, nullptr, g, st);
    return launch_gemm_t<EPI_ROWCOL, BF_S4, false, false, kOp>(a, b, nullptr, g, st);
  };
  if (g.out_op == OUT_GELU) return launch(std::integral_constant<int, OUT_GELU>{});
  if (g.out_op == OUT_GATED) return launch(std::integral_constant<int, OUT_GATED>{});
  return launch(std::integral_constant<int, OUT_PLAIN>{});
}

// W4A4 row/col GEMM with the SwiGLU output: b holds the weight rows interleaved in groups of 32 (16 gate rows, then
// their 16 up rows); out is bf16 [M, N / 2].
int launch_gemm_rowcol_glu(const int8_t* a, const float* sa, const void* b, const float* sb, const void* bias,
                           void* out, int M, int N, int K, cudaStream_t st, bool pdl) {
  GemmArgs g{};
  g.pdl = pdl;
  g.sa = sa;
  g.sb = sb;
  g.bias = static_cast<const __nv_bfloat16*>(bias);
  g.out = static_cast<__nv_bfloat16*>(out);
  g.M = M; g.N = N; g.K = K;
  if (use_pair_kernel(M, N)) return launch_gemm_pair_t<EPI_ROWCOL, BF_S4, true, true>(a, b, nullptr, g, st);
  return launch_gemm_t<EPI_ROWCOL, BF_S4, true, true>(a, b, nullptr, g, st);
}

int launch_gemm_affine(const int8_t* a, int a_kperm, const float* sa, const void* rsplit, const void* b,
                       const void* s, const void* zt, const void* bias, void* out, int M, int N, int K,
                       cudaStream_t st, void* const* outs, int n_outs, int col0, int64_t ldo, const OutOp* op,
                       bool pdl, float* partial) {
  const bool plain = op == nullptr || op->kind == OUT_PLAIN;
  // a few tokens (adaLN modulation): read the weights once with a warp per row instead of 256-token MMA tiles
  // (plain outputs only: the output operations live in the GEMM's epilogue)
  if (outs == nullptr && plain && gemv_affine_fits(M, a_kperm))
    return launch_gemv_affine(a, sa, b, s, zt, bias, out, M, N, K, st, pdl) == cudaSuccess ? CQ_OK : CQ_ERR_CUDA;
  GemmArgs g{};
  g.pdl = pdl;
  if (!plain) {
    g.out_op = op->kind;
    g.res = static_cast<const __nv_bfloat16*>(op->res);
    g.res_ld = op->res_ld;
    g.gate = static_cast<const __nv_bfloat16*>(op->gate);
  }
  g.sa = sa;
  g.nz = rsplit_cols(K) / 64;
  g.ws = static_cast<const __nv_bfloat16*>(s);
  g.zt = static_cast<const __nv_bfloat16*>(zt);
  g.bias = static_cast<const __nv_bfloat16*>(bias);
  g.out = static_cast<__nv_bfloat16*>(out);
  g.M = M; g.N = N; g.K = K;
  // split K over more CTAs when the tiles leave most SMs idle, if the caller gave room for the partial sums
  const bool res_pairs = plain || op->kind != OUT_GATED ||
                         ((reinterpret_cast<uintptr_t>(op->res) & 3u) == 0 && op->res_ld % 2 == 0 &&
                          (reinterpret_cast<uintptr_t>(op->gate) & 3u) == 0);   // the finalize reads pairs
  if (partial != nullptr && outs == nullptr && (reinterpret_cast<uintptr_t>(out) & 15u) == 0 && res_pairs) {
    g.ksplit = affine_ksplit(M, N, K);
    g.partial = partial;
  }
  const OutSpec spec{outs, n_outs, col0, ldo};
  const OutSpec* sp = outs != nullptr ? &spec : nullptr;
  auto launch = [&](auto op_c) {
    constexpr int kOp = decltype(op_c)::value;
    if (use_pair_kernel(M, N)) {
      if (a_kperm) return launch_gemm_pair_t<EPI_AFFINE, BF_U4, true, false, kOp>(a, b, rsplit, g, st, sp);
      return launch_gemm_pair_t<EPI_AFFINE, BF_U4, false, false, kOp>(a, b, rsplit, g, st, sp);
    }
    if (a_kperm) return launch_gemm_t<EPI_AFFINE, BF_U4, true, false, kOp>(a, b, rsplit, g, st, sp);
    return launch_gemm_t<EPI_AFFINE, BF_U4, false, false, kOp>(a, b, rsplit, g, st, sp);
  };
  if (g.out_op == OUT_GELU) return launch(std::integral_constant<int, OUT_GELU>{});
  if (g.out_op == OUT_GATED) return launch(std::integral_constant<int, OUT_GATED>{});
  return launch(std::integral_constant<int, OUT_PLAIN>{});
}

// Integer weight ratios per group (the reference's policies 5/7/15/17): int4 activation codes (int8-held) x packed
// signed int4 weights, acc = sum_g P_g * cw[g, n] in int32 over groups of cw_group (64 or 128) K columns, then
// bf16(float(acc) * sa[m] * sb[n] + bias).  cw is int32 or (cw_u8) uint8 [K/cw_group, N].
int launch_gemm_intratio(const int8_t* a, int a_kperm, const float* sa, const void* b, const float* sb, const void* cw,
                         int cw_u8, int cw_group, const void* bias, void* out, int M, int N, int K, cudaStream_t st) {
  GemmArgs g{};
  g.sa = sa;
  g.sb = sb;
  g.cw = cw;
  g.cw_u8 = cw_u8;
  g.cw_group = cw_group;
  g.bias = static_cast<const __nv_bfloat16*>(bias);
  g.out = static_cast<__nv_bfloat16*>(out);
  g.M = M; g.N = N; g.K = K;
  if (a_kperm) return launch_gemm_pair_t<EPI_INTRATIO, BF_S4, true>(a, b, nullptr, g, st);
  return launch_gemm_pair_t<EPI_INTRATIO, BF_S4, false>(a, b, nullptr, g, st);
}

// Per-group scales on both sides (the reference's policy 4): int4 activation codes (int8-held) x packed signed int4
// weights, acc += round(P_g * sbg[g, n]) * sag[g, m] in fp32 over the 128-wide groups g, then + bias -> bf16.
int launch_gemm_group(const int8_t* a, int a_kperm, const float* sag, int64_t sag_ld, const void* b, const float* sbg,
                      const void* bias, void* out, int M, int N, int K, cudaStream_t st) {
  GemmArgs g{};
  g.sbg = sbg;
  g.sag_ld = sag_ld;
  g.bias = static_cast<const __nv_bfloat16*>(bias);
  g.out = static_cast<__nv_bfloat16*>(out);
  g.M = M; g.N = N; g.K = K;
  if (a_kperm) return launch_gemm_pair_t<EPI_GROUP, BF_S4, true>(a, b, sag, g, st);
  return launch_gemm_pair_t<EPI_GROUP, BF_S4, false>(a, b, sag, g, st);
}

}  // namespace cq
