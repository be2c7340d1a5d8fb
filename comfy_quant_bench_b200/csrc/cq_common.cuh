// Shared device helpers for the sm_100a kernels: status codes, bounded mbarrier waits, TMA, tcgen05.
//
// Every wait in these kernels is bounded by wall time (%globaltimer): a wait that runs out records
// CQ_ERR_TIMEOUT in the device status word, raises the CTA's abort flag and returns false, so the kernel
// unwinds, frees its TMEM and exits instead of spinning forever.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/cq_b200.h"

namespace cq {

// Device status word: the first nonzero status a kernel records since the last cq_take_device_status().
// (index 0: status code, index 1: where it was raised).  The library is built as one translation unit
// (libcq.cu), so this single definition is the one every kernel and cq_take_device_status() see.
__device__ int g_device_status[2] = {0, 0};

constexpr unsigned long long kWaitLimitNs = 2000000000ull;   // 2 s per wait

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void record_status(int code, int where) {
  if (atomicCAS(&g_device_status[0], 0, code) == 0) g_device_status[1] = where;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Programmatic dependent launch.  grid_dep_launch: this CTA no longer holds back the launch of the next kernel in
// the stream (when that kernel was launched with programmatic stream serialization, it may start once every CTA of
// this grid has called this or exited).  grid_dep_wait: block until the previous kernel in the stream has completed
// and its memory operations are visible (returns at once for a kernel launched without the attribute).
// a cache-line prefetch into L2 (no register result, nothing waits on it)
__device__ __forceinline__ void prefetch_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar)) : "memory");
}

// `count` arrivals at once (a thread arriving on behalf of others that have nothing to signal)
__device__ __forceinline__ void mbar_arrive_cnt(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}"
               ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// Test for the completion of the phase with parity `parity`; a waiting thread is suspended in hardware (up to
// about 0.5 ms per call) instead of spinning, so waiting warps leave the issue slots to the working ones.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity), "r"(500000u) : "memory");
  return ok != 0;
}

// Non-blocking probe of the phase with parity `parity` (a few cycles when the phase is already complete, where the
// suspending form above costs several times more).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}

// Wait for the phase with parity `parity` to complete; false on timeout or when the CTA aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int where) {
  if (mbar_test_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++spins & 3u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        record_status(CQ_ERR_TIMEOUT, where);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

// Test / wait for `parity` with acquire semantics at cluster scope (the unwinding waits below).
__device__ __forceinline__ bool mbar_test_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity), "r"(500000u) : "memory");
  return ok != 0;
}
// Both phases complete?  Two non-blocking probes issued together (one round trip instead of two in a row).
__device__ __forceinline__ bool mbar_test_wait2(uint64_t* a, uint32_t pa, uint64_t* b, uint32_t pb) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 q, [%3], %4;\n\t"
      "and.pred p, p, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_u32(a)), "r"(pa), "r"(smem_u32(b)), "r"(pb) : "memory");
  return ok != 0;
}

// Wait for `parity` for at most `limit_ns`, whatever the abort flag says: used while unwinding after an abort, to
// let copies and tensor-core operations that were already issued finish before their memory goes away.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity, unsigned long long limit_ns) {
  if (mbar_test_wait_cluster(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
}

// Every stage of a ring of n stages that `issued` loads reached: wait (bounded, limit_ns each) for the phase of the
// last load issued into it.  Used before a CTA releases its shared memory, so that no copy still in flight can
// land in it (on a normal end every load was consumed long before, and each wait returns at once).
__device__ __forceinline__ void drain_ring(uint64_t* full, int n, uint32_t issued, unsigned long long limit_ns) {
  for (int s = 0; s < n; ++s) {
    if (issued <= static_cast<uint32_t>(s)) break;
    const uint32_t last = issued - 1 - ((issued - 1 - s) % n);   // index of the last load into stage s
    mbar_wait_drain(&full[s], (last / n) & 1u, limit_ns);
  }
}

// ---------------------------------------------------------------------------------------------
// thread-block clusters (CTA pairs of the 2-SM GEMM).  Remote mbarrier arrivals only; no multicast loads.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cta address -> the shared::cluster address of the same offset in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa_shared(uint32_t cta_addr, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(cta_addr), "r"(rank));
  return d;
}
// one arrival on the mbarrier at shared::cluster address `cluster_addr` (default semantics: release at CTA scope).
// The CTA-pair GEMM orders its cross-CTA hand-offs with these: TMEM reads are ordered by tcgen05 fences before the
// arrival, shared-memory operands by the producer's own barrier (TMA) or proxy fence before it.  A cluster-scope
// release would also wait for all of the thread's outstanding memory traffic, which measured ~1000 cycles per
// arrival under load.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// ---------------------------------------------------------------------------------------------
// TMA (tiled 2-D loads into shared memory, completion on an mbarrier). No multicast anywhere.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// TMA tensor store (2-D) from shared memory into global memory, tracked by this thread's bulk-async groups.
// Coordinates are element indices into the tensor map (never negative here); out-of-range parts are clipped.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
               ::"l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(smem_src)), "r"(x), "r"(y) : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// wait until every committed bulk store of this thread has finished reading its shared-memory source
__device__ __forceinline__ void bulk_wait_group_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// wait until every committed bulk store of this thread has completed
__device__ __forceinline__ void bulk_wait_group0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Generic-proxy shared-memory writes -> visible to the async proxy (tensor core / TMA).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------------------------
// tcgen05
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
               ::"r"(smem_u32(dst_smem)), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// All prior tcgen05.mma of this thread -> one arrive on `bar` when they complete.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(smem_u32(bar)) : "memory");
}
// D(tmem) (+)= A(smem desc) * B(smem desc), int8 x int8 -> int32.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}
// D(tmem) (+)= A(smem desc) * B(smem desc), bf16 x bf16 -> fp32.
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}
// 2-SM forms (a CTA pair of a cluster; every tcgen05 instruction of a kernel that uses them names cta_group::2).
// Allocation, permit release and deallocation are collective: one warp of EACH CTA of the pair executes them.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
               ::"r"(smem_u32(dst_smem)), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// All prior tcgen05.mma of this thread -> one arrive on the mbarrier at `bar`'s offset in BOTH CTAs of the pair.
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
               ::"r"(smem_u32(bar)), "h"(static_cast<uint16_t>(3)) : "memory");
}
// D(tmem, 128 lanes in each CTA) (+)= A (128 rows in each CTA's shared memory) * B (N/2 rows in each CTA's shared
// memory), int8 x int8 -> int32; issued by one thread of the even CTA.
__device__ __forceinline__ void mma_i8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}
__device__ __forceinline__ void mma_bf16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// tcgen05.wait::ld that also names the 32 destination registers of the load it waits for, so the compiler
// cannot schedule a read of them ahead of the wait (tcgen05.ld writes its registers asynchronously).
__device__ __forceinline__ void tmem_wait_ld_dep(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp gets row (lane_base + i), columns c..c+31.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// Shared-memory matrix descriptor for a K-major operand in the 128-byte swizzle layout: rows of 128 bytes,
// 8-row groups 1024 bytes apart (SBO), version 1 (sm_100), base offset 0 (tiles are 1024-byte aligned).
__device__ __forceinline__ uint64_t smem_desc_k_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);          // start address   [0,14)
  d |= static_cast<uint64_t>(1u) << 16;                          // LBO (unused for swizzled K-major) [16,30)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;                  // SBO = 1024 B     [32,46)
  d |= static_cast<uint64_t>(1u) << 46;                          // descriptor version 1 [46,48)
  d |= static_cast<uint64_t>(2u) << 61;                          // SWIZZLE_128B     [61,64)
  return d;
}

// Instruction descriptor, kind::i8: D s32, A/B signed int8, both K-major, shape M x N.
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n) {
  return (2u << 4)                                  // D format: s32
         | (1u << 7)                                // A: signed 8-bit
         | (1u << 10)                               // B: signed 8-bit
         | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}

// Instruction descriptor, kind::f16: D f32, A/B bf16, both K-major, shape M x N.
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n) {
  return (1u << 4)                                  // D format: f32
         | (1u << 7)                                // A: bf16
         | (1u << 10)                               // B: bf16
         | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}

// ---------------------------------------------------------------------------------------------
// misc
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// Ordered global accesses (asm volatile keeps them in program order, so the compiler cannot hoist a long run
// of loads ahead of the stores that consume them and blow up register pressure).
__device__ __forceinline__ float4 ld_nc_f4_ordered(const float* p) {
  float4 v;
  asm volatile("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ float ld_nc_f32_ordered(const float* p) {
  float v;
  asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}
// v0 -> *p0 and v1 -> *p1 as bf16 (round to nearest even): one paired conversion (cvt.rn.bf16x2.f32 runs at four
// times the rate of the single-value form) and two 16-bit stores.
__device__ __forceinline__ void st_bf16_pair_ordered(__nv_bfloat16* p0, __nv_bfloat16* p1, float v0, float v1) {
  asm volatile(
      "{\n\t.reg .b32 d;\n\t.reg .b16 lo, hi;\n\t"
      "cvt.rn.bf16x2.f32 d, %3, %2;\n\t"
      "mov.b32 {lo, hi}, d;\n\t"
      "st.global.b16 [%0], lo;\n\t"
      "st.global.b16 [%1], hi;\n\t}"
      ::"l"(p0), "l"(p1), "f"(v0), "f"(v1) : "memory");
}

// bf16 bits of lo (low half) and hi (high half), each rounded to nearest even
__device__ __forceinline__ uint32_t bf16x2_bits(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

__device__ __forceinline__ void sts_b32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.b32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

// The gated residual of two tokens of one output column, in packed bf16: o_i = bf16(r_i + g * bf16(v_i)) with one
// rounding of the exact value (fma.rn.bf16x2); r0, r1 are the residuals' bf16 bits, gate2 the gate's bits in both
// halves.  Against torch's addcmul on bf16 tensors (an fp32 result rounded to bf16) it can differ only where the fp32
// rounding lands on a bf16 rounding tie, about one output in 2^16.  -> shared addresses a0, a1.
__device__ __forceinline__ void sts_gated_pair(uint32_t a0, uint32_t a1, float v0, float v1, uint32_t gate2, uint32_t r0,
                                               uint32_t r1) {
  asm volatile(
      "{\n\t.reg .b32 y, r, o;\n\t.reg .b16 lo, hi;\n\t"
      "cvt.rn.bf16x2.f32 y, %3, %2;\n\t"
      "prmt.b32 r, %5, %6, 0x5410;\n\t"
      "fma.rn.bf16x2 o, %4, y, r;\n\t"
      "mov.b32 {lo, hi}, o;\n\t"
      "st.shared.b16 [%0], lo;\n\t"
      "st.shared.b16 [%1], hi;\n\t}"
      ::"r"(a0), "r"(a1), "f"(v0), "f"(v1), "r"(gate2), "r"(r0), "r"(r1) : "memory");
}

// v0 (low half) and v1 (high half) as a bf16 pair (round to nearest even)
__device__ __forceinline__ uint32_t bf16_pair_bits(float v0, float v1) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(v1), "f"(v0));
  return d;
}

// sts_gated_pair's value in a register: bf16(r_i + g * bf16(v_i)) for i = 0 (low half), 1 (high half)
__device__ __forceinline__ uint32_t gated_pair_bits(float v0, float v1, uint32_t gate2, uint32_t r0, uint32_t r1) {
  uint32_t o;
  asm("{\n\t.reg .b32 y, r;\n\t"
      "cvt.rn.bf16x2.f32 y, %2, %1;\n\t"
      "prmt.b32 r, %4, %5, 0x5410;\n\t"
      "fma.rn.bf16x2 %0, %3, y, r;\n\t}"
      : "=r"(o) : "f"(v0), "f"(v1), "r"(gate2), "r"(r0), "r"(r1));
  return o;
}

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t bits16) { return __uint_as_float(bits16 << 16); }

// Smallest bf16 value >= v for v > 0 (mantissa rounded up), as the reference's per-group quantizer does.
__device__ __forceinline__ float bf16_up(float v) {
  uint32_t u = __float_as_uint(v);
  const uint32_t low = u & 0xFFFFu;
  u &= 0xFFFF0000u;
  if (low) u += 0x10000u;
  return __uint_as_float(u);
}

__device__ __forceinline__ float bf16_round(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

}  // namespace cq
