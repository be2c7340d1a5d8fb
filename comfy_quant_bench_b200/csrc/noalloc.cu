// W4A8 affine linear that allocates nothing: its scratch lives in a fixed device array of this library.
//
// Some callers cannot allocate device memory at the point where they run the linear: code that runs while a
// memory pool is frozen or being defragmented, allocator hooks and custom memory managers that must not
// re-enter the allocator, and host integrations (plugins loaded by another runtime) that are handed only
// input and output buffers.  cq_linear_w4a8_affine_noalloc serves them: it runs the same two kernels as
// cq_linear_w4a8_affine (activation rotation + int8 quantization, then the tcgen05 GEMM) but keeps their
// scratch - the int8 activation codes, the per-token scales and the split group sums - in the file-scope
// array below instead of a caller-provided workspace.
//
// Properties of the shared scratch array:
//   * it is kNoallocScratchBytes (32 MiB) per device and every GPU that loads this library holds it until the
//     process exits;
//   * every call uses the same array and leaves the last call's data in it; nothing in it needs to start at
//     zero (the activation kernel writes every byte the GEMM reads), and calls that overlap on the GPU (two
//     streams, or two host threads) race on it - serialize them on one stream;
//   * its device address is looked up with cudaGetSymbolAddress on the first call made with a device current,
//     and again whenever that device's current context has changed since (after cudaDeviceReset the module is
//     loaded anew, possibly at another address); make the first call on a device, and the first one after a
//     reset, before any stream capture begins.
#include <mutex>

#include "kernels.cuh"

namespace cq {

constexpr int64_t kNoallocScratchBytes = 32ll << 20;
constexpr int kNoallocMaxDevices = 64;

// The scratch itself.  In host code this name is only a stand-in for the symbol; the device address comes
// from cudaGetSymbolAddress (noalloc_scratch_ptr below).
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoallocScratchBytes];

static std::mutex g_noalloc_mutex;
static void* g_noalloc_ptr[kNoallocMaxDevices] = {};
static CUcontext g_noalloc_ctx[kNoallocMaxDevices] = {};

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

// The driver's current context of the calling thread (the runtime makes the device's primary context current).
static int current_context(CUcontext* ctx) {
  static CtxGetCurrentFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || p == nullptr)
      return CQ_ERR_CUDA;
    fn = reinterpret_cast<CtxGetCurrentFn>(p);
  }
  *ctx = nullptr;
  return fn(ctx) == CUDA_SUCCESS ? CQ_OK : CQ_ERR_CUDA;   // null when no context is current on this thread yet
}

// Device address of the scratch array on the current device, cached per device together with the context it was
// looked up in: a different current context (the primary context was reset and re-created) looks it up again.
static int noalloc_scratch_ptr(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoallocMaxDevices) return CQ_ERR_CUDA;
  CUcontext ctx = nullptr;
  if (int e = current_context(&ctx)) return e;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_ptr[dev] == nullptr || ctx == nullptr || g_noalloc_ctx[dev] != ctx) {
    // the lookup also makes the device's primary context current on this thread when none was
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return CQ_ERR_CUDA;
    if (int e = current_context(&ctx)) return e;
    if (ctx == nullptr) return CQ_ERR_CUDA;
    g_noalloc_ptr[dev] = p;
    g_noalloc_ctx[dev] = ctx;
  }
  *out = g_noalloc_ptr[dev];
  return CQ_OK;
}

}  // namespace cq

extern "C" {

int cq_linear_w4a8_affine_noalloc(const void* x, int64_t M, int64_t K, int64_t N, int rot_group, int swiglu,
                                  const void* qweight, const void* s_bf16, const void* zt_bf16, int group,
                                  const void* bias, void* out, void* stream) {
  if (M == 0) return CQ_OK;
  const int64_t need = cq_linear_workspace_bytes(M, K);
  if (need < 0) return CQ_ERR_SHAPE;
  if (need > cq::kNoallocScratchBytes) return CQ_ERR_CAPACITY;   // problem larger than the fixed scratch array
  void* scratch = nullptr;
  if (int e = cq::noalloc_scratch_ptr(&scratch)) return e;
  // exactly the base workspace: the GEMM runs unsplit, as cq_linear_w4a8_affine does with that workspace
  return cq_linear_w4a8_affine(x, M, K, N, rot_group, swiglu, qweight, s_bf16, zt_bf16, group, bias, out, scratch, need,
                               stream);
}

}  // extern "C"
