// moe_noalloc.cu -- MoE token dispatch without any allocation.
//
// remora_b200_moe_dispatch needs a device workspace for its per-block
// expert counts, which the caller has to allocate.  Some callers cannot
// allocate device memory at the point where they dispatch: code that runs
// inside a memory pool or arena it does not own, embedders that forbid
// cudaMalloc after start-up so that memory use stays fixed, and runtimes
// that must not take the allocator's global lock on a latency-critical path.
// This variant keeps that scratch in a fixed array inside the library
// instead, so a call allocates nothing: no cudaMalloc, no cudaFree, no
// allocating library routine.
//
// Properties of the scratch array:
//   - Its size is fixed (kNoAllocScratchInts int32 slots, 1 MiB); a call
//     whose dispatch needs more (ceil(T*k / 1024) * E slots) is rejected
//     with REMORA_B200_ERR_INVALID before anything is launched.
//   - Every GPU that loads the library holds one copy until the process
//     exits.
//   - All calls on a device share it and it keeps the last call's contents.
//     Nothing in it needs to start at zero: the count kernel writes every
//     slot a dispatch reads before it is read.  Calls that overlap on the
//     GPU (on different streams, or from different host threads) race on
//     it; serialise them, e.g. by issuing them on one stream.
//   - In host code the array's name is only a host-side stand-in, so its
//     device address is looked up once per device with
//     cudaGetSymbolAddress, with that device current.  The first call on a
//     device performs this set-up; make that first call before any CUDA
//     stream capture that might include it.  The address belongs to the
//     device's CUDA context: it is cached together with the context's
//     unique id (cuCtxGetId), so after a cudaDeviceReset the next call sees
//     a new context and looks the address up again (that call is then a
//     first call again, with the same rule about stream capture).
#include <mutex>

#include "runtime.cuh"

namespace rb {
namespace moe {

constexpr int64_t kNoAllocScratchInts = 1 << 18;  // 1 MiB of int32 slots

static __device__ __align__(256) int32_t g_noalloc_dispatch_scratch[kNoAllocScratchInts];

constexpr int kMaxDevices = 64;
struct NoAllocSlot {
  int32_t* ptr;
  unsigned long long ctx_id;  // unique id of the context the address belongs to
};
static NoAllocSlot g_noalloc[kMaxDevices] = {};
static std::mutex g_noalloc_mu;


// Device address of the scratch array on the current device, looked up once
// per device and context.  If the context id cannot be read, the address is
// looked up on every call (cudaGetSymbolAddress allocates nothing).
static int noalloc_scratch(int32_t** out) {
  int dev = 0;
  RB_CUDA(cudaGetDevice(&dev));
  RB_CHECK_ARG(dev >= 0 && dev < kMaxDevices, "dispatch_noalloc: device %d out of range", dev);
  const unsigned long long ctx = current_ctx_id();
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  NoAllocSlot& slot = g_noalloc[dev];
  if (!slot.ptr || ctx == 0 || slot.ctx_id != ctx) {
    int32_t* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_noalloc_dispatch_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(REMORA_B200_ERR_CUDA, "dispatch_noalloc: cudaGetSymbolAddress failed: %s",
                  cudaGetErrorString(e));
    slot.ptr = p;
    // the lookup made the device's context current if no runtime call had
    // yet on this thread: read its id now
    slot.ctx_id = ctx ? ctx : current_ctx_id();
  }
  *out = slot.ptr;
  return REMORA_B200_OK;
}

}  // namespace moe
}  // namespace rb

extern "C" int remora_b200_moe_dispatch_noalloc(const int32_t* idx, int64_t T, int k, int E,
                                                int32_t* counts, int32_t* offsets, int32_t* perm,
                                                int32_t* inv, void* stream) {
  using namespace rb;
  using namespace rb::moe;
  clear_error();
  RB_CHECK_ARG(T >= 0 && k >= 1 && E >= 1 && E <= GMaxE, "dispatch_noalloc: bad sizes");
  RB_CHECK_ARG(T <= INT32_MAX / k,
               "dispatch_noalloc: T*k = %lld*%d exceeds the int32 range of perm and inv",
               (long long)T, k);
  RB_CHECK_ARG(T * k == 0 || (idx && counts && offsets && perm && inv),
               "dispatch_noalloc: null pointer");
  const int64_t need = dispatch_blocks(T * k) * (int64_t)E;
  RB_CHECK_ARG(need <= kNoAllocScratchInts,
               "dispatch_noalloc: needs %lld scratch slots (ceil(T*k/1024)*E), the fixed "
               "array holds %lld; use remora_b200_moe_dispatch with a workspace",
               (long long)need, (long long)kNoAllocScratchInts);
  int32_t* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  return dispatch_launch(idx, T, k, E, counts, offsets, perm, inv, scratch, as_stream(stream));
}
