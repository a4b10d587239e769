// runtime.cuh -- host-side plumbing shared by every launcher: the status
// codes and thread-local last-error text of the C ABI, CUDA error mapping,
// the device error word, and TMA tensor-map encoding through the driver
// entry point (no link-time dependency on libcuda).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdlib>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/remora_b200.h"
#include "ptx.cuh"

namespace rb {

static thread_local char t_last_error[512] = "";

inline int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return code;
}

inline void clear_error() { t_last_error[0] = '\0'; }

#define RB_CUDA(call)                                                                   \
  do {                                                                                  \
    cudaError_t _e = (call);                                                            \
    if (_e != cudaSuccess)                                                              \
      return ::rb::fail(REMORA_B200_ERR_CUDA, "%s: %s (%s:%d)", #call,                  \
                        cudaGetErrorString(_e), __FILE__, __LINE__);                    \
  } while (0)

#define RB_CHECK_ARG(cond, ...)                                                         \
  do {                                                                                  \
    if (!(cond)) return ::rb::fail(REMORA_B200_ERR_INVALID, __VA_ARGS__);               \
  } while (0)

#define RB_LAUNCH_CHECK()                                                               \
  do {                                                                                  \
    cudaError_t _e = cudaGetLastError();                                                \
    if (_e != cudaSuccess)                                                              \
      return ::rb::fail(REMORA_B200_ERR_CUDA, "launch failed: %s (%s:%d)",              \
                        cudaGetErrorString(_e), __FILE__, __LINE__);                    \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------- tensor maps
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Encodes a tiled tensor map.  dims / box are innermost-first; strides are
// the byte strides of dims 1..rank-1.
inline int make_tmap(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int rank,
                     const uint64_t* dims, const uint64_t* strides, const uint32_t* box,
                     CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(REMORA_B200_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) s[i] = strides[i];
  CUresult r = fn(m, dt, (cuuint32_t)rank, const_cast<void*>(base), d, s, b, e,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(REMORA_B200_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return REMORA_B200_OK;
}

inline int num_sms() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
  return n;
}

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

// Unique id of the current thread's CUDA context (ids are never reused
// within a process, unlike context handles).  0 when the driver cannot say.
inline unsigned long long current_ctx_id() {
  static CtxGetCurrentFn get_cur = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_cur = reinterpret_cast<CtxGetCurrentFn>(p);
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
  });
  CUcontext c = nullptr;
  unsigned long long id = 0;
  if (get_cur && get_id && get_cur(&c) == CUDA_SUCCESS && c && get_id(c, &id) == CUDA_SUCCESS)
    return id;
  return 0;
}

// Reads and clears the device error word (synchronises the stream).
inline int collect_device_error(cudaStream_t st) {
  int v = 0, zero = 0;
  RB_CUDA(cudaStreamSynchronize(st));
  RB_CUDA(cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)));
  if (v != 0) {
    RB_CUDA(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)));
    if (v == 1) return fail(REMORA_B200_ERR_TIMEOUT, "a device-side wait timed out");
    return fail(REMORA_B200_ERR_INVALID, "device reported error %d", v);
  }
  return REMORA_B200_OK;
}

}  // namespace rb
