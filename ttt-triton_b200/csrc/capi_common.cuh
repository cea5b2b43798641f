// Host-side helpers shared by the C-ABI entry points: status codes, the last-error
// message, argument checks and launch configuration.
#pragma once

#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>

#include <atomic>

#include "../../include/ttt_b200.h"

namespace ttt {

// Last error message of the calling host thread (returned by ttt_last_error()).
inline char* last_error_buffer() {
  static thread_local char buf[512] = {0};
  return buf;
}

inline int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(last_error_buffer(), 512, fmt, ap);
  va_end(ap);
  return code;
}

inline int ok() {
  last_error_buffer()[0] = 0;
  return TTT_OK;
}

inline bool valid_dtype(int dt) { return dt == TTT_DTYPE_F32 || dt == TTT_DTYPE_BF16 || dt == TTT_DTYPE_F16; }

// Configure dynamic shared memory for a kernel and check it fits one CTA of this device.
template <typename K>
inline int prepare_smem(K kernel, size_t smem_bytes, const char* name) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(TTT_ERR_CUDA, "%s: cudaGetDevice: %s", name, cudaGetErrorString(e));
  int max_optin = 0;
  e = cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e != cudaSuccess) return fail(TTT_ERR_CUDA, "%s: cudaDeviceGetAttribute: %s", name, cudaGetErrorString(e));
  if (smem_bytes > (size_t)max_optin)
    return fail(TTT_ERR_UNSUPPORTED, "%s: needs %zu bytes of shared memory per CTA, device allows %d", name, smem_bytes,
                max_optin);
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bytes);
  if (e != cudaSuccess) return fail(TTT_ERR_CUDA, "%s: cudaFuncSetAttribute: %s", name, cudaGetErrorString(e));
  return TTT_OK;
}

// Kernels the library has enqueued in this process (ttt_kernel_launches()).
inline std::atomic<unsigned long long>& launch_counter() {
  static std::atomic<unsigned long long> n{0};
  return n;
}

// After each kernel launch: reports a failed launch, counts a successful one.
inline int check_launch(const char* name) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(TTT_ERR_CUDA, "%s: launch failed: %s", name, cudaGetErrorString(e));
  launch_counter().fetch_add(1, std::memory_order_relaxed);
  return ok();
}

}  // namespace ttt

#define TTT_REQUIRE(cond, code, ...) \
  do {                               \
    if (!(cond)) return ::ttt::fail((code), __VA_ARGS__); \
  } while (0)
