// Shared helpers for the semx kernels: error reporting across the C ABI, argument
// checks, and small device utilities. Every entry point returns a semx_status code and
// records a message for semx_last_error(); nothing throws.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <initializer_list>

#include "semx.h"

namespace semx {

// Records `fmt` as this host thread's last error and returns `code`.
int fail(int code, const char* fmt, ...);
// Clears this host thread's last error.
void clear_error();
// Converts the pending CUDA error (if any) after a launch into SEMX_ERR_LAUNCH.
int check_launch(const char* what);

// Makes the GPU that owns the first non-NULL pointer of `ptrs` current for this host
// thread, so launches (including on a device's legacy default stream) go to the GPU
// that holds the operands, whichever device the caller's own runtime has current.
int bind_device(std::initializer_list<const void*> ptrs);

inline bool aligned(const void* p, uintptr_t a) {
  return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

inline cudaStream_t as_stream(semx_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// Raises the dynamic shared-memory limit of `kernel` when a launch needs more than the
// 48 KB default. Returns false (with the error recorded) if the attribute is refused.
template <typename K>
inline bool allow_smem(K kernel, size_t bytes) {
  if (bytes <= 48 * 1024) return true;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(bytes));
  if (e != cudaSuccess) {
    fail(SEMX_ERR_LAUNCH, "cudaFuncSetAttribute(%zu B smem): %s", bytes, cudaGetErrorString(e));
    return false;
  }
  return true;
}

}  // namespace semx

#define SEMX_CHECK_ARGS(args, T)                                                     \
  do {                                                                               \
    if ((args) == nullptr) return semx::fail(SEMX_ERR_NULL, "args is NULL");         \
    if ((args)->struct_size != sizeof(T))                                            \
      return semx::fail(SEMX_ERR_ABI, #T ".struct_size=%u but the library expects %zu", \
                        (unsigned)(args)->struct_size, sizeof(T));                   \
  } while (0)

#define SEMX_REQUIRE(cond, code, ...)                 \
  do {                                                \
    if (!(cond)) return semx::fail((code), __VA_ARGS__); \
  } while (0)
