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

// Token row of step t of sequence s: (s / G) * A + (s % G) * B + t' * Cst, t' = L - 1 - t
// when reversed (the layout fields of the selective-LRU and conv + SiLU structs), split as
// seq(s) + step(t): the reversal is folded into seq's constant term base = (L - 1) * Cst
// and a negative step stride dstep = -Cst, so a kernel that hoists seq(s) pays one
// multiply-add per token row, as for the sequence-major layout.
struct RowMap {
  int64_t G, A, B, base, dstep;
  // s and G below 2^31 (checked on the host): one 32-bit division.
  __host__ __device__ __forceinline__ int64_t seq(int64_t s) const {
    if (G == 1) return s * A + base;
    const int64_t q = (int64_t)((uint32_t)s / (uint32_t)G);
    return q * A + (s - q * G) * B + base;
  }
  __host__ __device__ __forceinline__ int64_t step(int64_t t) const { return t * dstep; }
};
// Fills `m` from the layout fields (zeros select the sequence-major layout: G = 1, A = L,
// Cst = 1) and checks that every (s, t) maps below S * L; returns a semx_status.
int make_rowmap(int64_t S, int64_t L, int reverse, int64_t G, int64_t A, int64_t B, int64_t Cst, RowMap* m,
                const char* what);

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
