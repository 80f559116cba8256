// ABI bookkeeping: version, status strings and the per-host-thread error message.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "semx_common.cuh"

namespace semx {

thread_local char g_last_error[512] = {0};
std::atomic<uint64_t> g_launches{0};

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

void clear_error() { g_last_error[0] = '\0'; }

int bind_device(std::initializer_list<const void*> ptrs) {
  const void* p = nullptr;
  for (const void* q : ptrs) {
    if (q != nullptr) {
      p = q;
      break;
    }
  }
  if (p == nullptr) return SEMX_OK;
  cudaPointerAttributes attr;
  cudaError_t e = cudaPointerGetAttributes(&attr, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(SEMX_ERR_DEVICE, "cudaPointerGetAttributes: %s", cudaGetErrorString(e));
  }
  if (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged)
    return fail(SEMX_ERR_DEVICE, "operand %p is not device memory", p);
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess || cur != attr.device) {
    e = cudaSetDevice(attr.device);
    if (e != cudaSuccess)
      return fail(SEMX_ERR_DEVICE, "cudaSetDevice(%d): %s", attr.device, cudaGetErrorString(e));
  }
  return SEMX_OK;
}

int make_rowmap(int64_t S, int64_t L, int reverse, int64_t G, int64_t A, int64_t B, int64_t Cst, RowMap* m,
                const char* what) {
  if (G < 0 || A < 0 || B < 0 || Cst < 0)
    return fail(SEMX_ERR_SHAPE, "%s: negative token-layout field", what);
  m->G = G > 0 ? G : 1;
  m->A = A > 0 ? A : L;
  m->B = B;
  const int64_t step = Cst > 0 ? Cst : 1;
  m->base = reverse && L > 0 ? (L - 1) * step : 0;
  m->dstep = reverse ? -step : step;
  if (S <= 0 || L <= 0) return SEMX_OK;
  if (S >= ((int64_t)1 << 31) || m->G >= ((int64_t)1 << 31))
    return fail(SEMX_ERR_SHAPE, "%s: token layout with S=%lld or seq_group=%lld >= 2^31", what, (long long)S,
                (long long)m->G);
  if (S % m->G != 0)
    return fail(SEMX_ERR_SHAPE, "%s: S=%lld is not a multiple of seq_group=%lld", what, (long long)S,
                (long long)m->G);
  // The largest row index any (s, t) reaches (every coefficient is non-negative, so the
  // map is monotone in each index), in 128-bit arithmetic so that no field value can wrap
  // it below the bound. The map is not checked to be one-to-one: a layout that sends two
  // tokens to one row gives undefined results, but every access stays inside the rows.
  const __int128 top = (__int128)((S - 1) / m->G) * m->A + (__int128)(m->G - 1 < S - 1 ? m->G - 1 : S - 1) * m->B +
                       (__int128)(L - 1) * step;
  if (top >= (__int128)S * L)
    return fail(SEMX_ERR_SHAPE, "%s: token layout reaches beyond row %lld", what, (long long)(S * L - 1));
  return SEMX_OK;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(SEMX_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return SEMX_OK;
}

}  // namespace semx

extern "C" {

int semx_abi_version(void) { return SEMX_ABI_VERSION; }

const char* semx_status_string(int status) {
  switch (status) {
    case SEMX_OK: return "ok";
    case SEMX_ERR_ABI: return "argument struct size mismatch (header/library version skew)";
    case SEMX_ERR_NULL: return "required pointer is NULL";
    case SEMX_ERR_SHAPE: return "invalid shape";
    case SEMX_ERR_UNSUPPORTED: return "unsupported configuration";
    case SEMX_ERR_ALIGN: return "misaligned pointer";
    case SEMX_ERR_LAUNCH: return "CUDA launch failed";
    case SEMX_ERR_WORKSPACE: return "workspace missing";
    case SEMX_ERR_DEVICE: return "operand is not device memory";
    default: return "unknown status";
  }
}

const char* semx_last_error(void) { return semx::g_last_error; }

uint64_t semx_launch_count(void) { return semx::g_launches.load(std::memory_order_relaxed); }

}  // extern "C"
