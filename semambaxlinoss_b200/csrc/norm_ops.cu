// RMS normalisation over the last dimension with a learned gain, for sm_100a.
//
// Reference behaviour (paths relative to the reference project): the pre-norm Block's
// RMSNorm (models/mamba_block.py:335-342 builds it with rms_norm=True; the reference takes
// the class from mamba_ssm), y = x / sqrt(mean(x^2) + eps) * w, evaluated in fp32 and
// returned in x's dtype.
//
// One warp per row of d elements (lane j owns elements j, j + 32, ...); a warp takes
// kRowsPerWarp consecutive rows. Forward reads a row once and writes y and the row's
// r = 1 / rms. Backward reads x, dy and r and writes
//   dx = r w dy - x r^3 mean(x w dy),
// summing dw = dy x r over its rows in registers; the warps of a CTA add their sums in
// shared memory in warp order, each CTA writes one partial row, and the rows are reduced
// over CTAs by the fixed-order column sum (bitwise deterministic).
#include <cuda_bf16.h>

#include "semx_common.cuh"
#include "semx_reduce.cuh"

namespace {

constexpr int kWarps = 8;
constexpr int kRowsPerWarp = 16;
constexpr int kRowsPerCta = kWarps * kRowsPerWarp;
constexpr int kMaxD = 1024;

struct NormParams {
  int64_t n, d;
  float eps;
  const void* x;
  const float* w;
  void* y;
  float* rstd;
  const void* dy;
  void* dx;
  float* part;  // (CTAs, d) partial dw rows
};

template <bool BF16>
__device__ __forceinline__ float ldf(const void* base, int64_t i) {
  if (BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[i]);
  return reinterpret_cast<const float*>(base)[i];
}
template <bool BF16>
__device__ __forceinline__ void stf(void* base, int64_t i, float v) {
  if (BF16) reinterpret_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16(v);
  else reinterpret_cast<float*>(base)[i] = v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  return v;
}

// EPL elements per lane (32 EPL >= d).
template <bool BF16, int EPL>
__global__ void __launch_bounds__(kWarps * 32) rms_norm_fwd_kernel(const NormParams p) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int d = (int)p.d;
  const int64_t r0 = ((int64_t)blockIdx.x * kWarps + warp) * kRowsPerWarp;
  float w[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) w[e] = lane + 32 * e < d ? p.w[lane + 32 * e] : 0.f;
  for (int i = 0; i < kRowsPerWarp; ++i) {
    const int64_t r = r0 + i;
    if (r >= p.n) break;
    float v[EPL];
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const int j = lane + 32 * e;
      v[e] = j < d ? ldf<BF16>(p.x, r * d + j) : 0.f;
      ss = fmaf(v[e], v[e], ss);
    }
    const float rs = rsqrtf(warp_sum(ss) / (float)d + p.eps);
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const int j = lane + 32 * e;
      if (j < d) stf<BF16>(p.y, r * d + j, (v[e] * rs) * w[e]);
    }
    if (lane == 0 && p.rstd != nullptr) p.rstd[r] = rs;
  }
}

template <bool BF16, int EPL>
__global__ void __launch_bounds__(kWarps * 32) rms_norm_bwd_kernel(const NormParams p) {
  __shared__ float red[kWarps][32 * EPL];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int d = (int)p.d;
  const int64_t r0 = ((int64_t)blockIdx.x * kWarps + warp) * kRowsPerWarp;
  float w[EPL], dw[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    w[e] = lane + 32 * e < d ? p.w[lane + 32 * e] : 0.f;
    dw[e] = 0.f;
  }
  for (int i = 0; i < kRowsPerWarp; ++i) {
    const int64_t r = r0 + i;
    if (r >= p.n) break;
    const float rs = p.rstd[r];
    float v[EPL], g[EPL];
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const int j = lane + 32 * e;
      v[e] = j < d ? ldf<BF16>(p.x, r * d + j) : 0.f;
      g[e] = j < d ? ldf<BF16>(p.dy, r * d + j) : 0.f;
      s = fmaf(v[e], w[e] * g[e], s);
      dw[e] = fmaf(g[e], v[e] * rs, dw[e]);
    }
    const float m = warp_sum(s) / (float)d;
    const float c = rs * rs * rs * m;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const int j = lane + 32 * e;
      if (j < d) stf<BF16>(p.dx, r * d + j, rs * w[e] * g[e] - v[e] * c);
    }
  }
#pragma unroll
  for (int e = 0; e < EPL; ++e) red[warp][lane + 32 * e] = dw[e];
  __syncthreads();
  for (int j = threadIdx.x; j < d; j += kWarps * 32) {
    float acc = 0.f;
#pragma unroll
    for (int q = 0; q < kWarps; ++q) acc += red[q][j];
    p.part[(int64_t)blockIdx.x * d + j] = acc;
  }
}

int epl_for(int64_t d) {
  int e = 1;
  while (32 * e < d) e *= 2;
  return e;
}

template <bool BF16>
int launch_norm(bool bwd, const NormParams& p, cudaStream_t st) {
  const unsigned grid = (unsigned)semx::cdiv(p.n, kRowsPerCta);
  switch (epl_for(p.d)) {
#define SEMX_E(EV)                                                                \
  case EV:                                                                        \
    if (bwd) rms_norm_bwd_kernel<BF16, EV><<<grid, kWarps * 32, 0, st>>>(p);      \
    else rms_norm_fwd_kernel<BF16, EV><<<grid, kWarps * 32, 0, st>>>(p);          \
    return semx::check_launch(bwd ? "rms_norm_bwd_kernel" : "rms_norm_fwd_kernel");
    SEMX_E(1)
    SEMX_E(2)
    SEMX_E(4)
    SEMX_E(8)
    SEMX_E(16)
    SEMX_E(32)
#undef SEMX_E
  }
  return semx::fail(SEMX_ERR_UNSUPPORTED, "rms_norm: width %lld", (long long)p.d);
}

int norm_validate(const SemxRmsNormArgs* a, bool bwd) {
  SEMX_REQUIRE(a->n >= 0 && a->d >= 1, SEMX_ERR_SHAPE, "rms_norm: n=%lld, d=%lld", (long long)a->n,
               (long long)a->d);
  SEMX_REQUIRE(a->d <= kMaxD, SEMX_ERR_UNSUPPORTED, "rms_norm: width %lld > %d", (long long)a->d, kMaxD);
  SEMX_REQUIRE(a->eps >= 0.f, SEMX_ERR_SHAPE, "rms_norm: eps < 0");
  if (a->n > 0) {
    SEMX_REQUIRE(a->x && a->weight, SEMX_ERR_NULL, "rms_norm: x / weight is NULL");
    if (!bwd) SEMX_REQUIRE(a->y, SEMX_ERR_NULL, "rms_norm: y is NULL");
    if (bwd)
      SEMX_REQUIRE(a->rstd && a->dy && a->dx, SEMX_ERR_NULL, "rms_norm bwd: rstd / dy / dx is NULL");
  }
  return SEMX_OK;
}

NormParams norm_params(const SemxRmsNormArgs* a) {
  NormParams p = {};
  p.n = a->n; p.d = a->d; p.eps = a->eps;
  p.x = a->x; p.w = a->weight; p.y = a->y; p.rstd = a->rstd; p.dy = a->dy; p.dx = a->dx;
  return p;
}

}  // namespace

extern "C" {

size_t semx_rms_norm_args_size(void) { return sizeof(SemxRmsNormArgs); }

size_t semx_rms_norm_workspace_bytes(const SemxRmsNormArgs* a) {
  if (a == nullptr || a->n < 0 || a->d < 1) return 0;
  const int64_t rows = semx::cdiv(a->n, kRowsPerCta);
  return ((size_t)rows * a->d + semx::colsum_group_floats(rows, a->d)) * sizeof(float);
}

int semx_rms_norm_fwd(const SemxRmsNormArgs* a, semx_stream_t stream) {
  SEMX_CHECK_ARGS(a, SemxRmsNormArgs);
  int rc = norm_validate(a, false);
  if (rc != SEMX_OK) return rc;
  if (a->n == 0) return SEMX_OK;
  rc = semx::bind_device({a->y});
  if (rc != SEMX_OK) return rc;
  const NormParams p = norm_params(a);
  cudaStream_t st = semx::as_stream(stream);
  return a->bf16 ? launch_norm<true>(false, p, st) : launch_norm<false>(false, p, st);
}

int semx_rms_norm_bwd(const SemxRmsNormArgs* a, semx_stream_t stream) {
  SEMX_CHECK_ARGS(a, SemxRmsNormArgs);
  int rc = norm_validate(a, true);
  if (rc != SEMX_OK) return rc;
  SEMX_REQUIRE(a->dweight != nullptr, SEMX_ERR_NULL, "rms_norm bwd: dweight is NULL");
  SEMX_REQUIRE(a->workspace != nullptr, SEMX_ERR_WORKSPACE, "rms_norm bwd: workspace is NULL");
  rc = semx::bind_device({a->dweight});
  if (rc != SEMX_OK) return rc;
  cudaStream_t st = semx::as_stream(stream);
  NormParams p = norm_params(a);
  float* ws = reinterpret_cast<float*>(a->workspace);
  p.part = ws;
  const int64_t rows = semx::cdiv(a->n, kRowsPerCta);
  if (rows == 0) {
    cudaMemsetAsync(a->dweight, 0, (size_t)a->d * sizeof(float), st);  // no rows: dw = 0
    return SEMX_OK;
  }
  rc = a->bf16 ? launch_norm<true>(true, p, st) : launch_norm<false>(true, p, st);
  if (rc != SEMX_OK) return rc;
  semx::Segments seg = {};
  seg.n = 1;
  seg.out[0] = a->dweight;
  seg.len[0] = a->d;
  return semx::colsum(ws, rows, a->d, ws + (size_t)rows * a->d, seg, st);
}

}  // extern "C"
