// LinOSS readout and D skip, for sm_100a.
//
// Reference behaviour (paths relative to the reference project):
//   models/linoss/linoss.py:118-120   Cy = einsum("fn,btn->btf", C, ys).real; Du = x * D;
//                                     return Cy + Du
// i.e. per token row r and channel h (C complex (H, P) stored as (H, P, 2)):
//   y[r, h] = sum_p (C_re[h, p] y2_re[r, p] - C_im[h, p] y2_im[r, p]) + D[h] x[r, h].
// With P <= 32 oscillators the readout is 2P multiply-adds per output, so both directions
// are bound by the (rows, H) tensors they stream, not by arithmetic.
//
// Thread h of a CTA owns channel h of a 256-channel tile and keeps C[h, :] in registers;
// a CTA walks kRowsPerCta rows, the y2 rows of kStage rows at a time staged in shared
// memory (every thread reads the same row: broadcast loads).
// Forward: y as above (x and y fp32).
// Backward: dx = D dy and the parameter sums dC_re[h, p] += dy y2_re, dC_im[h, p] -=
// dy y2_im, dD[h] += dy x, summed per thread over the CTA's rows, written as one partial
// row per row block and reduced over row blocks by the fixed-order column sum (bitwise
// reproducible). The state gradient dy2[r, p] = sum_h dy[r, h] conj(C[h, p]), a contraction
// over channels, is left to a GEMM on the caller's side.
#include "semx_common.cuh"
#include "semx_reduce.cuh"

namespace {

constexpr int kThreads = 256;        // channels per CTA tile
constexpr int kRowsPerCta = 512;
constexpr int kStage = 32;           // y2 rows staged at a time
constexpr int kUnroll = 16;          // rows whose loads a thread issues together (forward)
constexpr int kUnrollB = 8;          // the same in the backward, whose accumulators leave fewer registers
constexpr int kMaxP = 32;

struct RParams {
  int64_t rows, H, P;
  const float* x;
  const float* y2;  // (rows, P) complex, interleaved
  const float* C;   // (H, P, 2)
  const float* D;
  float* y;
  const float* dy;
  float* dx;
  float* part;  // (row blocks, 2 H P + H)
};

template <int PT>
__device__ __forceinline__ void load_c(const RParams& p, int64_t h, float (&cr)[PT], float (&ci)[PT]) {
#pragma unroll
  for (int k = 0; k < PT; ++k) {
    const bool ok = h < p.H && k < p.P;
    cr[k] = ok ? p.C[(h * p.P + k) * 2] : 0.f;
    ci[k] = ok ? p.C[(h * p.P + k) * 2 + 1] : 0.f;
  }
}

// Stages y2 rows [r, r + n) into s (kStage rows of 2 PT floats; slots past P or n zero).
template <int PT>
__device__ __forceinline__ void stage_y2(const RParams& p, float* s, int64_t r, int n) {
  for (int i = threadIdx.x; i < kStage * 2 * PT; i += kThreads) {
    const int row = i / (2 * PT), col = i % (2 * PT);
    s[i] = (row < n && col < 2 * p.P) ? p.y2[(r + row) * 2 * p.P + col] : 0.f;
  }
}

template <int PT>
__global__ void __launch_bounds__(kThreads) linoss_readout_fwd_kernel(const RParams p) {
  __shared__ __align__(16) float s_y2[kStage * 2 * PT];
  const int64_t h = (int64_t)blockIdx.y * kThreads + threadIdx.x;
  const bool hv = h < p.H;
  float cr[PT], ci[PT];
  load_c<PT>(p, h, cr, ci);
  const float d = hv ? p.D[h] : 0.f;
  const int64_t r0 = (int64_t)blockIdx.x * kRowsPerCta;
  const int64_t r1 = min(r0 + kRowsPerCta, p.rows);
  for (int64_t rs = r0; rs < r1; rs += kStage) {
    const int n = (int)min((int64_t)kStage, r1 - rs);
    __syncthreads();  // the previous stage's rows are consumed
    stage_y2<PT>(p, s_y2, rs, n);
    __syncthreads();
    for (int i0 = 0; i0 < n; i0 += kUnroll) {
      // kUnroll rows' loads are issued before any of them is used.
      float xv[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) xv[u] = (hv && i0 + u < n) ? __ldcs(p.x + (rs + i0 + u) * p.H + h) : 0.f;
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        if (i0 + u >= n) break;
        const float4* row = reinterpret_cast<const float4*>(s_y2 + (i0 + u) * 2 * PT);
        float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
        for (int q = 0; q < PT / 2; ++q) {
          const float4 v = row[q];  // (re, im) of oscillators 2q, 2q + 1
          acc0 = fmaf(cr[2 * q], v.x, acc0);
          acc1 = fmaf(-ci[2 * q], v.y, acc1);
          acc0 = fmaf(cr[2 * q + 1], v.z, acc0);
          acc1 = fmaf(-ci[2 * q + 1], v.w, acc1);
        }
        if (hv) __stcs(p.y + (rs + i0 + u) * p.H + h, (acc0 + acc1) + d * xv[u]);
      }
    }
  }
}

template <int PT>
__global__ void __launch_bounds__(kThreads) linoss_readout_bwd_kernel(const RParams p) {
  __shared__ __align__(16) float s_y2[kStage * 2 * PT];
  const int64_t h = (int64_t)blockIdx.y * kThreads + threadIdx.x;
  const bool hv = h < p.H;
  const float d = hv ? p.D[h] : 0.f;
  float gr[PT], gi[PT];
#pragma unroll
  for (int k = 0; k < PT; ++k) gr[k] = gi[k] = 0.f;
  float gd = 0.f;
  const int64_t r0 = (int64_t)blockIdx.x * kRowsPerCta;
  const int64_t r1 = min(r0 + kRowsPerCta, p.rows);
  for (int64_t rs = r0; rs < r1; rs += kStage) {
    const int n = (int)min((int64_t)kStage, r1 - rs);
    __syncthreads();
    stage_y2<PT>(p, s_y2, rs, n);
    __syncthreads();
    for (int i0 = 0; i0 < n; i0 += kUnrollB) {
      float gv[kUnrollB], xv[kUnrollB];
#pragma unroll
      for (int u = 0; u < kUnrollB; ++u) {
        const bool ok = hv && i0 + u < n;
        gv[u] = ok ? __ldcs(p.dy + (rs + i0 + u) * p.H + h) : 0.f;
        xv[u] = ok ? __ldcs(p.x + (rs + i0 + u) * p.H + h) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < kUnrollB; ++u) {
        if (i0 + u >= n) break;
        const float g = gv[u];
        if (hv) __stcs(p.dx + (rs + i0 + u) * p.H + h, d * g);
        gd = fmaf(g, xv[u], gd);
        const float4* row = reinterpret_cast<const float4*>(s_y2 + (i0 + u) * 2 * PT);
#pragma unroll
        for (int q = 0; q < PT / 2; ++q) {
          const float4 v = row[q];
          gr[2 * q] = fmaf(g, v.x, gr[2 * q]);
          gi[2 * q] = fmaf(-g, v.y, gi[2 * q]);
          gr[2 * q + 1] = fmaf(g, v.z, gr[2 * q + 1]);
          gi[2 * q + 1] = fmaf(-g, v.w, gi[2 * q + 1]);
        }
      }
    }
  }
  if (!hv) return;
  // Partial row of this row block: [dC (H, P, 2) | dD (H)].
  float* prow = p.part + (int64_t)blockIdx.x * (2 * p.H * p.P + p.H);
#pragma unroll
  for (int k = 0; k < PT; ++k) {
    if (k < p.P) {
      prow[(h * p.P + k) * 2] = gr[k];
      prow[(h * p.P + k) * 2 + 1] = gi[k];
    }
  }
  prow[2 * p.H * p.P + h] = gd;
}

template <int PT>
int launch(bool bwd, const RParams& p, cudaStream_t st) {
  const dim3 grid((unsigned)semx::cdiv(p.rows, kRowsPerCta), (unsigned)semx::cdiv(p.H, kThreads));
  if (bwd) {
    linoss_readout_bwd_kernel<PT><<<grid, kThreads, 0, st>>>(p);
    return semx::check_launch("linoss_readout_bwd_kernel");
  }
  linoss_readout_fwd_kernel<PT><<<grid, kThreads, 0, st>>>(p);
  return semx::check_launch("linoss_readout_fwd_kernel");
}

int dispatch(bool bwd, const RParams& p, cudaStream_t st) {
  if (p.P <= 8) return launch<8>(bwd, p, st);
  if (p.P <= 16) return launch<16>(bwd, p, st);
  return launch<32>(bwd, p, st);
}

int readout_validate(const SemxLinossReadoutArgs* a, bool bwd) {
  SEMX_REQUIRE(a->rows >= 0 && a->H >= 1 && a->P >= 1, SEMX_ERR_SHAPE, "linoss_readout: rows=%lld, H=%lld, P=%lld",
               (long long)a->rows, (long long)a->H, (long long)a->P);
  SEMX_REQUIRE(a->P <= kMaxP, SEMX_ERR_UNSUPPORTED, "linoss_readout: P=%lld > %d", (long long)a->P, kMaxP);
  SEMX_REQUIRE(semx::cdiv(a->rows, kRowsPerCta) <= 0x7fffffff && semx::cdiv(a->H, kThreads) <= 65535,
               SEMX_ERR_SHAPE, "linoss_readout: grid too large");
  if (a->rows > 0) {
    SEMX_REQUIRE(a->x && a->y2 && a->C && a->D, SEMX_ERR_NULL, "linoss_readout: x / y2 / C / D is NULL");
    if (!bwd) SEMX_REQUIRE(a->y, SEMX_ERR_NULL, "linoss_readout: y is NULL");
    if (bwd) {
      SEMX_REQUIRE(a->dy && a->dx && a->dC && a->dD, SEMX_ERR_NULL, "linoss_readout bwd: dy / dx / dC / dD is NULL");
      SEMX_REQUIRE(a->workspace != nullptr, SEMX_ERR_WORKSPACE, "linoss_readout bwd: workspace is NULL");
    }
  }
  return SEMX_OK;
}

RParams readout_params(const SemxLinossReadoutArgs* a) {
  RParams p = {};
  p.rows = a->rows; p.H = a->H; p.P = a->P;
  p.x = a->x; p.y2 = a->y2; p.C = a->C; p.D = a->D; p.y = a->y; p.dy = a->dy; p.dx = a->dx;
  return p;
}

}  // namespace

extern "C" {

size_t semx_linoss_readout_args_size(void) { return sizeof(SemxLinossReadoutArgs); }

size_t semx_linoss_readout_workspace_bytes(const SemxLinossReadoutArgs* a) {
  if (a == nullptr || a->rows < 0 || a->H < 1 || a->P < 1) return 0;
  const int64_t nrb = semx::cdiv(a->rows, kRowsPerCta);
  const int64_t K = 2 * a->H * a->P + a->H;
  return ((size_t)nrb * K + semx::colsum_group_floats(nrb, K)) * sizeof(float);
}

int semx_linoss_readout_fwd(const SemxLinossReadoutArgs* a, semx_stream_t stream) {
  SEMX_CHECK_ARGS(a, SemxLinossReadoutArgs);
  int rc = readout_validate(a, false);
  if (rc != SEMX_OK) return rc;
  if (a->rows == 0) return SEMX_OK;
  rc = semx::bind_device({a->y});
  if (rc != SEMX_OK) return rc;
  return dispatch(false, readout_params(a), semx::as_stream(stream));
}

int semx_linoss_readout_bwd(const SemxLinossReadoutArgs* a, semx_stream_t stream) {
  SEMX_CHECK_ARGS(a, SemxLinossReadoutArgs);
  int rc = readout_validate(a, true);
  if (rc != SEMX_OK) return rc;
  rc = semx::bind_device({a->dC});
  if (rc != SEMX_OK) return rc;
  cudaStream_t st = semx::as_stream(stream);
  const int64_t K = 2 * a->H * a->P + a->H;
  if (a->rows == 0) {  // no rows: the parameter gradients are zero
    cudaMemsetAsync(a->dC, 0, (size_t)(2 * a->H * a->P) * sizeof(float), st);
    cudaMemsetAsync(a->dD, 0, (size_t)a->H * sizeof(float), st);
    return semx::check_launch("linoss_readout bwd: zero gradients");
  }
  RParams p = readout_params(a);
  float* ws = reinterpret_cast<float*>(a->workspace);
  p.part = ws;
  rc = dispatch(true, p, st);
  if (rc != SEMX_OK) return rc;
  const int64_t nrb = semx::cdiv(a->rows, kRowsPerCta);
  semx::Segments seg = {};
  seg.n = 2;
  seg.out[0] = a->dC;
  seg.len[0] = 2 * a->H * a->P;
  seg.out[1] = a->dD;
  seg.len[1] = a->H;
  return semx::colsum(ws, nrb, K, ws + (size_t)nrb * K, seg, st);
}

}  // extern "C"
