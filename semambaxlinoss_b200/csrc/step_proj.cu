// Low-rank selective-step projections of the SelectiveLRU layer, for sm_100a.
//
// Reference behaviour (paths relative to the reference project):
//   models/selective_lru/selective_lru.py:151-152  dt_nu_up, dt_theta_up = Linear(r, C)
//   models/selective_lru/selective_lru.py:216-220  delta_nu = softplus(dt_nu_up(dnu_r)),
//                                                  delta_theta = dt_theta_up(dth_r)
// (and the rate scale applied to delta_nu, selective_lru.py:205-218). With r = ceil(C / 64)
// these are (rows x r) x (r x C) products: r multiply-adds per output, so both directions
// are bound by the (rows, C) fp32 tensors they write or read, not by arithmetic.
//
// Forward: one pass writes delta_nu = scale * softplus(z_nu W_nu^T + b_nu) and
// delta_theta = z_th W_th^T + b_th; z_nu / z_th are read in place from the token
// projection rows (bf16 or fp32, row stride ldz).
// Backward: one pass over d_delta_nu / d_delta_theta computes
//   g_nu = d_delta_nu * scale * sigmoid(pre_nu)   (pre_nu recomputed from z_nu),
//   g_th = d_delta_theta,
//   dz = g W (per row, summed over channels), dW = g^T z and db = sum_t g (per channel,
// summed over rows). A CTA covers kRowsPerCta rows of one 64-channel tile; a warp takes
// kBatch consecutive rows at a time, loading all of them before computing; lane j owns
// channels 2 j, 2 j + 1 of the tile. Per-row sums over a tile are one transposed warp
// reduction of the 2 r values; with more than one tile, each tile writes its row sums and
// dz_sum_kernel adds the tiles in order. Per-channel sums are summed per lane over the
// CTA's rows, over the CTA's warps in warp order, written as one partial row per row
// block and reduced over row blocks by the fixed-order column sum: every output is
// bitwise reproducible.
#include <cuda_bf16.h>

#include "semx_common.cuh"
#include "semx_math.cuh"
#include "semx_reduce.cuh"

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kTileC = 64;   // channels per CTA tile (2 per lane)
// Consecutive rows a warp loads before it computes them: 4 in the forward. The backward
// of ranks up to 4 takes 2 rows, which fit 80 registers and so 3 CTAs per SM (4 rows:
// 112 registers, 2 CTAs; 513,600 x 256, rank 4: backward 0.844 -> 0.777 ms per call;
// the forward with 2 rows went 0.343 -> 0.400 ms). Higher ranks would spill at 80
// registers and keep 4 rows at the default bound.
constexpr int kBatchF = 4;
template <int R>
constexpr int bwd_batch() { return R <= 4 ? 2 : 4; }
template <int R>
constexpr int bwd_min_ctas() { return R <= 4 ? 3 : 1; }
constexpr int kRowsPerCta = 256;
constexpr int kMaxRank = 8;

struct PParams {
  int64_t rows, C, ldz;
  int ntiles;
  float scale;
  const void* zn;
  const void* zt;
  const float* Wn;
  const float* bn;
  const float* Wt;
  const float* bt;
  float* dnu;
  float* dth;
  const float* gdnu;
  const float* gdth;
  void* dzn;
  void* dzt;
  float* part;    // (row blocks, 2 (C R + C)) per-channel partial sums
  float* dzpart;  // (ntiles, rows, 2 R) per-tile row sums when ntiles > 1
};

template <bool BF16>
__device__ __forceinline__ float ldz(const void* base, int64_t i) {
  if (BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[i]);
  return reinterpret_cast<const float*>(base)[i];
}
template <bool BF16>
__device__ __forceinline__ void stz(void* base, int64_t i, float v) {
  if (BF16) reinterpret_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16(v);
  else reinterpret_cast<float*>(base)[i] = v;
}

// This lane's channels c0, c0 + 1 of the tile: weights and biases (zero past C).
template <int R>
struct LaneW {
  float wn[2][R], wt[2][R], bn[2], bt[2];
};
template <int R>
__device__ __forceinline__ void load_lane_w(const PParams& p, int64_t c0, LaneW<R>& w) {
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int64_t c = c0 + j;
    const bool ok = c < p.C;
#pragma unroll
    for (int k = 0; k < R; ++k) {
      w.wn[j][k] = ok ? p.Wn[c * R + k] : 0.f;
      w.wt[j][k] = ok ? p.Wt[c * R + k] : 0.f;
    }
    w.bn[j] = ok ? p.bn[c] : 0.f;
    w.bt[j] = ok ? p.bt[c] : 0.f;
  }
}

// Two consecutive fp32 values of row r at channel c0 (vector form when both are in range
// and C is even, so every row start is 8-byte aligned).
__device__ __forceinline__ float2 ld2f(const float* base, int64_t r, int64_t C, int64_t c0, bool vec) {
  if (vec && c0 + 1 < C) return __ldcs(reinterpret_cast<const float2*>(base + r * C + c0));
  return make_float2(c0 < C ? __ldcs(base + r * C + c0) : 0.f, c0 + 1 < C ? __ldcs(base + r * C + c0 + 1) : 0.f);
}
__device__ __forceinline__ void st2f(float* base, int64_t r, int64_t C, int64_t c0, bool vec, float a, float b) {
  if (vec && c0 + 1 < C) {
    __stcs(reinterpret_cast<float2*>(base + r * C + c0), make_float2(a, b));
  } else {
    if (c0 < C) __stcs(base + r * C + c0, a);
    if (c0 + 1 < C) __stcs(base + r * C + c0 + 1, b);
  }
}

// The z values of a batch of kBatch rows, spread over the lanes: value q = b * 2R + k
// (row b of the batch; k < R: z_nu[k], else z_th[k - R]) is register q / 32 of lane
// q % 32, read back with a shuffle. Rows past the end repeat the last row.
template <int R, int NB>
constexpr int z_regs() { return (NB * 2 * R + 31) / 32; }
template <bool BF16, int R, int NB>
__device__ __forceinline__ void load_batch_z(const PParams& p, int64_t rb, int lane, float (&zv)[z_regs<R, NB>()]) {
#pragma unroll
  for (int i = 0; i < z_regs<R, NB>(); ++i) {
    const int q = i * 32 + lane;
    const int b = q / (2 * R), k = q % (2 * R);
    float v = 0.f;
    if (b < NB) {
      const int64_t r = min(rb + b, p.rows - 1);
      v = k < R ? ldz<BF16>(p.zn, r * p.ldz + k) : ldz<BF16>(p.zt, r * p.ldz + k - R);
    }
    zv[i] = v;
  }
}
template <int R, int NB>
__device__ __forceinline__ float batch_z(const float (&zv)[z_regs<R, NB>()], int b, int k) {
  const int q = b * 2 * R + k;
  return __shfl_sync(0xffffffffu, zv[q / 32], q % 32);
}

// A warp takes kBatch consecutive rows at a time and issues the loads of its next batch
// before computing the current one, so its reads stay in flight while it computes.
template <bool BF16, int R>
__global__ void __launch_bounds__(kThreads) step_proj_fwd_kernel(const PParams p) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t c0 = (int64_t)blockIdx.y * kTileC + 2 * lane;
  LaneW<R> w;
  load_lane_w<R>(p, c0, w);
  const bool vec = (p.C % 2) == 0;
  const int64_t r0 = (int64_t)blockIdx.x * kRowsPerCta;
  constexpr int kBatch = kBatchF;
  constexpr int kStep = kWarps * kBatch;
  float zn_next[z_regs<R, kBatch>()];
  if (r0 + warp * kBatch < p.rows) load_batch_z<BF16, R, kBatch>(p, r0 + warp * kBatch, lane, zn_next);
  for (int i0 = warp * kBatch; i0 < kRowsPerCta; i0 += kStep) {
    if (r0 + i0 >= p.rows) break;
    float zv[z_regs<R, kBatch>()];
#pragma unroll
    for (int i = 0; i < z_regs<R, kBatch>(); ++i) zv[i] = zn_next[i];
    if (i0 + kStep < kRowsPerCta && r0 + i0 + kStep < p.rows) load_batch_z<BF16, R, kBatch>(p, r0 + i0 + kStep, lane, zn_next);
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const int64_t r = r0 + i0 + b;
      float zn[R], zt[R];
#pragma unroll
      for (int k = 0; k < R; ++k) {
        zn[k] = batch_z<R, kBatch>(zv, b, k);
        zt[k] = batch_z<R, kBatch>(zv, b, R + k);
      }
      if (r >= p.rows) break;
      float on[2], ot[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float a = w.bn[j], t = w.bt[j];
#pragma unroll
        for (int k = 0; k < R; ++k) {
          a = fmaf(w.wn[j][k], zn[k], a);
          t = fmaf(w.wt[j][k], zt[k], t);
        }
        on[j] = semx::softplus(a) * p.scale;
        ot[j] = t;
      }
      st2f(p.dnu, r, p.C, c0, vec, on[0], on[1]);
      st2f(p.dth, r, p.C, c0, vec, ot[0], ot[1]);
    }
  }
}

// Sums v[0..V) (V a power of two <= 32) over the 32 lanes: transposed halving, each round
// sending half of the remaining values, then butterflies; lane l ends with the total of
// value index l / (32 / V). log2(V) + log2(32 / V) rounds, V - 1 + log2(32 / V) shuffles.
template <int V>
__device__ __forceinline__ float warp_reduce_transposed(float (&v)[V], int lane) {
#pragma unroll
  for (int r = 0; (1 << r) < V; ++r) {
    const int m = 16 >> r;
    const int n = V >> (r + 1);
    const bool up = (lane & m) != 0;
#pragma unroll
    for (int i = 0; i < n; ++i) {
      const float send = up ? v[i] : v[i + n];
      const float keep = up ? v[i + n] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, m);
    }
  }
#pragma unroll
  for (int m = (32 / V) / 2; m >= 1; m /= 2) v[0] += __shfl_xor_sync(0xffffffffu, v[0], m);
  return v[0];
}

// d softplus / dx = sigmoid(x) (1 above the softplus threshold 20) from the fast
// exponential __expf (relative error a few units in the last place, well inside the
// backward's tolerance) and the reciprocal __frcp_rn, instead of the division of
// semx::softplus_grad.
__device__ __forceinline__ float softplus_grad_fast(float x) {
  return x > 20.f ? 1.f : __frcp_rn(1.f + __expf(-x));
}

template <int R>
constexpr int dz_values() {  // 2 R rounded up to a power of two
  return 2 * R <= 2 ? 2 : 2 * R <= 4 ? 4 : 2 * R <= 8 ? 8 : 16;
}

template <bool BF16, int R>
__global__ void __launch_bounds__(kThreads, bwd_min_ctas<R>()) step_proj_bwd_kernel(const PParams p) {
  constexpr int V = dz_values<R>();
  __shared__ float red[kWarps][kTileC];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t c0 = (int64_t)blockIdx.y * kTileC + 2 * lane;
  LaneW<R> w;
  load_lane_w<R>(p, c0, w);
  const bool vec = (p.C % 2) == 0;
  float dWn[2][R], dWt[2][R], dbn[2], dbt[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    dbn[j] = dbt[j] = 0.f;
#pragma unroll
    for (int k = 0; k < R; ++k) dWn[j][k] = dWt[j][k] = 0.f;
  }
  const int64_t r0 = (int64_t)blockIdx.x * kRowsPerCta;
  constexpr int kBatch = bwd_batch<R>();
  constexpr int kStep = kWarps * kBatch;
  // The batch at i0: z values spread over the lanes, and this lane's gradient pairs.
  auto load = [&](int i0, float (&zv)[z_regs<R, kBatch>()], float2 (&gn)[kBatch], float2 (&gt)[kBatch]) {
    load_batch_z<BF16, R, kBatch>(p, r0 + i0, lane, zv);
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const int64_t r = min(r0 + i0 + b, p.rows - 1);
      gn[b] = p.gdnu != nullptr ? ld2f(p.gdnu, r, p.C, c0, vec) : make_float2(0.f, 0.f);
      gt[b] = p.gdth != nullptr ? ld2f(p.gdth, r, p.C, c0, vec) : make_float2(0.f, 0.f);
    }
  };
  float zv_next[z_regs<R, kBatch>()];
  float2 gn_next[kBatch], gt_next[kBatch];
  if (r0 + warp * kBatch < p.rows) load(warp * kBatch, zv_next, gn_next, gt_next);
  for (int i0 = warp * kBatch; i0 < kRowsPerCta; i0 += kStep) {
    if (r0 + i0 >= p.rows) break;
    float zv[z_regs<R, kBatch>()];
    float2 gn[kBatch], gt[kBatch];
#pragma unroll
    for (int i = 0; i < z_regs<R, kBatch>(); ++i) zv[i] = zv_next[i];
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      gn[b] = gn_next[b];
      gt[b] = gt_next[b];
    }
    if (i0 + kStep < kRowsPerCta && r0 + i0 + kStep < p.rows) load(i0 + kStep, zv_next, gn_next, gt_next);
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const int64_t r = r0 + i0 + b;
      float zn[R], zt[R];
#pragma unroll
      for (int k = 0; k < R; ++k) {
        zn[k] = batch_z<R, kBatch>(zv, b, k);
        zt[k] = batch_z<R, kBatch>(zv, b, R + k);
      }
      if (r >= p.rows) break;
      float g1[2] = {gn[b].x, gn[b].y}, g2[2] = {gt[b].x, gt[b].y};
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float a = w.bn[j];
#pragma unroll
        for (int k = 0; k < R; ++k) a = fmaf(w.wn[j][k], zn[k], a);
        g1[j] *= p.scale * softplus_grad_fast(a);
      }
      float v[V];
#pragma unroll
      for (int k = 0; k < V; ++k) v[k] = 0.f;
#pragma unroll
      for (int k = 0; k < R; ++k) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          v[k] = fmaf(w.wn[j][k], g1[j], v[k]);
          v[R + k] = fmaf(w.wt[j][k], g2[j], v[R + k]);
          dWn[j][k] = fmaf(g1[j], zn[k], dWn[j][k]);
          dWt[j][k] = fmaf(g2[j], zt[k], dWt[j][k]);
        }
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        dbn[j] += g1[j];
        dbt[j] += g2[j];
      }
      const float tot = warp_reduce_transposed<V>(v, lane);
      const int idx = lane / (32 / V);
      if ((lane % (32 / V)) == 0 && idx < 2 * R) {
        if (p.ntiles > 1) {
          p.dzpart[((int64_t)blockIdx.y * p.rows + r) * (2 * R) + idx] = tot;
        } else if (idx < R) {
          stz<BF16>(p.dzn, r * R + idx, tot);
        } else {
          stz<BF16>(p.dzt, r * R + idx - R, tot);
        }
      }
    }
  }
  // Per-channel sums of the CTA, quantity by quantity: warps in order, one partial row
  // [dW_nu (C R) | db_nu (C) | dW_th (C R) | db_th (C)] per row block.
  const int64_t K = 2 * (p.C * R + p.C);
  float* prow = p.part + (int64_t)blockIdx.x * K;
  for (int q = 0; q < 2 * (R + 1); ++q) {
    const bool th = q >= R + 1;
    const int k = th ? q - (R + 1) : q;  // k == R: the bias
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float v = 0.f;
#pragma unroll
      for (int kk = 0; kk <= R; ++kk) {
        if (kk == k) v = kk == R ? (th ? dbt[j] : dbn[j]) : (th ? dWt[j][kk < R ? kk : 0] : dWn[j][kk < R ? kk : 0]);
      }
      red[warp][2 * lane + j] = v;
    }
    __syncthreads();
    if (threadIdx.x < kTileC) {
      const int64_t c = (int64_t)blockIdx.y * kTileC + threadIdx.x;
      if (c < p.C) {
        float acc = 0.f;
#pragma unroll
        for (int ww = 0; ww < kWarps; ++ww) acc += red[ww][threadIdx.x];
        const int64_t base = th ? p.C * R + p.C : 0;
        prow[base + (k == R ? p.C * R + c : c * R + k)] = acc;
      }
    }
    __syncthreads();
  }
}

// dz rows from the per-tile row sums, tiles in order.
template <bool BF16, int R>
__global__ void __launch_bounds__(256) dz_sum_kernel(const PParams p) {
  const int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (i >= p.rows * 2 * R) return;
  const int64_t r = i / (2 * R);
  const int k = (int)(i % (2 * R));
  float acc = 0.f;
  for (int t = 0; t < p.ntiles; ++t) acc += p.dzpart[((int64_t)t * p.rows + r) * (2 * R) + k];
  if (k < R) stz<BF16>(p.dzn, r * R + k, acc);
  else stz<BF16>(p.dzt, r * R + k - R, acc);
}

template <bool BF16, int R>
int launch(bool bwd, const PParams& p, cudaStream_t st) {
  const dim3 grid((unsigned)semx::cdiv(p.rows, kRowsPerCta), (unsigned)p.ntiles);
  if (!bwd) {
    step_proj_fwd_kernel<BF16, R><<<grid, kThreads, 0, st>>>(p);
    return semx::check_launch("step_proj_fwd_kernel");
  }
  step_proj_bwd_kernel<BF16, R><<<grid, kThreads, 0, st>>>(p);
  int rc = semx::check_launch("step_proj_bwd_kernel");
  if (rc != SEMX_OK || p.ntiles == 1) return rc;
  dz_sum_kernel<BF16, R><<<(unsigned)semx::cdiv(p.rows * 2 * R, 256), 256, 0, st>>>(p);
  return semx::check_launch("dz_sum_kernel");
}

template <bool BF16>
int dispatch(bool bwd, int R, const PParams& p, cudaStream_t st) {
  switch (R) {
#define SEMX_R(RV) \
  case RV:         \
    return launch<BF16, RV>(bwd, p, st);
    SEMX_R(1)
    SEMX_R(2)
    SEMX_R(3)
    SEMX_R(4)
    SEMX_R(5)
    SEMX_R(6)
    SEMX_R(7)
    SEMX_R(8)
#undef SEMX_R
  }
  return semx::fail(SEMX_ERR_UNSUPPORTED, "step_proj: rank %d (1..%d)", R, kMaxRank);
}

int proj_validate(const SemxStepProjArgs* a, bool bwd) {
  SEMX_REQUIRE(a->rows >= 0 && a->C >= 1, SEMX_ERR_SHAPE, "step_proj: rows=%lld, C=%lld", (long long)a->rows,
               (long long)a->C);
  SEMX_REQUIRE(a->rank >= 1 && a->rank <= kMaxRank, SEMX_ERR_UNSUPPORTED, "step_proj: rank %d (1..%d)", a->rank,
               kMaxRank);
  SEMX_REQUIRE(a->ldz >= a->rank, SEMX_ERR_SHAPE, "step_proj: row stride %lld < rank %d", (long long)a->ldz,
               a->rank);
  SEMX_REQUIRE(semx::cdiv(a->rows, kRowsPerCta) <= 0x7fffffff && semx::cdiv(a->C, kTileC) <= 65535, SEMX_ERR_SHAPE,
               "step_proj: grid too large");
  if (a->rows > 0) {
    SEMX_REQUIRE(a->z_nu && a->z_th && a->W_nu && a->b_nu && a->W_th && a->b_th, SEMX_ERR_NULL,
                 "step_proj: z / W / b is NULL");
    if (!bwd) SEMX_REQUIRE(a->delta_nu && a->delta_th, SEMX_ERR_NULL, "step_proj: delta_nu / delta_th is NULL");
    if (bwd) {
      SEMX_REQUIRE(a->dz_nu && a->dz_th && a->dW_nu && a->db_nu && a->dW_th && a->db_th, SEMX_ERR_NULL,
                   "step_proj bwd: dz / dW / db is NULL");
      SEMX_REQUIRE(a->workspace != nullptr, SEMX_ERR_WORKSPACE, "step_proj bwd: workspace is NULL");
    }
  }
  if ((a->C % 2) == 0 && a->rows > 0) {
    const bool al = bwd ? ((!a->d_delta_nu || semx::aligned(a->d_delta_nu, 8)) &&
                           (!a->d_delta_th || semx::aligned(a->d_delta_th, 8)))
                        : (semx::aligned(a->delta_nu, 8) && semx::aligned(a->delta_th, 8));
    SEMX_REQUIRE(al, SEMX_ERR_ALIGN, "step_proj: (rows, C) tensors must be 8-byte aligned when C is even");
  }
  return SEMX_OK;
}

PParams proj_params(const SemxStepProjArgs* a) {
  PParams p = {};
  p.rows = a->rows; p.C = a->C; p.ldz = a->ldz;
  p.ntiles = (int)semx::cdiv(a->C, kTileC);
  p.scale = a->scale;
  p.zn = a->z_nu; p.zt = a->z_th;
  p.Wn = a->W_nu; p.bn = a->b_nu; p.Wt = a->W_th; p.bt = a->b_th;
  p.dnu = a->delta_nu; p.dth = a->delta_th;
  p.gdnu = a->d_delta_nu; p.gdth = a->d_delta_th;
  p.dzn = a->dz_nu; p.dzt = a->dz_th;
  return p;
}

size_t part_floats(const SemxStepProjArgs* a) {
  return (size_t)semx::cdiv(a->rows, kRowsPerCta) * (size_t)(2 * (a->C * a->rank + a->C));
}
size_t dzpart_floats(const SemxStepProjArgs* a) {
  const int64_t nt = semx::cdiv(a->C, kTileC);
  return nt > 1 ? (size_t)nt * (size_t)a->rows * (size_t)(2 * a->rank) : 0;
}

}  // namespace

extern "C" {

size_t semx_step_proj_args_size(void) { return sizeof(SemxStepProjArgs); }

size_t semx_step_proj_workspace_bytes(const SemxStepProjArgs* a) {
  if (a == nullptr || a->rows < 0 || a->C < 1 || a->rank < 1 || a->rank > kMaxRank) return 0;
  const int64_t nrb = semx::cdiv(a->rows, kRowsPerCta);
  const int64_t K = 2 * (a->C * a->rank + a->C);
  return (part_floats(a) + semx::colsum_group_floats(nrb, K) + dzpart_floats(a)) * sizeof(float);
}

int semx_step_proj_fwd(const SemxStepProjArgs* a, semx_stream_t stream) {
  SEMX_CHECK_ARGS(a, SemxStepProjArgs);
  int rc = proj_validate(a, false);
  if (rc != SEMX_OK) return rc;
  if (a->rows == 0) return SEMX_OK;
  rc = semx::bind_device({a->delta_nu});
  if (rc != SEMX_OK) return rc;
  const PParams p = proj_params(a);
  cudaStream_t st = semx::as_stream(stream);
  return a->bf16 ? dispatch<true>(false, a->rank, p, st) : dispatch<false>(false, a->rank, p, st);
}

int semx_step_proj_bwd(const SemxStepProjArgs* a, semx_stream_t stream) {
  SEMX_CHECK_ARGS(a, SemxStepProjArgs);
  int rc = proj_validate(a, true);
  if (rc != SEMX_OK) return rc;
  rc = semx::bind_device({a->dW_nu});
  if (rc != SEMX_OK) return rc;
  cudaStream_t st = semx::as_stream(stream);
  const int64_t R = a->rank, C = a->C;
  if (a->rows == 0) {  // no rows: every parameter gradient is zero
    cudaMemsetAsync(a->dW_nu, 0, (size_t)(C * R) * sizeof(float), st);
    cudaMemsetAsync(a->db_nu, 0, (size_t)C * sizeof(float), st);
    cudaMemsetAsync(a->dW_th, 0, (size_t)(C * R) * sizeof(float), st);
    cudaMemsetAsync(a->db_th, 0, (size_t)C * sizeof(float), st);
    return semx::check_launch("step_proj bwd: zero gradients");
  }
  PParams p = proj_params(a);
  float* ws = reinterpret_cast<float*>(a->workspace);
  const int64_t nrb = semx::cdiv(a->rows, kRowsPerCta);
  const int64_t K = 2 * (C * R + C);
  p.part = ws;
  float* groups = ws + part_floats(a);
  p.dzpart = groups + semx::colsum_group_floats(nrb, K);
  rc = a->bf16 ? dispatch<true>(true, a->rank, p, st) : dispatch<false>(true, a->rank, p, st);
  if (rc != SEMX_OK) return rc;
  semx::Segments seg = {};
  seg.n = 4;
  seg.out[0] = a->dW_nu;
  seg.len[0] = C * R;
  seg.out[1] = a->db_nu;
  seg.len[1] = C;
  seg.out[2] = a->dW_th;
  seg.len[2] = C * R;
  seg.out[3] = a->db_th;
  seg.len[3] = C;
  return semx::colsum(ws, nrb, K, groups, seg, st);
}

}  // extern "C"
