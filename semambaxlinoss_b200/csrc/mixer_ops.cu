// Elementwise surround of the Mamba-style mixer, channels-last, for sm_100a.
//
// Reference behaviour (paths relative to the reference project):
//   models/mixer.py:82-99  u, z = in_proj(x).chunk(2); u = silu(conv1d(pad(u^T))^T);
//                          y = ssm(u) * silu(z)
//
// conv_silu: depthwise convolution of width K along the sequence with bias, then SiLU,
//   v[s,t,c] = silu(b[c] + sum_k w[c,k] u[s, t - left + k, c])   (u = 0 outside [0, L))
//   read straight from the in_proj output (row stride 2C, u = columns [0, C)), so the
//   transposes, the padding copy and the chunk copy of the reference formulation never
//   materialise. One thread owns 4 channels of one sequence (of a quarter of it for long
//   sequences, the `_split` kernels) and slides a K-step window along t, so every input
//   is read once (plus a K - 1 step halo per quarter); consecutive threads own
//   consecutive channels. The backward slides the same window, recomputing the
//   pre-activation, and writes du into columns [0, C) of dxz; dw and db are summed per
//   thread over its steps (over the quarters in shared memory), written per sequence and
//   reduced over sequences by the fixed-order column sum.
// gate_silu: o = y * silu(z) with z = columns [C, 2C) of the in_proj output; its backward
//   writes dz into columns [C, 2C) of the same dxz buffer.
#include <cuda_bf16.h>

#include "semx_common.cuh"
#include "semx_reduce.cuh"

namespace {

constexpr int kT = 128;
constexpr int kCV = 4;  // channels per thread

// Loads / stores 4 consecutive channels at element i; `vec` selects one vector access
// (all 4 valid and aligned), otherwise only the first cn channels are touched (loads give
// 0 for the rest).
template <bool BF16>
__device__ __forceinline__ void ld4(const void* base, int64_t i, bool vec, float (&v)[kCV], int cn = kCV) {
  if (BF16) {
    const __nv_bfloat16* p = reinterpret_cast<const __nv_bfloat16*>(base) + i;
    if (vec) {
      const uint2 r = *reinterpret_cast<const uint2*>(p);
      const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&r.x);
      const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&r.y);
      v[0] = __low2float(a); v[1] = __high2float(a); v[2] = __low2float(b); v[3] = __high2float(b);
    } else {
#pragma unroll
      for (int j = 0; j < kCV; ++j) v[j] = j < cn ? __bfloat162float(p[j]) : 0.f;
    }
  } else {
    const float* p = reinterpret_cast<const float*>(base) + i;
    if (vec) {
      const float4 r = *reinterpret_cast<const float4*>(p);
      v[0] = r.x; v[1] = r.y; v[2] = r.z; v[3] = r.w;
    } else {
#pragma unroll
      for (int j = 0; j < kCV; ++j) v[j] = j < cn ? p[j] : 0.f;
    }
  }
}

template <bool BF16>
__device__ __forceinline__ void st4(void* base, int64_t i, bool vec, const float (&v)[kCV], int cn = kCV) {
  if (BF16) {
    __nv_bfloat16* p = reinterpret_cast<__nv_bfloat16*>(base) + i;
    if (vec) {
      uint2 r;
      *reinterpret_cast<__nv_bfloat162*>(&r.x) = __floats2bfloat162_rn(v[0], v[1]);
      *reinterpret_cast<__nv_bfloat162*>(&r.y) = __floats2bfloat162_rn(v[2], v[3]);
      *reinterpret_cast<uint2*>(p) = r;
    } else {
#pragma unroll
      for (int j = 0; j < kCV; ++j)
        if (j < cn) p[j] = __float2bfloat16(v[j]);
    }
  } else {
    float* p = reinterpret_cast<float*>(base) + i;
    if (vec) {
      *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
#pragma unroll
      for (int j = 0; j < kCV; ++j)
        if (j < cn) p[j] = v[j];
    }
  }
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.f / (1.f + __expf(-x)); }

struct ConvParams {
  semx::RowMap rm;      // token row of (sequence, step)
  int64_t S, L, C, ld;  // ld = row stride of xz / dxz in elements (2C)
  int left;             // taps before t
  const void* xz;       // u = columns [0, C)
  const float* w;       // (C, K)
  const float* b;       // (C)
  float* v;             // (S, L, C) fp32
  const float* dv;      // (S, L, C) fp32
  void* dxz;            // du -> columns [0, C)
  float* part;          // (S, C*(K+1)) partial dw | db rows
};

// Thread (s, channel group): slides over t with the window of the K inputs u[t-left .. t-left+K-1].
template <bool BF16, int K>
__global__ void __launch_bounds__(kT) conv_silu_fwd_kernel(const ConvParams p) {
  const int64_t groups = (p.C + kCV - 1) / kCV;
  const int64_t gid = (int64_t)blockIdx.x * kT + threadIdx.x;
  if (gid >= p.S * groups) return;
  const int64_t s = gid / groups;
  const int64_t sb = p.rm.seq(s);  // token row of step t: sb + p.rm.step(t)
  const int c0 = (int)(gid % groups) * kCV;
  const int cn = (int)min((int64_t)kCV, p.C - c0);
  const bool full = cn == kCV;
  const bool vin = full && ((p.ld % kCV) == 0) &&
                   ((reinterpret_cast<uintptr_t>(p.xz) & (BF16 ? 7 : 15)) == 0);
  const bool vout = full && ((p.C % kCV) == 0) && ((reinterpret_cast<uintptr_t>(p.v) & 15) == 0);
  float w[K][kCV], bias[kCV];
#pragma unroll
  for (int j = 0; j < kCV; ++j) {
    const int c = min(c0 + j, (int)p.C - 1);
#pragma unroll
    for (int k = 0; k < K; ++k) w[k][j] = p.w[(int64_t)c * K + k];
    bias[j] = p.b ? p.b[c] : 0.f;
  }
  const int L = (int)p.L, left = p.left;
  float win[K][kCV];  // win[k] = u[t - left + k]
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int tt = k - left;  // for t = 0
#pragma unroll
    for (int j = 0; j < kCV; ++j) win[k][j] = 0.f;
    if (k < K - 1 && tt >= 0 && tt < L) {
      float tmp[kCV];
      ld4<BF16>(p.xz, (sb + p.rm.step(tt)) * p.ld + c0, vin, tmp, cn);
#pragma unroll
      for (int j = 0; j < kCV; ++j) win[k][j] = tmp[j];
    }
  }
  for (int t = 0; t < L; ++t) {
    // Shift in u[t - left + K - 1].
    {
      const int tt = t - left + K - 1;
#pragma unroll
      for (int j = 0; j < kCV; ++j) win[K - 1][j] = 0.f;
      if (tt >= 0 && tt < L) {
        float tmp[kCV];
        ld4<BF16>(p.xz, (sb + p.rm.step(tt)) * p.ld + c0, vin, tmp, cn);
#pragma unroll
        for (int j = 0; j < kCV; ++j) win[K - 1][j] = tmp[j];
      }
    }
    float out[kCV];
#pragma unroll
    for (int j = 0; j < kCV; ++j) {
      float a = bias[j];
#pragma unroll
      for (int k = 0; k < K; ++k) a = fmaf(w[k][j], win[k][j], a);
      out[j] = a * sigmoidf_(a);
    }
    st4<false>(p.v, (sb + p.rm.step(t)) * p.C + c0, vout, out, cn);
#pragma unroll
    for (int k = 0; k + 1 < K; ++k)
#pragma unroll
      for (int j = 0; j < kCV; ++j) win[k][j] = win[k + 1][j];
  }
}

// Backward: step jt computes dpre[jt] from the u window of jt (pre-activation recomputed)
// and, once dpre[t + left] is known, emits du[t] = sum_k w[k] dpre[t + left - k] (a delay
// of `left` steps).
template <bool BF16, int K>
__global__ void __launch_bounds__(kT) conv_silu_bwd_kernel(const ConvParams p) {
  const int64_t groups = (p.C + kCV - 1) / kCV;
  const int64_t gid = (int64_t)blockIdx.x * kT + threadIdx.x;
  if (gid >= p.S * groups) return;
  const int64_t s = gid / groups;
  const int64_t sb = p.rm.seq(s);  // token row of step t: sb + p.rm.step(t)
  const int c0 = (int)(gid % groups) * kCV;
  const int cn = (int)min((int64_t)kCV, p.C - c0);
  const bool full = cn == kCV;
  const bool vin = full && ((p.ld % kCV) == 0) &&
                   ((reinterpret_cast<uintptr_t>(p.xz) & (BF16 ? 7 : 15)) == 0) &&
                   ((reinterpret_cast<uintptr_t>(p.dxz) & (BF16 ? 7 : 15)) == 0);
  const bool vdv = full && ((p.C % kCV) == 0) && ((reinterpret_cast<uintptr_t>(p.dv) & 15) == 0);
  float w[K][kCV], bias[kCV], dw[K][kCV], db[kCV];
#pragma unroll
  for (int j = 0; j < kCV; ++j) {
    const int c = min(c0 + j, (int)p.C - 1);
#pragma unroll
    for (int k = 0; k < K; ++k) {
      w[k][j] = p.w[(int64_t)c * K + k];
      dw[k][j] = 0.f;
    }
    bias[j] = p.b ? p.b[c] : 0.f;
    db[j] = 0.f;
  }
  const int L = (int)p.L, left = p.left;
  float win[K][kCV];  // u[j - left + k]
  float dp[K][kCV];   // dp[k] = dpre[j - (K - 1) + k]
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int tt = k - left;
#pragma unroll
    for (int j = 0; j < kCV; ++j) {
      win[k][j] = 0.f;
      dp[k][j] = 0.f;
    }
    if (k < K - 1 && tt >= 0 && tt < L) {
      float tmp[kCV];
      ld4<BF16>(p.xz, (sb + p.rm.step(tt)) * p.ld + c0, vin, tmp, cn);
#pragma unroll
      for (int j = 0; j < kCV; ++j) win[k][j] = tmp[j];
    }
  }
  // The step's two loads (u[jt - left + K - 1], dv[jt]) are issued one step ahead.
  float nu[kCV], ng[kCV];
  auto fetch = [&](int jt) {
    const int tt = jt - left + K - 1;
#pragma unroll
    for (int j = 0; j < kCV; ++j) nu[j] = ng[j] = 0.f;
    if (jt < L && tt >= 0 && tt < L) ld4<BF16>(p.xz, (sb + p.rm.step(tt)) * p.ld + c0, vin, nu, cn);
    if (jt < L) ld4<false>(p.dv, (sb + p.rm.step(jt)) * p.C + c0, vdv, ng, cn);
  };
  fetch(0);
  for (int jt = 0; jt < L + left; ++jt) {
    float g[kCV];
#pragma unroll
    for (int j = 0; j < kCV; ++j) {
      win[K - 1][j] = nu[j];
      g[j] = ng[j];
    }
    if (jt + 1 < L + left) fetch(jt + 1);
    // dpre[jt] (zero beyond the sequence end).
#pragma unroll
    for (int k = 0; k + 1 < K; ++k)
#pragma unroll
      for (int j = 0; j < kCV; ++j) dp[k][j] = dp[k + 1][j];
    if (jt < L) {
#pragma unroll
      for (int j = 0; j < kCV; ++j) {
        float a = bias[j];
#pragma unroll
        for (int k = 0; k < K; ++k) a = fmaf(w[k][j], win[k][j], a);
        const float sg = sigmoidf_(a);
        const float d = g[j] * sg * (1.f + a * (1.f - sg));
        dp[K - 1][j] = d;
        db[j] += d;
#pragma unroll
        for (int k = 0; k < K; ++k) dw[k][j] = fmaf(d, win[k][j], dw[k][j]);
      }
#pragma unroll
      for (int k = 0; k + 1 < K; ++k)
#pragma unroll
        for (int j = 0; j < kCV; ++j) win[k][j] = win[k + 1][j];
    } else {
#pragma unroll
      for (int j = 0; j < kCV; ++j) dp[K - 1][j] = 0.f;
    }
    // du[t] with t = jt - left: sum_k w[k] dpre[t + left - k] = sum_k w[k] dp[K - 1 - k].
    const int t = jt - left;
    if (t >= 0) {
      float du[kCV];
#pragma unroll
      for (int j = 0; j < kCV; ++j) {
        float a = 0.f;
#pragma unroll
        for (int k = 0; k < K; ++k) a = fmaf(w[k][j], dp[K - 1 - k][j], a);
        du[j] = a;
      }
      st4<BF16>(p.dxz, (sb + p.rm.step(t)) * p.ld + c0, vin, du, cn);
    }
  }
  // Per-sequence partials: [dw (C, K) | db (C)].
  float* row = p.part + s * (p.C * (K + 1));
#pragma unroll
  for (int j = 0; j < kCV; ++j) {
    if (c0 + j < p.C) {
#pragma unroll
      for (int k = 0; k < K; ++k) row[(int64_t)(c0 + j) * K + k] = dw[k][j];
      row[p.C * K + c0 + j] = db[j];
    }
  }
}

// Threads are (sequence s, channel group of 4, time block tq): a CTA holds TS time blocks
// of kT / TS consecutive channel groups (thread tid: tq = tid / (kT / TS), group slot
// tid % (kT / TS)), so a warp still reads 32 consecutive channel groups of one step. Time
// block tq covers steps [tq TB, (tq + 1) TB), TB = ceil(L / TS), and slides a K-step
// window over them (plus the K - 1 halo steps its window or its du needs), with a 4-way
// unrolled step loop, so the chain of dependent steps per thread is a quarter of the
// sequence. Used for long sequences (L >= kSplitL; the whole-sequence kernels above
// serve the rest): measured at C = 256 channels, bf16, 1600 x 321, forward 0.38 -> 0.31
// ms and backward 0.93 -> 0.79 ms; at 5136 x 100 the whole-sequence kernels were faster
// (backward 0.63 against 0.78 ms), since that shape already has many sequences in flight.
constexpr int kSplitL = 256;

struct Slot {
  int64_t s;
  int c0, cn, tq, t0, t1;
  bool ok;
};
template <int TS>
__device__ __forceinline__ Slot slot_of(const ConvParams& p) {
  constexpr int GB = kT / TS;
  Slot q;
  const int64_t groups = (p.C + kCV - 1) / kCV;
  const int64_t gg = (int64_t)blockIdx.x * GB + threadIdx.x % GB;
  q.tq = threadIdx.x / GB;
  q.ok = gg < p.S * groups;
  q.s = q.ok ? gg / groups : 0;
  q.c0 = q.ok ? (int)(gg % groups) * kCV : 0;
  q.cn = (int)min((int64_t)kCV, p.C - q.c0);
  const int L = (int)p.L, tb = (L + TS - 1) / TS;
  q.t0 = min(L, q.tq * tb);
  q.t1 = min(L, q.t0 + tb);
  return q;
}

template <bool BF16, int K, int TS>
__global__ void __launch_bounds__(kT) conv_silu_fwd_split_kernel(const ConvParams p) {
  const Slot q = slot_of<TS>(p);
  if (!q.ok || q.t0 >= q.t1) return;
  const int64_t s = q.s;
  const int64_t sb = p.rm.seq(s);  // token row of step t: sb + p.rm.step(t)
  const int c0 = q.c0, cn = q.cn;
  const bool full = cn == kCV;
  const bool vin = full && ((p.ld % kCV) == 0) &&
                   ((reinterpret_cast<uintptr_t>(p.xz) & (BF16 ? 7 : 15)) == 0);
  const bool vout = full && ((p.C % kCV) == 0) && ((reinterpret_cast<uintptr_t>(p.v) & 15) == 0);
  float w[K][kCV], bias[kCV];
#pragma unroll
  for (int j = 0; j < kCV; ++j) {
    const int c = min(c0 + j, (int)p.C - 1);
#pragma unroll
    for (int k = 0; k < K; ++k) w[k][j] = p.w[(int64_t)c * K + k];
    bias[j] = p.b ? p.b[c] : 0.f;
  }
  const int L = (int)p.L, left = p.left;
  float win[K][kCV];  // win[k] = u[t - left + k]
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int tt = q.t0 + k - left;
#pragma unroll
    for (int j = 0; j < kCV; ++j) win[k][j] = 0.f;
    if (k < K - 1 && tt >= 0 && tt < L) {
      float tmp[kCV];
      ld4<BF16>(p.xz, (sb + p.rm.step(tt)) * p.ld + c0, vin, tmp, cn);
#pragma unroll
      for (int j = 0; j < kCV; ++j) win[k][j] = tmp[j];
    }
  }
  // Element offsets of the next input row (step t - left + K - 1) and output row (step t),
  // advanced by one step stride per step instead of recomputed from the row map.
  const int64_t din = p.rm.step(1) * p.ld, dout = p.rm.step(1) * p.C;
  int64_t oin = (sb + p.rm.step(q.t0 - left + K - 1)) * p.ld + c0;
  int64_t oout = (sb + p.rm.step(q.t0)) * p.C + c0;
  auto step = [&](int t) {
    // Shift in u[t - left + K - 1].
    {
      const int tt = t - left + K - 1;
#pragma unroll
      for (int j = 0; j < kCV; ++j) win[K - 1][j] = 0.f;
      if (tt >= 0 && tt < L) {
        float tmp[kCV];
        ld4<BF16>(p.xz, oin, vin, tmp, cn);
#pragma unroll
        for (int j = 0; j < kCV; ++j) win[K - 1][j] = tmp[j];
      }
      oin += din;
    }
    float out[kCV];
#pragma unroll
    for (int j = 0; j < kCV; ++j) {
      float a = bias[j];
#pragma unroll
      for (int k = 0; k < K; ++k) a = fmaf(w[k][j], win[k][j], a);
      out[j] = a * sigmoidf_(a);
    }
    st4<false>(p.v, oout, vout, out, cn);
    oout += dout;
#pragma unroll
    for (int k = 0; k + 1 < K; ++k)
#pragma unroll
      for (int j = 0; j < kCV; ++j) win[k][j] = win[k + 1][j];
  };
  if (TS > 1) {
#pragma unroll 4
    for (int t = q.t0; t < q.t1; ++t) step(t);
  } else {
    for (int t = q.t0; t < q.t1; ++t) step(t);
  }
}

// Backward of time block [t0, t1): step jt computes dpre[jt] (zero outside [0, L)) from the
// u window of jt (pre-activation recomputed) and, once dpre[t + left] is known, emits
// du[t] = sum_k w[k] dpre[t + left - k] (a delay of `left` steps). du[t0 .. t1) needs dpre
// on [t0 + left - K + 1, t1 + left); dw and db take only the block's own steps [t0, t1).
// The TS time blocks of a channel group are summed in shared memory in block order.
template <bool BF16, int K, int TS>
__global__ void __launch_bounds__(kT) conv_silu_bwd_split_kernel(const ConvParams p) {
  constexpr int GB = kT / TS;
  __shared__ float red[TS > 1 ? kT : 1][kCV * (K + 1)];
  const Slot q = slot_of<TS>(p);
  const int64_t s = q.s;
  const int64_t sb = p.rm.seq(s);  // token row of step t: sb + p.rm.step(t)
  const int c0 = q.c0, cn = q.cn;
  const bool full = cn == kCV;
  const bool vin = full && ((p.ld % kCV) == 0) &&
                   ((reinterpret_cast<uintptr_t>(p.xz) & (BF16 ? 7 : 15)) == 0) &&
                   ((reinterpret_cast<uintptr_t>(p.dxz) & (BF16 ? 7 : 15)) == 0);
  const bool vdv = full && ((p.C % kCV) == 0) && ((reinterpret_cast<uintptr_t>(p.dv) & 15) == 0);
  float w[K][kCV], bias[kCV], dw[K][kCV], db[kCV];
#pragma unroll
  for (int j = 0; j < kCV; ++j) {
    const int c = min(c0 + j, (int)p.C - 1);
#pragma unroll
    for (int k = 0; k < K; ++k) {
      w[k][j] = p.w[(int64_t)c * K + k];
      dw[k][j] = 0.f;
    }
    bias[j] = p.b ? p.b[c] : 0.f;
    db[j] = 0.f;
  }
  const int L = (int)p.L, left = p.left;
  if (q.ok && q.t0 < q.t1) {
    const int ja = q.t0 + left - (K - 1), jb = q.t1 + left;  // jt in [ja, jb)
    float win[K][kCV];  // u[jt - left + k]
    float dp[K][kCV];   // dp[k] = dpre[jt - (K - 1) + k]
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int tt = ja - left + k;
#pragma unroll
      for (int j = 0; j < kCV; ++j) {
        win[k][j] = 0.f;
        dp[k][j] = 0.f;
      }
      if (k < K - 1 && tt >= 0 && tt < L) {
        float tmp[kCV];
        ld4<BF16>(p.xz, (sb + p.rm.step(tt)) * p.ld + c0, vin, tmp, cn);
#pragma unroll
        for (int j = 0; j < kCV; ++j) win[k][j] = tmp[j];
      }
    }
    // The step's two loads (u[jt - left + K - 1], dv[jt]) are issued one step ahead, so
    // each thread keeps a step of reads in flight while it computes.
    float nu[kCV], ng[kCV];
    auto fetch = [&](int jt) {
      const int tt = jt - left + K - 1;
#pragma unroll
      for (int j = 0; j < kCV; ++j) nu[j] = ng[j] = 0.f;
      if (jt < L && tt >= 0 && tt < L) ld4<BF16>(p.xz, (sb + p.rm.step(tt)) * p.ld + c0, vin, nu, cn);
      if (jt >= 0 && jt < L) ld4<false>(p.dv, (sb + p.rm.step(jt)) * p.C + c0, vdv, ng, cn);
    };
    fetch(ja);
    auto step = [&](int jt) {
      float g[kCV];
#pragma unroll
      for (int j = 0; j < kCV; ++j) {
        win[K - 1][j] = nu[j];
        g[j] = ng[j];
      }
      if (jt + 1 < jb) fetch(jt + 1);
#pragma unroll
      for (int k = 0; k + 1 < K; ++k)
#pragma unroll
        for (int j = 0; j < kCV; ++j) dp[k][j] = dp[k + 1][j];
#pragma unroll
      for (int j = 0; j < kCV; ++j) dp[K - 1][j] = 0.f;
      if (jt < L) {
        if (jt >= 0) {
          const bool own = jt >= q.t0 && jt < q.t1;
#pragma unroll
          for (int j = 0; j < kCV; ++j) {
            float a = bias[j];
#pragma unroll
            for (int k = 0; k < K; ++k) a = fmaf(w[k][j], win[k][j], a);
            const float sg = sigmoidf_(a);
            const float d = g[j] * sg * (1.f + a * (1.f - sg));
            dp[K - 1][j] = d;
            if (own) {
              db[j] += d;
#pragma unroll
              for (int k = 0; k < K; ++k) dw[k][j] = fmaf(d, win[k][j], dw[k][j]);
            }
          }
        }
#pragma unroll
        for (int k = 0; k + 1 < K; ++k)
#pragma unroll
          for (int j = 0; j < kCV; ++j) win[k][j] = win[k + 1][j];
      }
      // du[t] with t = jt - left: sum_k w[k] dpre[t + left - k] = sum_k w[k] dp[K - 1 - k].
      const int t = jt - left;
      if (t >= q.t0) {
        float du[kCV];
#pragma unroll
        for (int j = 0; j < kCV; ++j) {
          float a = 0.f;
#pragma unroll
          for (int k = 0; k < K; ++k) a = fmaf(w[k][j], dp[K - 1 - k][j], a);
          du[j] = a;
        }
        st4<BF16>(p.dxz, (sb + p.rm.step(t)) * p.ld + c0, vin, du, cn);
      }
    };
    // TS > 1: unrolled by 4; TS = 1: the compiler's own unrolling (measured faster there).
    if (TS > 1) {
#pragma unroll 4
      for (int jt = ja; jt < jb; ++jt) step(jt);
    } else {
      for (int jt = ja; jt < jb; ++jt) step(jt);
    }
  }
  // dw | db of this time block (summed over the TS blocks in order) into the per-sequence row.
  if (TS > 1) {
#pragma unroll
    for (int j = 0; j < kCV; ++j) {
#pragma unroll
      for (int k = 0; k < K; ++k) red[threadIdx.x][j * (K + 1) + k] = dw[k][j];
      red[threadIdx.x][j * (K + 1) + K] = db[j];
    }
    __syncthreads();
  }
  if (q.tq != 0 || !q.ok) return;
  float* row = p.part + s * (p.C * (K + 1));
  const int gl = threadIdx.x % GB;
#pragma unroll
  for (int j = 0; j < kCV; ++j) {
    if (c0 + j < p.C) {
#pragma unroll
      for (int k = 0; k <= K; ++k) {
        float acc = 0.f;
        if (TS > 1) {
#pragma unroll
          for (int b = 0; b < TS; ++b) acc += red[b * GB + gl][j * (K + 1) + k];
        } else {
          acc = k < K ? dw[k][j] : db[j];
        }
        if (k < K) row[(int64_t)(c0 + j) * K + k] = acc;
        else row[p.C * K + c0 + j] = acc;
      }
    }
  }
}

struct GateParams {
  int64_t n, C, ld;  // n = S*L rows
  const float* y;    // (n, C) fp32
  const void* xz;    // z = columns [C, 2C)
  void* o;           // (n, C), dtype of xz
  const void* dout;  // (n, C), dtype of xz
  float* dy;         // (n, C) fp32
  void* dxz;         // dz -> columns [C, 2C)
};

template <bool BF16>
__global__ void __launch_bounds__(256) gate_silu_fwd_kernel(const GateParams p) {
  const int64_t groups = (p.C + kCV - 1) / kCV;
  const int64_t gid = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (gid >= p.n * groups) return;
  const int64_t r = gid / groups;
  const int c0 = (int)(gid % groups) * kCV;
  const bool full = c0 + kCV <= p.C && (p.C % kCV) == 0;
  const bool vz = full && (p.ld % kCV) == 0 && ((reinterpret_cast<uintptr_t>(p.xz) & (BF16 ? 7 : 15)) == 0);
  const bool vy = full && ((reinterpret_cast<uintptr_t>(p.y) & 15) == 0) &&
                  ((reinterpret_cast<uintptr_t>(p.o) & (BF16 ? 7 : 15)) == 0);
  float y[kCV], z[kCV], o[kCV];
  if (full) {
    ld4<false>(p.y, r * p.C + c0, vy, y);
    ld4<BF16>(p.xz, r * p.ld + p.C + c0, vz, z);
#pragma unroll
    for (int j = 0; j < kCV; ++j) o[j] = y[j] * (z[j] * sigmoidf_(z[j]));
    st4<BF16>(p.o, r * p.C + c0, vy, o);
  } else {
    for (int j = 0; j < kCV && c0 + j < p.C; ++j) {
      const float yy = p.y[r * p.C + c0 + j];
      float zz;
      if (BF16) zz = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.xz)[r * p.ld + p.C + c0 + j]);
      else zz = reinterpret_cast<const float*>(p.xz)[r * p.ld + p.C + c0 + j];
      const float v = yy * (zz * sigmoidf_(zz));
      if (BF16) reinterpret_cast<__nv_bfloat16*>(p.o)[r * p.C + c0 + j] = __float2bfloat16(v);
      else reinterpret_cast<float*>(p.o)[r * p.C + c0 + j] = v;
    }
  }
}

template <bool BF16>
__global__ void __launch_bounds__(256) gate_silu_bwd_kernel(const GateParams p) {
  const int64_t groups = (p.C + kCV - 1) / kCV;
  const int64_t gid = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (gid >= p.n * groups) return;
  const int64_t r = gid / groups;
  const int c0 = (int)(gid % groups) * kCV;
  const int cn = (int)min((int64_t)kCV, p.C - c0);
  // One vector access per operand when the 4 channels are full and every row is aligned.
  constexpr uintptr_t am = BF16 ? 7 : 15;
  const bool vec = cn == kCV && (p.C % kCV) == 0 && (p.ld % kCV) == 0 &&
                   ((reinterpret_cast<uintptr_t>(p.xz) & am) == 0) &&
                   ((reinterpret_cast<uintptr_t>(p.dxz) & am) == 0) &&
                   ((reinterpret_cast<uintptr_t>(p.dout) & am) == 0) &&
                   ((reinterpret_cast<uintptr_t>(p.y) & 15) == 0) && ((reinterpret_cast<uintptr_t>(p.dy) & 15) == 0);
  float z[kCV], go[kCV], y[kCV], dy[kCV], dz[kCV];
  ld4<BF16>(p.xz, r * p.ld + p.C + c0, vec, z, cn);
  ld4<BF16>(p.dout, r * p.C + c0, vec, go, cn);
  ld4<false>(p.y, r * p.C + c0, vec, y, cn);
#pragma unroll
  for (int j = 0; j < kCV; ++j) {
    const float sg = sigmoidf_(z[j]);
    dy[j] = go[j] * z[j] * sg;
    dz[j] = go[j] * y[j] * sg * (1.f + z[j] * (1.f - sg));
  }
  st4<false>(p.dy, r * p.C + c0, vec, dy, cn);
  st4<BF16>(p.dxz, r * p.ld + p.C + c0, vec, dz, cn);
}

template <bool BF16>
int launch_conv(bool bwd, int K, const ConvParams& p, cudaStream_t st) {
  constexpr int TS = 4;
  const bool split = p.L >= kSplitL;
  const int64_t groups = semx::cdiv(p.C, kCV);
  const unsigned grid = (unsigned)semx::cdiv(p.S * groups, split ? kT / TS : kT);
  switch (K) {
#define SEMX_K(KV)                                                                         \
  case KV:                                                                                 \
    if (split) {                                                                           \
      if (bwd) conv_silu_bwd_split_kernel<BF16, KV, TS><<<grid, kT, 0, st>>>(p);            \
      else conv_silu_fwd_split_kernel<BF16, KV, TS><<<grid, kT, 0, st>>>(p);                \
    } else {                                                                               \
      if (bwd) conv_silu_bwd_kernel<BF16, KV><<<grid, kT, 0, st>>>(p);                     \
      else conv_silu_fwd_kernel<BF16, KV><<<grid, kT, 0, st>>>(p);                         \
    }                                                                                      \
    return semx::check_launch(bwd ? "conv_silu_bwd_kernel" : "conv_silu_fwd_kernel");
    SEMX_K(1)
    SEMX_K(2)
    SEMX_K(3)
    SEMX_K(4)
    SEMX_K(5)
    SEMX_K(6)
    SEMX_K(7)
    SEMX_K(8)
#undef SEMX_K
  }
  return semx::fail(SEMX_ERR_UNSUPPORTED, "conv_silu: kernel width %d (1..8)", K);
}

int conv_validate(const SemxConvSiluArgs* a, bool bwd) {
  SEMX_REQUIRE(a->S >= 0 && a->L >= 0 && a->C >= 0, SEMX_ERR_SHAPE, "conv_silu: negative size");
  SEMX_REQUIRE(a->K >= 1 && a->K <= 8, SEMX_ERR_UNSUPPORTED, "conv_silu: kernel width %d (1..8)", a->K);
  SEMX_REQUIRE(a->left >= 0 && a->left < a->K, SEMX_ERR_SHAPE, "conv_silu: left=%d outside [0, K)", a->left);
  SEMX_REQUIRE(a->ld >= a->C, SEMX_ERR_SHAPE, "conv_silu: row stride %lld < C", (long long)a->ld);
  {
    semx::RowMap rm;
    const int rc = semx::make_rowmap(a->S, a->L, a->reverse, a->seq_group, a->group_stride, a->seq_stride,
                                     a->step_stride, &rm, "conv_silu");
    if (rc != SEMX_OK) return rc;
  }
  if (a->S * a->L * a->C > 0) {
    SEMX_REQUIRE(a->xz && a->w, SEMX_ERR_NULL, "conv_silu: xz / w is NULL");
    if (!bwd) SEMX_REQUIRE(a->v, SEMX_ERR_NULL, "conv_silu: v is NULL");
    if (bwd) SEMX_REQUIRE(a->dv && a->dxz && a->workspace, SEMX_ERR_NULL, "conv_silu bwd: dv / dxz / workspace is NULL");
  }
  return SEMX_OK;
}

ConvParams conv_params(const SemxConvSiluArgs* a) {
  ConvParams p = {};
  semx::make_rowmap(a->S, a->L, a->reverse, a->seq_group, a->group_stride, a->seq_stride, a->step_stride, &p.rm,
                    "conv_silu");
  p.S = a->S; p.L = a->L; p.C = a->C; p.ld = a->ld; p.left = a->left;
  p.xz = a->xz; p.w = a->w; p.b = a->b; p.v = a->v; p.dv = a->dv; p.dxz = a->dxz;
  return p;
}

}  // namespace

extern "C" {

size_t semx_conv_silu_args_size(void) { return sizeof(SemxConvSiluArgs); }
size_t semx_gate_silu_args_size(void) { return sizeof(SemxGateSiluArgs); }

size_t semx_conv_silu_workspace_bytes(const SemxConvSiluArgs* a) {
  if (a == nullptr || a->S < 0 || a->C < 0 || a->K < 1) return 0;
  const int64_t Kc = a->C * (a->K + 1);
  return ((size_t)a->S * Kc + semx::colsum_group_floats(a->S, Kc)) * sizeof(float);
}

int semx_conv_silu_fwd(const SemxConvSiluArgs* a, semx_stream_t stream) {
  SEMX_CHECK_ARGS(a, SemxConvSiluArgs);
  int rc = conv_validate(a, false);
  if (rc != SEMX_OK) return rc;
  if (a->S * a->L * a->C == 0) return SEMX_OK;
  rc = semx::bind_device({a->v});
  if (rc != SEMX_OK) return rc;
  const ConvParams p = conv_params(a);
  cudaStream_t st = semx::as_stream(stream);
  return a->bf16 ? launch_conv<true>(false, a->K, p, st) : launch_conv<false>(false, a->K, p, st);
}

int semx_conv_silu_bwd(const SemxConvSiluArgs* a, semx_stream_t stream) {
  SEMX_CHECK_ARGS(a, SemxConvSiluArgs);
  int rc = conv_validate(a, true);
  if (rc != SEMX_OK) return rc;
  if (a->S * a->C == 0) return SEMX_OK;
  SEMX_REQUIRE(a->workspace, SEMX_ERR_WORKSPACE, "conv_silu bwd: workspace is NULL");
  rc = semx::bind_device({a->workspace});
  if (rc != SEMX_OK) return rc;
  cudaStream_t st = semx::as_stream(stream);
  ConvParams p = conv_params(a);
  float* ws = reinterpret_cast<float*>(a->workspace);
  p.part = ws;
  const int64_t Kc = a->C * (a->K + 1);
  if (a->L > 0) {
    rc = a->bf16 ? launch_conv<true>(true, a->K, p, st) : launch_conv<false>(true, a->K, p, st);
    if (rc != SEMX_OK) return rc;
  } else {
    cudaMemsetAsync(ws, 0, (size_t)a->S * Kc * sizeof(float), st);
  }
  semx::Segments seg = {};
  seg.n = 2;
  seg.out[0] = a->dw;
  seg.out[1] = a->db;
  seg.len[0] = a->C * a->K;
  seg.len[1] = a->C;
  return semx::colsum(ws, a->S, Kc, ws + (size_t)a->S * Kc, seg, st);
}

int semx_gate_silu_fwd(const SemxGateSiluArgs* a, semx_stream_t stream) {
  SEMX_CHECK_ARGS(a, SemxGateSiluArgs);
  SEMX_REQUIRE(a->n >= 0 && a->C >= 0 && a->ld >= 2 * a->C, SEMX_ERR_SHAPE, "gate_silu: bad shape");
  if (a->n * a->C == 0) return SEMX_OK;
  SEMX_REQUIRE(a->y && a->xz && a->o, SEMX_ERR_NULL, "gate_silu: NULL operand");
  int rc = semx::bind_device({a->o});
  if (rc != SEMX_OK) return rc;
  GateParams p = {};
  p.n = a->n; p.C = a->C; p.ld = a->ld; p.y = a->y; p.xz = a->xz; p.o = a->o;
  const unsigned grid = (unsigned)semx::cdiv(p.n * semx::cdiv(p.C, kCV), 256);
  cudaStream_t st = semx::as_stream(stream);
  if (a->bf16) gate_silu_fwd_kernel<true><<<grid, 256, 0, st>>>(p);
  else gate_silu_fwd_kernel<false><<<grid, 256, 0, st>>>(p);
  return semx::check_launch("gate_silu_fwd_kernel");
}

int semx_gate_silu_bwd(const SemxGateSiluArgs* a, semx_stream_t stream) {
  SEMX_CHECK_ARGS(a, SemxGateSiluArgs);
  SEMX_REQUIRE(a->n >= 0 && a->C >= 0 && a->ld >= 2 * a->C, SEMX_ERR_SHAPE, "gate_silu: bad shape");
  if (a->n * a->C == 0) return SEMX_OK;
  SEMX_REQUIRE(a->y && a->xz && a->dout && a->dy && a->dxz, SEMX_ERR_NULL, "gate_silu bwd: NULL operand");
  int rc = semx::bind_device({a->dy});
  if (rc != SEMX_OK) return rc;
  GateParams p = {};
  p.n = a->n; p.C = a->C; p.ld = a->ld; p.y = a->y; p.xz = a->xz; p.dout = a->dout; p.dy = a->dy;
  p.dxz = a->dxz;
  const unsigned grid = (unsigned)semx::cdiv(p.n * semx::cdiv(p.C, kCV), 256);
  cudaStream_t st = semx::as_stream(stream);
  if (a->bf16) gate_silu_bwd_kernel<true><<<grid, 256, 0, st>>>(p);
  else gate_silu_bwd_kernel<false><<<grid, 256, 0, st>>>(p);
  return semx::check_launch("gate_silu_bwd_kernel");
}

}  // extern "C"
