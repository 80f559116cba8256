// Selective-LRU SISO scan with fused discretisation, readout and D skip, for sm_100a.
//
// Reference behaviour (paths relative to the reference project):
//   models/selective_lru/selective_lru.py:242-276   materialised SelectiveLRU path
//   models/selective_lru/selective_lru.py:590-599   _selective_recurrence
//   models/selective_lru/selective_lru_triton.py:528-577  fused_selective_lru operator
//
// Thread layout. A thread owns (sequence s, channel c, group g of kGM = 4 modes): lane
// = cl * NG + g, where NG = ceil(N / 4) lanes share a channel and a warp covers 32 / NG
// channels of the same sequence. A CTA of kThreads covers CB = kThreads / NG channels;
// grid = (channel blocks, sequences). The operands of a block of consecutive steps for the
// CTA's channels (delta_nu, x, delta_theta, dy; B_t, C_t) are staged in shared memory by
// all threads together with cp.async, double-buffered; the pole, drive and gain of every
// (t, c, n) are computed in registers and never touch HBM.
//
// Forward: y_t = sum over modes (reduced over the NG lanes of a channel by shuffles).
// Training forwards also store the state entering every `chunk`-step block.
//
// Backward, per chunk (last first), on the chunk's staged operands:
//   pass 1  re-runs the chunk from its checkpoint, dropping the state every kR steps
//           into shared memory;
//   pass 2  walks kR-step sub-blocks backwards: recompute the kR states into registers,
//           then run the adjoint through them in carry form, c_t = conj(lam_t) G_t,
//           G_t = g_t + c_{t+1}. Per-(t, c) gradients are reduced over the NG lanes by
//           shuffles; per-(t, n) gradients dB / dC are reduced over channels in a fixed
//           order: transposed shuffles inside the warp, then shared memory across warps,
//           then DSMEM across the CTAs of a thread-block cluster of up to kMaxClusterCTAs
//           channel blocks every flush_steps() steps; when the sequence has more channel blocks
//           than one cluster, each cluster writes its sums per (t, n) and dbc_sum_kernel
//           adds the clusters in order.
// Per-(c, n) parameter gradients are summed per thread over time, written per sequence,
// and reduced over sequences by a two-stage fixed-order column sum.
#include <cooperative_groups.h>

#include "semx_common.cuh"
#include "semx_math.cuh"
#include "semx_reduce.cuh"

namespace cg = cooperative_groups;
using semx::ex2_approx;
using semx::rcp_approx;
using semx::rsqrt_approx;
using semx::sin_reduced;
using semx::sincos_reduced;

namespace {

constexpr int kThreads = 128;
constexpr int kGM = 4;      // modes per thread
constexpr int kR = 4;       // steps per register-resident sub-block (backward)
// Steps per dB/dC cluster reduction (backward). The real kernels keep 8: their 6 CTAs per SM
// are bounded by shared memory, which a longer flush window cuts to 5 (measured 1.153 ->
// 1.171 ms at 404 x 321); the complex kernels, bounded at 3 CTAs per SM by registers, take
// 16 and halve their cluster barriers (1616 x 321: 12.01 -> 11.71 ms).
template <bool REAL> constexpr int flush_steps() { return REAL ? 8 : 16; }
constexpr int kTileF = 32;  // steps per staged tile, forward (real)
// Complex forwards stage 16 steps: their 40 KB of double-buffered 32-step tiles held 5 CTAs
// per SM where registers allow 7 (404 x 321 gamma forward 0.852 -> 0.824 ms).
template <bool REAL> constexpr int tile_f() { return REAL ? kTileF : 16; }
constexpr int kTileB = 16;  // steps per staged tile, backward
// Two CTAs per cluster: measured faster than 8 (which spans a 256-channel sequence and
// needs no cluster sums in HBM) on every shape tried — real 404 x 321 backward 1.53 ->
// 1.44 ms, complex 200 x 321 2.21 -> 2.09 ms, complex 1600 x 321 15.7 -> 15.2 ms — since
// small clusters schedule more freely and their barriers wait on fewer CTAs.
constexpr int kMaxClusterCTAs = 2;
constexpr float kLog2e = 1.4426950408889634f;

struct SParams {
  semx::RowMap rm;  // token row of (sequence, step)
  int real, gain, chunk, nchunks;
  int64_t S, L, C, N;
  int detune, envelope;
  int ncl;        // CTAs per cluster
  int nclusters;  // clusters per sequence (channel-block groups)
  const float* dnu;
  const float* dth;
  const float* a;
  const float* om;
  const float* Bre;
  const float* Bim;
  const float* Cre;
  const float* Cim;
  const float* x;
  const float* D;
  const float* g;
  const float* sdet;
  const float* h0r;
  const float* h0i;
  float* y;
  float* hfr;
  float* hfi;
  float* ckpt;
  const float* dy;
  const float* dhfr;
  const float* dhfi;
  float* d_dnu;
  float* d_dth;
  float* dx;
  float* dBre;
  float* dBim;
  float* dCre;
  float* dCim;
  float* dh0r;
  float* dh0i;
  float* part;      // (S, 4*C*N + C) per-sequence parameter-gradient partials
  float* dbc_part;  // (S*L, nclusters, narr*N) when nclusters > 1
};

// Pole, drive gain and their intermediates for one (t, c, n): lam = nu (cs + j sn),
// gain = gr + j gi; rs = 1 / gr for the gamma gain, inv_den = 1 / |A_c|^2 for ZOH.
struct Disc {
  float nu, cs, sn, base, lre, lim, gr, gi, rs, inv_den;
};

template <bool REAL, int GAIN>
__device__ __forceinline__ Disc discretise(float a, float om, float sd, bool detune,
                                           float dnu, float dth) {
  Disc d;
  d.nu = ex2_approx(-dnu * (a * kLog2e));
  if (REAL) {
    d.cs = 1.f;
    d.sn = 0.f;
    d.base = 0.f;
    d.lre = d.nu;
    d.lim = 0.f;
  } else {
    d.base = om + (detune ? sd * dth : dth);
    sincos_reduced(dnu * d.base, &d.sn, &d.cs);
    d.lre = d.nu * d.cs;
    d.lim = d.nu * d.sn;
  }
  d.gi = 0.f;
  d.rs = 1.f;
  d.inv_den = 1.f;
  if (GAIN == SEMX_GAIN_GAMMA) {
    // sqrt(max(1 - nu^2, 1e-6)) as q * rsqrt(q): the reciprocal serves the backward.
    const float q = fmaxf(1.f - d.nu * d.nu, 1e-6f);
    d.rs = rsqrt_approx(q);
    d.gr = q * d.rs;
  } else if (GAIN == SEMX_GAIN_MAMBA) {
    d.gr = dnu;
  } else {  // ZOH: (lam - 1) / A_c, A_c = -a + j base, with lam - 1 from expm1
    const float em1 = expm1f(-dnu * a);
    if (REAL) {
      d.inv_den = rcp_approx(fmaxf(a * a, 1e-8f));
      d.gr = -(a * em1) * d.inv_den;
    } else {
      const float sh = sin_reduced(0.5f * (dnu * d.base));
      const float lm1r = em1 * d.cs - 2.f * sh * sh;
      const float lm1i = d.lim;
      d.inv_den = rcp_approx(fmaxf(a * a + d.base * d.base, 1e-8f));
      d.gr = (d.base * lm1i - a * lm1r) * d.inv_den;
      d.gi = -(a * lm1i + d.base * lm1r) * d.inv_den;
    }
  }
  return d;
}

template <bool REAL>
struct StepIn {
  float dnu, dth, x, dy;
  float bre[kGM], bim[kGM], cre[kGM], cim[kGM];
};

__device__ __forceinline__ bool semx_aligned16(const void* ptr) {
  return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0;
}

struct ModeParams {
  float a[kGM], om[kGM], sd[kGM], ge[kGM];
  bool ok[kGM];
};

__device__ __forceinline__ void load_params(const SParams& p, int c, int g, bool cval,
                                            ModeParams& mp) {
#pragma unroll
  for (int j = 0; j < kGM; ++j) {
    const int n = g * kGM + j;
    mp.ok[j] = cval && n < p.N;
    const int64_t i = (int64_t)c * p.N + n;
    mp.a[j] = mp.ok[j] ? p.a[i] : 0.f;
    mp.om[j] = (mp.ok[j] && !p.real) ? p.om[i] : 0.f;
    mp.sd[j] = (mp.ok[j] && p.detune) ? p.sdet[i] : 1.f;
    mp.ge[j] = (mp.ok[j] && p.envelope) ? p.g[i] : 0.f;
  }
}

template <int NG>
__device__ __forceinline__ float sum_lanes(float v) {
#pragma unroll
  for (int m = NG / 2; m >= 1; m /= 2) v += __shfl_xor_sync(0xffffffffu, v, m);
  return v;
}

// Sums v[0..V) over the CW lanes lane = cl * NG + g that share g (cl = 0..CW-1).
// V >= CW: lane cl ends with the totals of value indices [cl*V/CW, (cl+1)*V/CW) in
//          v[0..V/CW);
// V <  CW: every lane ends with the total of value index cl / (CW/V) in v[0].
// Transposed halving (each round sends half of the remaining values) followed by
// butterfly rounds when there are more lanes than values.
template <int V, int CW, int NG>
__device__ __forceinline__ void lane_reduce(float (&v)[V], int cl) {
  constexpr int kT = (V < CW) ? V : CW;
#pragma unroll
  for (int r = 0; (1 << r) < kT; ++r) {
    const int m = CW >> (r + 1);
    const int n = V >> (r + 1);
    const bool up = (cl & m) != 0;
#pragma unroll
    for (int i = 0; i < n; ++i) {
      const float send = up ? v[i] : v[i + n];
      const float keep = up ? v[i + n] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, m * NG);
    }
  }
#pragma unroll
  for (int m = (CW / kT) / 2; m >= 1; m /= 2) v[0] += __shfl_xor_sync(0xffffffffu, v[0], m * NG);
}

// ------------------------------------------------------------------- staged operand tiles
// The operands of TT consecutive steps for a CTA's channel block are copied into shared
// memory by all of the CTA's threads together (cp.async, 16 B per copy when the rows are
// 16-byte aligned), double-buffered so the next tile is in flight while the current one
// is consumed. Per buffer:
//   channel rows [kRowC][TT][CB]: delta_nu, x, delta_theta (complex only), dy (backward)
//   mode rows    [kRowN][TT][NP]: B_re, C_re, B_im, C_im (imaginary rows complex only)
// with CB = channels per CTA and NP = NG * kGM padded modes. Slots for channels >= C or
// modes >= N are zeroed once and never written by the copies, so those lanes compute on
// zeros: their state stays exactly zero and they contribute nothing.
template <bool REAL, int NG, int TT, bool DY>
struct Tiles {
  static constexpr int kTT = TT;
  static constexpr int CB = kThreads / NG;
  static constexpr int NP = NG * kGM;
  static constexpr int kRowTh = REAL ? -1 : 2;
  static constexpr int kRowDy = DY ? (REAL ? 2 : 3) : -1;
  static constexpr int kRowC = (REAL ? 2 : 3) + (DY ? 1 : 0);
  static constexpr int kRowN = REAL ? 2 : 4;
  static constexpr int kBuf = TT * (kRowC * CB + kRowN * NP);  // floats per buffer
  __host__ __device__ static constexpr size_t bytes() { return (size_t)2 * kBuf * sizeof(float); }
  __device__ static float* chan(float* buf, int row) { return buf + row * TT * CB; }
  __device__ static float* mode(float* buf, int row) { return buf + kRowC * TT * CB + row * TT * NP; }
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }

// Zeroes the padding slots of both buffers (channels >= nc, modes >= N).
template <class T>
__device__ void tile_zero_padding(float* smem, int nc, int N) {
  for (int b = 0; b < 2; ++b) {
    float* buf = smem + b * T::kBuf;
    for (int i = threadIdx.x; i < T::kRowC * T::kTT * T::CB; i += kThreads)
      if (i % T::CB >= nc) buf[i] = 0.f;
    float* mb = T::mode(buf, 0);
    for (int i = threadIdx.x; i < T::kRowN * T::kTT * T::NP; i += kThreads)
      if (i % T::NP >= N) mb[i] = 0.f;
  }
}

template <class T>
__device__ __forceinline__ const float* chan_src(const SParams& p, int row) {
  if (row == 0) return p.dnu;
  if (row == 1) return p.x;
  if (row == T::kRowTh) return p.dth;
  return p.dy;
}
__device__ __forceinline__ const float* mode_src(const SParams& p, int row) {
  return row == 0 ? p.Bre : (row == 1 ? p.Cre : (row == 2 ? p.Bim : p.Cim));
}

// Issues the copies of steps [t0, t0 + nt) of the sequence whose token rows are
// sb + p.rm.step(t) into `buf` (does not commit).
// A full tile (TT steps, CB channels, N = NP modes, 16-byte rows) takes the first branch,
// whose item -> (row, step, chunk) split uses compile-time shapes (shifts instead of the
// general branch's runtime divisions: the copy loop is a tenth of the kernels' issue slots
// otherwise); ragged tiles take the general branch.
template <class T>
__device__ void tile_load(const SParams& p, float* buf, int64_t sb, int t0, int nt, int c0, int nc,
                          bool vecC, bool vecN) {
  const int N = (int)p.N;
  if (vecC && vecN && nt == T::kTT && nc == T::CB && N == T::NP) {
    constexpr int qc = T::CB / 4, per_c = T::kTT * qc, items_c = T::kRowC * per_c;
#pragma unroll
    for (int it0 = 0; it0 < items_c; it0 += kThreads) {
      const unsigned it = it0 + threadIdx.x;
      if (items_c % kThreads == 0 || it < (unsigned)items_c) {
        const unsigned a = it / per_c, rem = it % per_c, i = rem / qc, j = rem % qc;
        cp_async16(T::chan(buf, a) + i * T::CB + 4 * j,
                   chan_src<T>(p, a) + ((sb + p.rm.step(t0 + i)) * p.C + c0) + 4 * j);
      }
    }
    constexpr int qn = T::NP / 4, per_n = T::kTT * qn, items_n = T::kRowN * per_n;
#pragma unroll
    for (int it0 = 0; it0 < items_n; it0 += kThreads) {
      const unsigned it = it0 + threadIdx.x;
      if (items_n % kThreads == 0 || it < (unsigned)items_n) {
        const unsigned a = it / per_n, rem = it % per_n, i = rem / qn, j = rem % qn;
        cp_async16(T::mode(buf, a) + i * T::NP + 4 * j,
                   mode_src(p, a) + (sb + p.rm.step(t0 + i)) * T::NP + 4 * j);
      }
    }
    return;
  }
  if (vecC) {
    const int q = nc >> 2;  // 16-byte chunks per channel row
    const int items = T::kRowC * nt * q;
    for (int it = threadIdx.x; it < items; it += kThreads) {
      const int a = it / (nt * q), rem = it % (nt * q), i = rem / q, j = rem % q;
      const float* src = chan_src<T>(p, a) + ((sb + p.rm.step(t0 + i)) * p.C + c0) + 4 * j;
      cp_async16(T::chan(buf, a) + i * T::CB + 4 * j, src);
    }
  } else {
    const int items = T::kRowC * nt * nc;
    for (int it = threadIdx.x; it < items; it += kThreads) {
      const int a = it / (nt * nc), rem = it % (nt * nc), i = rem / nc, j = rem % nc;
      cp_async4(T::chan(buf, a) + i * T::CB + j, chan_src<T>(p, a) + ((sb + p.rm.step(t0 + i)) * p.C + c0) + j);
    }
  }
  if (vecN) {
    const int q = N >> 2;
    const int items = T::kRowN * nt * q;
    for (int it = threadIdx.x; it < items; it += kThreads) {
      const int a = it / (nt * q), rem = it % (nt * q), i = rem / q, j = rem % q;
      cp_async16(T::mode(buf, a) + i * T::NP + 4 * j, mode_src(p, a) + (sb + p.rm.step(t0 + i)) * p.N + 4 * j);
    }
  } else {
    const int items = T::kRowN * nt * N;
    for (int it = threadIdx.x; it < items; it += kThreads) {
      const int a = it / (nt * N), rem = it % (nt * N), i = rem / N, j = rem % N;
      cp_async4(T::mode(buf, a) + i * T::NP + j, mode_src(p, a) + (sb + p.rm.step(t0 + i)) * p.N + j);
    }
  }
}

// Reads step i of a staged tile for this thread's channel and modes.
template <bool REAL, class T, bool WITH_C>
__device__ __forceinline__ void tile_step(float* buf, int i, int cl, int g, StepIn<REAL>& in) {
  in.dnu = T::chan(buf, 0)[i * T::CB + cl];
  in.x = T::chan(buf, 1)[i * T::CB + cl];
  in.dth = REAL ? 0.f : T::chan(buf, T::kRowTh < 0 ? 0 : T::kRowTh)[i * T::CB + cl];
  in.dy = T::kRowDy < 0 ? 0.f : T::chan(buf, T::kRowDy < 0 ? 0 : T::kRowDy)[i * T::CB + cl];
  const float4 br = *reinterpret_cast<const float4*>(T::mode(buf, 0) + i * T::NP + g * kGM);
  in.bre[0] = br.x; in.bre[1] = br.y; in.bre[2] = br.z; in.bre[3] = br.w;
  if (WITH_C) {
    const float4 cr = *reinterpret_cast<const float4*>(T::mode(buf, 1) + i * T::NP + g * kGM);
    in.cre[0] = cr.x; in.cre[1] = cr.y; in.cre[2] = cr.z; in.cre[3] = cr.w;
  }
  if (!REAL) {
    const float4 bi = *reinterpret_cast<const float4*>(T::mode(buf, 2) + i * T::NP + g * kGM);
    in.bim[0] = bi.x; in.bim[1] = bi.y; in.bim[2] = bi.z; in.bim[3] = bi.w;
    if (WITH_C) {
      const float4 ci = *reinterpret_cast<const float4*>(T::mode(buf, 3) + i * T::NP + g * kGM);
      in.cim[0] = ci.x; in.cim[1] = ci.y; in.cim[2] = ci.z; in.cim[3] = ci.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < kGM; ++j) in.bim[j] = in.cim[j] = 0.f;
  }
}

// One step of the recurrence for this thread's modes: h = lam h + gain x B.
template <bool REAL, int GAIN>
__device__ __forceinline__ void advance(const ModeParams& mp, bool detune, const StepIn<REAL>& in,
                                        float (&hr)[kGM], float (&hi)[kGM]) {
#pragma unroll
  for (int j = 0; j < kGM; ++j) {
    const Disc d = discretise<REAL, GAIN>(mp.a[j], mp.om[j], mp.sd[j], detune, in.dnu, in.dth);
    const float gxr = d.gr * in.x;
    if (REAL) {
      hr[j] = d.lre * hr[j] + gxr * in.bre[j];
    } else {
      const float gxi = d.gi * in.x;
      const float ur = gxr * in.bre[j] - gxi * in.bim[j];
      const float ui = gxr * in.bim[j] + gxi * in.bre[j];
      const float nr = d.lre * hr[j] - d.lim * hi[j] + ur;
      const float ni = d.lre * hi[j] + d.lim * hr[j] + ui;
      hr[j] = nr;
      hi[j] = ni;
    }
  }
}

// The complex gamma-gain Disc of a step from its kept pole: nu^2 = |lam|^2, the gain
// sqrt(max(1 - nu^2, 1e-6)) as q rsqrt(q); nu itself is not needed (nu2 is returned).
__device__ __forceinline__ Disc kept_pole(float lre, float lim, float om, float sd, bool detune, float dth,
                                          float& nu2) {
  Disc d;
  d.lre = lre;
  d.lim = lim;
  d.base = om + (detune ? sd * dth : dth);
  nu2 = fmaf(lre, lre, lim * lim);
  const float q = fmaxf(1.f - nu2, 1e-6f);
  d.rs = rsqrt_approx(q);
  d.gr = q * d.rs;
  d.gi = 0.f;
  d.nu = 0.f;
  d.cs = d.sn = 0.f;
  d.inv_den = 1.f;
  return d;
}

// advance(), also returning each mode's pole (lre, lim) for the adjoint of the same step.
template <bool REAL, int GAIN>
__device__ __forceinline__ void advance_keep(const ModeParams& mp, bool detune, const StepIn<REAL>& in,
                                             float (&hr)[kGM], float (&hi)[kGM], float (&lr)[kGM],
                                             float (&li)[kGM]) {
#pragma unroll
  for (int j = 0; j < kGM; ++j) {
    const Disc d = discretise<REAL, GAIN>(mp.a[j], mp.om[j], mp.sd[j], detune, in.dnu, in.dth);
    lr[j] = d.lre;
    li[j] = d.lim;
    const float gxr = d.gr * in.x;
    if (REAL) {
      hr[j] = d.lre * hr[j] + gxr * in.bre[j];
    } else {
      const float gxi = d.gi * in.x;
      const float ur = gxr * in.bre[j] - gxi * in.bim[j];
      const float ui = gxr * in.bim[j] + gxi * in.bre[j];
      const float nr = d.lre * hr[j] - d.lim * hi[j] + ur;
      const float ni = d.lre * hi[j] + d.lim * hr[j] + ui;
      hr[j] = nr;
      hi[j] = ni;
    }
  }
}

// ----------------------------------------------------------------------------- forward
template <bool REAL, int GAIN, int NG, bool EXTRA>
__global__ void __launch_bounds__(kThreads) slru_fwd_kernel(const SParams p) {
  constexpr int TF = tile_f<REAL>();
  using T = Tiles<REAL, NG, TF, false>;
  constexpr int CW = 32 / NG;
  extern __shared__ float4 fwd_smem4[];
  float* smem = reinterpret_cast<float*>(fwd_smem4);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cl = lane / NG, g = lane % NG;
  const int c_local = warp * CW + cl;
  const int c0 = blockIdx.x * T::CB;
  const int c = c0 + c_local;
  const int64_t s = blockIdx.y;
  const int64_t sb = p.rm.seq(s);  // token row of step t: sb + p.rm.step(t)
  const bool cval = c < p.C;
  const int nc = (int)min((int64_t)T::CB, p.C - c0);
  const int L = (int)p.L;
  const bool vecC = (p.C % 4) == 0 && semx_aligned16(p.dnu) && semx_aligned16(p.x) &&
                    (REAL || semx_aligned16(p.dth));
  // Per-mode detune (complex only) and envelope readout exist only in the EXTRA build.
  const bool detune = EXTRA && !REAL && p.detune;
  const bool envelope = EXTRA && p.envelope;
  const bool vecN = (p.N % 4) == 0 && semx_aligned16(p.Bre) && semx_aligned16(p.Cre) &&
                    (REAL || (semx_aligned16(p.Bim) && semx_aligned16(p.Cim)));

  ModeParams mp;
  load_params(p, c, g, cval, mp);
  const float Dc = cval ? p.D[c] : 0.f;
  float hr[kGM], hi[kGM];
#pragma unroll
  for (int j = 0; j < kGM; ++j) {
    const int64_t i = (s * p.C + c) * p.N + g * kGM + j;
    hr[j] = (mp.ok[j] && p.h0r) ? p.h0r[i] : 0.f;
    hi[j] = (mp.ok[j] && p.h0i && !REAL) ? p.h0i[i] : 0.f;
  }

  tile_zero_padding<T>(smem, nc, (int)p.N);
  const int ntiles = (L + TF - 1) / TF;
  if (ntiles > 0) tile_load<T>(p, smem, sb, 0, min(TF, L), c0, nc, vecC, vecN);
  cp_async_commit();
  int next_ck = 0;
  float* yrow = p.y + sb * p.C + c;  // step t: yrow[p.rm.step(t) * C]
  for (int k = 0; k < ntiles; ++k) {
    cp_async_wait_all();
    __syncthreads();
    if (k + 1 < ntiles)
      tile_load<T>(p, smem + ((k + 1) & 1) * T::kBuf, sb, (k + 1) * TF,
                   min(TF, L - (k + 1) * TF), c0, nc, vecC, vecN);
    cp_async_commit();
    float* buf = smem + (k & 1) * T::kBuf;
    const int t0 = k * TF, nt = min(TF, L - t0);
    // Unrolled so the poles of later steps (which do not depend on the state) issue
    // between the state updates: real 404 x 321 forward 0.38 -> 0.30 ms.
#pragma unroll 8
    for (int i = 0; i < nt; ++i) {
      const int t = t0 + i;
      if (p.ckpt != nullptr && t == next_ck) {
        const int64_t base = ((s * p.nchunks + t / p.chunk) * p.C + c) * p.N + g * kGM;
#pragma unroll
        for (int j = 0; j < kGM; ++j) {
          if (mp.ok[j]) {
            if (REAL) p.ckpt[base + j] = hr[j];
            else reinterpret_cast<float2*>(p.ckpt)[base + j] = make_float2(hr[j], hi[j]);
          }
        }
        next_ck += p.chunk;
      }
      StepIn<REAL> cur;
      tile_step<REAL, T, true>(buf, i, c_local, g, cur);
      advance<REAL, GAIN>(mp, detune, cur, hr, hi);
      float yp = 0.f;
#pragma unroll
      for (int j = 0; j < kGM; ++j) {
        yp += cur.cre[j] * hr[j];
        if (!REAL) yp -= cur.cim[j] * hi[j];
      }
      if (envelope) {
#pragma unroll
        for (int j = 0; j < kGM; ++j) yp += mp.ge[j] * (hr[j] * hr[j] + (REAL ? 0.f : hi[j] * hi[j]));
      }
      yp = sum_lanes<NG>(yp);
      if (g == 0 && cval) yrow[p.rm.step(t) * p.C] = yp + Dc * cur.x;
    }
  }
  if (p.hfr != nullptr) {
#pragma unroll
    for (int j = 0; j < kGM; ++j) {
      if (mp.ok[j]) {
        const int64_t i = (s * p.C + c) * p.N + g * kGM + j;
        p.hfr[i] = hr[j];
        if (!REAL && p.hfi) p.hfi[i] = hi[j];
      }
    }
  }
}

// ------------------------------------------------- forward, real, modes in registers
// The real scan with N <= 16 modes: one thread per (sequence, channel) holding all of the
// channel's modes in registers, so y_t = D x_t + sum_n C_t[n] h_t[n] is summed inside the
// thread (no lane shuffles) and each staged dnu / x value is read once per step instead
// of once per 4-mode group. A CTA covers kRmCB channels of one sequence; operand tiles of
// kRmTT steps are staged by cp.async (dnu, x per channel; B_t, C_t per mode, padded to 16
// with zeros: a padded mode keeps a zero state and adds nothing). Checkpoints hold the same
// (S, nchunks, C, N) layout as slru_fwd_kernel's, so the backward is shared.
constexpr int kRmCB = 128;  // channels per CTA
constexpr int kRmTT = 16;   // steps per staged tile
constexpr int kRmNM = 16;   // modes held per thread

struct TilesRM {
  static constexpr int kTT = kRmTT;
  static constexpr int CB = kRmCB;
  static constexpr int NP = kRmNM;
  static constexpr int kRowTh = -1;
  static constexpr int kRowDy = -1;
  static constexpr int kRowC = 2;  // delta_nu, x
  static constexpr int kRowN = 2;  // B, C
  static constexpr int kBuf = kTT * (kRowC * CB + kRowN * NP);
  __host__ __device__ static constexpr size_t bytes() { return (size_t)2 * kBuf * sizeof(float); }
  __device__ static float* chan(float* buf, int row) { return buf + row * kTT * CB; }
  __device__ static float* mode(float* buf, int row) { return buf + kRowC * kTT * CB + row * kTT * NP; }
};

template <int GAIN, bool EXTRA>
__global__ void __launch_bounds__(kRmCB, 6) slru_fwd_real16_kernel(const SParams p) {
  using T = TilesRM;
  constexpr int NM = kRmNM, TT = kRmTT;
  extern __shared__ float4 rm_smem4[];
  float* smem = reinterpret_cast<float*>(rm_smem4);
  const int tid = threadIdx.x;
  const int c0 = blockIdx.x * T::CB;
  const int c = c0 + tid;
  const int64_t s = blockIdx.y;
  const int64_t sb = p.rm.seq(s);  // token row of step t: sb + p.rm.step(t)
  const bool cval = c < p.C;
  const int nc = (int)min((int64_t)T::CB, p.C - c0);
  const int L = (int)p.L, N = (int)p.N;
  const bool vecC = (p.C % 4) == 0 && semx_aligned16(p.dnu) && semx_aligned16(p.x);
  const bool vecN = (p.N % 4) == 0 && semx_aligned16(p.Bre) && semx_aligned16(p.Cre);
  const bool envelope = EXTRA && p.envelope;

  float a[NM], ge[NM], h[NM];
#pragma unroll
  for (int n = 0; n < NM; ++n) {
    const bool ok = cval && n < N;
    const int64_t i = (int64_t)c * N + n;
    a[n] = ok ? p.a[i] : 0.f;
    ge[n] = (ok && envelope) ? p.g[i] : 0.f;
    h[n] = (ok && p.h0r) ? p.h0r[(s * p.C + c) * N + n] : 0.f;
  }
  const float Dc = cval ? p.D[c] : 0.f;

  tile_zero_padding<T>(smem, nc, N);
  const int ntiles = (L + TT - 1) / TT;
  if (ntiles > 0) tile_load<T>(p, smem, sb, 0, min(TT, L), c0, nc, vecC, vecN);
  cp_async_commit();
  int next_ck = 0;
  float* yrow = p.y + sb * p.C + c;  // step t: yrow[p.rm.step(t) * C]
  const bool ck16 = N == NM && semx_aligned16(p.ckpt);
  for (int k = 0; k < ntiles; ++k) {
    cp_async_wait_all();
    __syncthreads();
    if (k + 1 < ntiles)
      tile_load<T>(p, smem + ((k + 1) & 1) * T::kBuf, sb, (k + 1) * TT, min(TT, L - (k + 1) * TT), c0, nc,
                   vecC, vecN);
    cp_async_commit();
    const float* buf = smem + (k & 1) * T::kBuf;
    const float* dnus = buf;
    const float* xs = buf + TT * T::CB;
    const float* Bs = buf + T::kRowC * TT * T::CB;
    const float* Cs = Bs + TT * T::NP;
    const int t0 = k * TT, nt = min(TT, L - t0);
#pragma unroll 2
    for (int i = 0; i < nt; ++i) {
      const int t = t0 + i;
      if (p.ckpt != nullptr && t == next_ck) {
        if (cval) {
          float* ck = p.ckpt + ((s * p.nchunks + t / p.chunk) * p.C + c) * N;
          if (ck16) {
#pragma unroll
            for (int n = 0; n < NM; n += 4)
              *reinterpret_cast<float4*>(ck + n) = make_float4(h[n], h[n + 1], h[n + 2], h[n + 3]);
          } else {
#pragma unroll
            for (int n = 0; n < NM; ++n)
              if (n < N) ck[n] = h[n];
          }
        }
        next_ck += p.chunk;
      }
      const float dnu = dnus[i * T::CB + tid], x = xs[i * T::CB + tid];
      const float dx_m = dnu * x;  // the Mamba gain's drive scale
      // Four partial readout sums (one per mode of a float4 group), so the readout is four
      // chains of four FMAs instead of one chain of sixteen.
      float yq[4] = {Dc * x, 0.f, 0.f, 0.f};
#pragma unroll
      for (int n4 = 0; n4 < NM; n4 += 4) {
        const float4 b4 = *reinterpret_cast<const float4*>(Bs + i * T::NP + n4);
        const float4 c4 = *reinterpret_cast<const float4*>(Cs + i * T::NP + n4);
        const float bb[4] = {b4.x, b4.y, b4.z, b4.w}, cc[4] = {c4.x, c4.y, c4.z, c4.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int n = n4 + j;
          const Disc d = discretise<true, GAIN>(a[n], 0.f, 1.f, false, dnu, 0.f);
          const float gx = GAIN == SEMX_GAIN_MAMBA ? dx_m : d.gr * x;
          h[n] = fmaf(d.lre, h[n], gx * bb[j]);
          yq[j] = fmaf(cc[j], h[n], yq[j]);
          if (envelope) yq[j] = fmaf(ge[n], h[n] * h[n], yq[j]);
        }
      }
      if (cval) yrow[p.rm.step(t) * p.C] = (yq[0] + yq[1]) + (yq[2] + yq[3]);
    }
  }
  if (p.hfr != nullptr && cval) {
#pragma unroll
    for (int n = 0; n < NM; ++n)
      if (n < N) p.hfr[(s * p.C + c) * N + n] = h[n];
  }
}

// ---------------------------------------------------------------------------- backward
template <bool REAL, int NG>
struct BwdLayout {
  using T = Tiles<REAL, NG, kTileB, true>;
  static constexpr int kHS = REAL ? 1 : 2;    // float4 groups per sub-checkpoint (re [, im])
  static constexpr int kNArr = REAL ? 2 : 4;  // dB(re [, im]), dC(re [, im])
  static constexpr int kV = kNArr * kGM;      // dB/dC values per thread per step
  static constexpr int kNV = NG * kV;         // values per warp per step
  static constexpr int kNW = kThreads / 32;
  __host__ __device__ static constexpr size_t tile_floats() { return 2 * (size_t)T::kBuf; }
  static constexpr int kFlush = flush_steps<REAL>();
  __host__ __device__ static constexpr size_t red_floats() { return (size_t)2 * kFlush * kNW * kNV; }
  __host__ __device__ static size_t sub_floats(int chunk) {
    return (size_t)(chunk / kR) * kHS * kThreads * kGM;
  }
  __host__ __device__ static size_t bytes(int chunk) {
    return (tile_floats() + red_floats() + sub_floats(chunk)) * sizeof(float);
  }
};

// The backward visits each chunk's staged tiles in this order: a chunk of one tile once
// (pass 1 and pass 2 on the same tile); a longer chunk's tiles forwards for pass 1, then
// backwards for pass 2.
struct TileEntry {
  int t0, nt;
  bool p1, p2;
};
__device__ __forceinline__ int tiles_in_chunk(int k, int K, int L) {
  const int t0 = k * K, t1 = min(t0 + K, L);
  return (t1 - t0 + kTileB - 1) / kTileB;
}
__device__ __forceinline__ int entries_of(int k, int K, int L) {
  const int nq = tiles_in_chunk(k, K, L);
  return nq == 1 ? 1 : 2 * nq;
}
__device__ __forceinline__ TileEntry entry_of(int k, int e, int K, int L) {
  const int t0 = k * K, t1 = min(t0 + K, L);
  const int nq = tiles_in_chunk(k, K, L);
  TileEntry E;
  int q;
  if (nq == 1) {
    q = 0;
    E.p1 = E.p2 = true;
  } else if (e < nq) {
    q = e;
    E.p1 = true;
    E.p2 = false;
  } else {
    q = 2 * nq - 1 - e;
    E.p1 = false;
    E.p2 = true;
  }
  E.t0 = t0 + q * kTileB;
  E.nt = min(kTileB, t1 - E.t0);
  return E;
}

// Complex gamma kernels run 3 CTAs per SM: with the kept poles they need more than the 128
// registers of 4 CTAs (which spilled; 404 x 321 backward 3.233 -> 3.203 ms at 164).
template <bool REAL, int GAIN, int NG, bool EXTRA>
__global__ void __launch_bounds__(kThreads, REAL ? 0 : (GAIN == SEMX_GAIN_GAMMA ? 3 : 4)) slru_bwd_kernel(const SParams p) {
  using Lay = BwdLayout<REAL, NG>;
  using T = typename Lay::T;
  constexpr int CW = 32 / NG;
  constexpr int V = Lay::kV;
  constexpr int NV = Lay::kNV;
  constexpr int NW = Lay::kNW;
  constexpr int HS = Lay::kHS;
  extern __shared__ float4 bwd_smem4[];
  float* tiles = reinterpret_cast<float*>(bwd_smem4);
  constexpr int kFlush = Lay::kFlush;
  float* red = tiles + Lay::tile_floats();                                  // [2][kFlush][NW][NV]
  float4* sub = reinterpret_cast<float4*>(red + Lay::red_floats());         // [chunk/kR][HS][kThreads]
  cg::cluster_group cluster = cg::this_cluster();
  const int crank = (int)cluster.block_rank();

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cl = lane / NG, g = lane % NG;
  const int c_local = warp * CW + cl;
  const int c0 = blockIdx.x * T::CB;
  const int c = c0 + c_local;
  const int64_t s = blockIdx.y;
  const int64_t sb = p.rm.seq(s);  // token row of step t: sb + p.rm.step(t)
  const bool cval = c < p.C;
  const int nc = (int)max((int64_t)0, min((int64_t)T::CB, p.C - c0));
  const int L = (int)p.L;
  const int N = (int)p.N;
  const int K = p.chunk;
  const bool vecC = (p.C % 4) == 0 && semx_aligned16(p.dnu) && semx_aligned16(p.x) &&
                    semx_aligned16(p.dy) && (REAL || semx_aligned16(p.dth));
  const bool detune = EXTRA && !REAL && p.detune;
  const bool envelope = EXTRA && p.envelope;
  const bool vecN = (p.N % 4) == 0 && semx_aligned16(p.Bre) && semx_aligned16(p.Cre) &&
                    (REAL || (semx_aligned16(p.Bim) && semx_aligned16(p.Cim)));

  ModeParams mp;
  load_params(p, c, g, cval, mp);
  const float Dc = cval ? p.D[c] : 0.f;

  // Carry c_{t+1} = conj(lam_{t+1}) G_{t+1}; it starts as the final-state gradient.
  float cr[kGM], ci[kGM];
  float acc_a[kGM], acc_om[kGM], acc_s[kGM], acc_g[kGM];
  float acc_D = 0.f;
#pragma unroll
  for (int j = 0; j < kGM; ++j) {
    const int64_t i = (s * p.C + c) * p.N + g * kGM + j;
    const bool has = mp.ok[j] && p.dhfr != nullptr;
    cr[j] = has ? p.dhfr[i] : 0.f;
    ci[j] = (has && !REAL && p.dhfi) ? p.dhfi[i] : 0.f;
    acc_a[j] = acc_om[j] = acc_s[j] = acc_g[j] = 0.f;
  }

  tile_zero_padding<T>(tiles, nc, N);
  if (p.nchunks > 0) {
    const TileEntry E = entry_of(p.nchunks - 1, 0, K, L);
    tile_load<T>(p, tiles, sb, E.t0, E.nt, c0, nc, vecC, vecN);
  }
  cp_async_commit();
  int bsel = 0;

  for (int k = p.nchunks - 1; k >= 0; --k) {
    const int t0c = k * K;
    const int nE = entries_of(k, K, L);
    // Pass-1 state: the checkpoint stored by the forward at the start of chunk k.
    float hr[kGM], hi[kGM];
    {
      const int64_t cb = ((s * p.nchunks + k) * p.C + c) * p.N + g * kGM;
#pragma unroll
      for (int j = 0; j < kGM; ++j) {
        if (REAL) {
          hr[j] = mp.ok[j] ? p.ckpt[cb + j] : 0.f;
          hi[j] = 0.f;
        } else {
          const float2 v = mp.ok[j] ? reinterpret_cast<const float2*>(p.ckpt)[cb + j]
                                    : make_float2(0.f, 0.f);
          hr[j] = v.x;
          hi[j] = v.y;
        }
      }
    }
    for (int e = 0; e < nE; ++e) {
      const TileEntry E = entry_of(k, e, K, L);
      cp_async_wait_all();
      __syncthreads();
      {
        const int kn = (e + 1 < nE) ? k : k - 1;
        const int en = (e + 1 < nE) ? e + 1 : 0;
        if (kn >= 0) {
          const TileEntry En = entry_of(kn, en, K, L);
          tile_load<T>(p, tiles + (bsel ^ 1) * T::kBuf, sb, En.t0, En.nt, c0, nc, vecC, vecN);
        }
        cp_async_commit();
      }
      float* buf = tiles + bsel * T::kBuf;

      if (E.p1 && K == kR) {  // the checkpoint is the chunk's only sub-block start
        sub[tid] = make_float4(hr[0], hr[1], hr[2], hr[3]);
        if (!REAL) sub[kThreads + tid] = make_float4(hi[0], hi[1], hi[2], hi[3]);
      } else if (E.p1) {  // Pass 1: recurrence from the checkpoint, state every kR steps kept.
#pragma unroll 4
        for (int i = 0; i < E.nt; ++i) {
          const int t = E.t0 + i;
          if (((t - t0c) % kR) == 0) {
            const int si = (t - t0c) / kR;
            sub[(si * HS) * kThreads + tid] = make_float4(hr[0], hr[1], hr[2], hr[3]);
            if (!REAL) sub[(si * HS + 1) * kThreads + tid] = make_float4(hi[0], hi[1], hi[2], hi[3]);
          }
          StepIn<REAL> in;
          tile_step<REAL, T, false>(buf, i, c_local, g, in);
          advance<REAL, GAIN>(mp, detune, in, hr, hi);
        }
      }

      if (E.p2) {  // Pass 2: kR-step sub-blocks, last first.
        const int nsb = (E.nt + kR - 1) / kR;
        for (int r = nsb - 1; r >= 0; --r) {
          const int ta = E.t0 + r * kR;
          const int nr = min(kR, E.t0 + E.nt - ta);
          const int si = (ta - t0c) / kR;
          float H0r[kGM], H0i[kGM], Hr[kR][kGM], Hi[kR][kGM];
          // Complex gamma gain: the recompute keeps each step's pole for the adjoint, which
          // then evaluates only the gain's rsqrt (nu^2 = |lam|^2) instead of ex2, sin and cos.
          constexpr bool KEEP = !REAL && GAIN == SEMX_GAIN_GAMMA;
          float Lr[kR][kGM], Li[kR][kGM];
          {
            const float4 v = sub[(si * HS) * kThreads + tid];
            H0r[0] = v.x; H0r[1] = v.y; H0r[2] = v.z; H0r[3] = v.w;
            if (!REAL) {
              const float4 w = sub[(si * HS + 1) * kThreads + tid];
              H0i[0] = w.x; H0i[1] = w.y; H0i[2] = w.z; H0i[3] = w.w;
            } else {
#pragma unroll
              for (int j = 0; j < kGM; ++j) H0i[j] = 0.f;
            }
          }
          // Recompute the sub-block's states.
#pragma unroll
          for (int i = 0; i < kR; ++i) {
#pragma unroll
            for (int j = 0; j < kGM; ++j) {
              Hr[i][j] = i == 0 ? H0r[j] : Hr[i > 0 ? i - 1 : 0][j];
              Hi[i][j] = i == 0 ? H0i[j] : Hi[i > 0 ? i - 1 : 0][j];
            }
            if (i < nr) {
              StepIn<REAL> in;
              tile_step<REAL, T, false>(buf, ta - E.t0 + i, c_local, g, in);
              if (KEEP) advance_keep<REAL, GAIN>(mp, detune, in, Hr[i], Hi[i], Lr[i], Li[i]);
              else advance<REAL, GAIN>(mp, detune, in, Hr[i], Hi[i]);
            }
          }
          // Adjoint through the sub-block.
#pragma unroll
          for (int i = kR - 1; i >= 0; --i) {
            if (i < nr) {
              const int t = ta + i;
              StepIn<REAL> in;
              tile_step<REAL, T, true>(buf, t - E.t0, c_local, g, in);
              const float dyv = in.dy;
              float sum_dnu = 0.f, sum_dth = 0.f, sum_dx = 0.f;
              float vals[V];
#pragma unroll
              for (int j = 0; j < kGM; ++j) {
                const float hrt = Hr[i][j], hit = Hi[i][j];
                const float hpr = i == 0 ? H0r[j] : Hr[i > 0 ? i - 1 : 0][j];
                const float hpi = i == 0 ? H0i[j] : Hi[i > 0 ? i - 1 : 0][j];
                float nu2k = 0.f;
                const Disc d = KEEP ? kept_pole(Lr[i][j], Li[i][j], mp.om[j], mp.sd[j], detune, in.dth, nu2k)
                                    : discretise<REAL, GAIN>(mp.a[j], mp.om[j], mp.sd[j], detune,
                                                             in.dnu, in.dth);
                // Local adjoint from the readout (and the envelope term).
                float gre = dyv * in.cre[j];
                float gim = REAL ? 0.f : -dyv * in.cim[j];
                if (envelope) {
                  const float w = 2.f * dyv * mp.ge[j];
                  gre += w * hrt;
                  if (!REAL) gim += w * hit;
                  acc_g[j] += dyv * (hrt * hrt + (REAL ? 0.f : hit * hit));
                }
                const float Gr = gre + cr[j];
                const float Gi = REAL ? 0.f : gim + ci[j];
                cr[j] = REAL ? d.lre * Gr : d.lre * Gr + d.lim * Gi;
                ci[j] = REAL ? 0.f : d.lre * Gi - d.lim * Gr;
                // Drive Bu = gain x B. With bG = conj(B) G: dB = conj(gain x) G,
                // dx += Re(conj(gain) bG), d(gain) = x bG.
                const float bGr = REAL ? in.bre[j] * Gr : in.bre[j] * Gr + in.bim[j] * Gi;
                const float bGi = REAL ? 0.f : in.bre[j] * Gi - in.bim[j] * Gr;
                const float gxr = d.gr * in.x, gxi = d.gi * in.x;
                const float vBr = REAL ? gxr * Gr : gxr * Gr + gxi * Gi;
                const float vBi = REAL ? 0.f : gxr * Gi - gxi * Gr;
                sum_dx += (GAIN == SEMX_GAIN_ZOH && !REAL) ? d.gr * bGr + d.gi * bGi : d.gr * bGr;
                const float dgr = in.x * bGr;
                const float dgi = in.x * bGi;
                // P = nu * dL/dnu and d_th = dL/d(angle), from d lam = G conj(h_{t-1}):
                // nu (dlre cs + dlim sn) = dlre lre + dlim lim, nu (dlim cs - dlre sn) =
                // dlim lre - dlre lim.
                const float dlre = REAL ? Gr * hpr : Gr * hpr + Gi * hpi;
                const float dlim = REAL ? 0.f : Gi * hpr - Gr * hpi;
                float P = REAL ? dlre * d.lre : dlre * d.lre + dlim * d.lim;
                const float d_th = REAL ? 0.f : dlim * d.lre - dlre * d.lim;
                float d_dnu = 0.f, da_extra = 0.f, dbase_extra = 0.f;
                if (GAIN == SEMX_GAIN_GAMMA) {
                  // gain = sqrt(max(1 - nu^2, 1e-6)): nu d gain / d nu = -nu^2 / gain where live.
                  const float nu2 = KEEP ? nu2k : d.nu * d.nu;
                  P -= ((1.f - nu2) >= 1e-6f) ? dgr * nu2 * d.rs : 0.f;
                } else if (GAIN == SEMX_GAIN_MAMBA) {
                  d_dnu = dgr;
                } else {
                  // d gain / d delta_nu = lam; d gain / d A_c = (dnu lam - gain) / A_c = q.
                  d_dnu = dgr * d.lre + dgi * d.lim;
                  const float pr = in.dnu * d.lre - d.gr;
                  const float pi = in.dnu * d.lim - d.gi;
                  const float qr = (d.base * pi - mp.a[j] * pr) * d.inv_den;
                  const float qi = -(mp.a[j] * pi + d.base * pr) * d.inv_den;
                  da_extra = -(dgr * qr + dgi * qi);
                  dbase_extra = dgi * qr - dgr * qi;
                }
                // nu = exp(-dnu a): d nu / d dnu = -a nu, d nu / d a = -dnu nu.
                d_dnu -= mp.a[j] * P;
                acc_a[j] += da_extra - in.dnu * P;
                if (!REAL) {
                  d_dnu += d_th * d.base;
                  const float dbase = d_th * in.dnu + dbase_extra;
                  acc_om[j] += dbase;
                  sum_dth += detune ? dbase * mp.sd[j] : dbase;
                  if (detune) acc_s[j] += dbase * in.dth;
                }
                sum_dnu += d_dnu;
                vals[0 * kGM + j] = vBr;
                if (REAL) {
                  vals[1 * kGM + j] = dyv * hrt;
                } else {
                  vals[1 * kGM + j] = vBi;
                  vals[2 * kGM + j] = dyv * hrt;
                  vals[3 * kGM + j] = -dyv * hit;
                }
              }
              if (g == 0) acc_D += dyv * in.x;
              sum_dnu = sum_lanes<NG>(sum_dnu);
              sum_dx = sum_lanes<NG>(sum_dx);
              if (!REAL) sum_dth = sum_lanes<NG>(sum_dth);
              if (g == 0 && cval) {
                const int64_t ic = (sb + p.rm.step(t)) * p.C + c;
                if (p.d_dnu) p.d_dnu[ic] = sum_dnu;
                if (!REAL && p.d_dth) p.d_dth[ic] = sum_dth;
                if (p.dx) p.dx[ic] = sum_dx + dyv * Dc;
              }
              lane_reduce<V, CW, NG>(vals, cl);
              float* dst = red + ((size_t)(((t / kFlush) & 1) * kFlush + (t % kFlush)) * NW + warp) * NV + g * V;
              if (V >= CW) {
#pragma unroll
                for (int m = 0; m < (V >= CW ? V / CW : 1); ++m) dst[cl * (V / CW) + m] = vals[m];
              } else if ((cl % (V < CW ? CW / V : 1)) == 0) {
                dst[cl / (V < CW ? CW / V : 1)] = vals[0];
              }
            }
          }
          if ((ta % kFlush) == 0) {
            // Steps [ta, ta + kFlush) complete on every CTA of the cluster: sum dB / dC over
            // warps and over the cluster's CTAs in a fixed order.
            cluster.sync();
            const float* redb = red + (size_t)((ta / kFlush) & 1) * kFlush * NW * NV;
            const int nitems = min(kFlush, L - ta) * NV;
            const int stride = p.ncl * kThreads;
            for (int it = crank * kThreads + tid; it < nitems; it += stride) {
              const int tl = it / NV, kk = it % NV;
              const int gg = kk / V, vv = kk % V;
              const int arr = vv / kGM, n = gg * kGM + (vv % kGM);
              if (n >= N) continue;
              float acc = 0.f;
              for (int q = 0; q < p.ncl; ++q) {
                const float* peer = cluster.map_shared_rank(redb, q);
#pragma unroll
                for (int w = 0; w < NW; ++w) acc += peer[((size_t)tl * NW + w) * NV + kk];
              }
              const int64_t row = sb + p.rm.step(ta + tl);
              if (p.nclusters > 1) {
                const int clid = blockIdx.x / p.ncl;
                p.dbc_part[(row * p.nclusters + clid) * (Lay::kNArr * N) + arr * N + n] = acc;
              } else {
                float* outp = REAL ? (arr == 0 ? p.dBre : p.dCre)
                                   : (arr == 0 ? p.dBre : arr == 1 ? p.dBim : arr == 2 ? p.dCre : p.dCim);
                if (outp) outp[row * N + n] = acc;
              }
            }
          }
        }
      }
      bsel ^= 1;
    }
  }

  // Initial-state gradient: dh0 = conj(lam_0) G_0, the final carry.
  if (p.dh0r != nullptr) {
#pragma unroll
    for (int j = 0; j < kGM; ++j) {
      if (mp.ok[j]) {
        const int64_t i = (s * p.C + c) * p.N + g * kGM + j;
        p.dh0r[i] = cr[j];
        if (!REAL && p.dh0i) p.dh0i[i] = ci[j];
      }
    }
  }
  // Per-sequence parameter-gradient partials: [da | domega | ds | dg] (C, N) each, dD (C).
  {
    const int64_t Kp = 4 * p.C * p.N + p.C;
    float* row = p.part + s * Kp;
    const int64_t CN = p.C * p.N;
#pragma unroll
    for (int j = 0; j < kGM; ++j) {
      if (mp.ok[j]) {
        const int64_t i = (int64_t)c * p.N + g * kGM + j;
        row[0 * CN + i] = acc_a[j];
        row[1 * CN + i] = acc_om[j];
        row[2 * CN + i] = acc_s[j];
        row[3 * CN + i] = acc_g[j];
      }
    }
    if (g == 0 && cval) row[4 * CN + c] = acc_D;
  }
  cluster.sync();  // no CTA leaves while a peer may still read its shared memory
}

// --------------------------------------------------------------------- reductions
// dB / dC over cluster groups when one cluster cannot span all channel blocks.
__global__ void dbc_sum_kernel(const SParams p, int narr) {
  const int64_t total = p.S * p.L * narr * p.N;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int64_t row = i / (narr * p.N);
  const int rem = (int)(i % (narr * p.N));
  const int arr = rem / (int)p.N, n = rem % (int)p.N;
  float acc = 0.f;
  for (int q = 0; q < p.nclusters; ++q) acc += p.dbc_part[(row * p.nclusters + q) * (narr * p.N) + rem];
  float* outp = narr == 2 ? (arr == 0 ? p.dBre : p.dCre)
                          : (arr == 0 ? p.dBre : arr == 1 ? p.dBim : arr == 2 ? p.dCre : p.dCim);
  if (outp) outp[row * p.N + n] = acc;
}

// The same with 4 consecutive modes per thread (N % 4 == 0, every buffer 16-byte aligned).
__global__ void dbc_sum4_kernel(const SParams p, int narr) {
  const int64_t nq = p.N / 4;
  const int64_t total = p.S * p.L * narr * nq;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int64_t row = i / (narr * nq);
  const int rem = (int)(i % (narr * nq));
  const int arr = rem / (int)nq, n = (rem % (int)nq) * 4;
  const float4* src = reinterpret_cast<const float4*>(p.dbc_part + row * p.nclusters * (narr * p.N) + arr * p.N + n);
  const int64_t stride = (narr * p.N) / 4;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int q = 0; q < p.nclusters; ++q) {
    const float4 v = src[q * stride];
    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
  }
  float* outp = narr == 2 ? (arr == 0 ? p.dBre : p.dCre)
                          : (arr == 0 ? p.dBre : arr == 1 ? p.dBim : arr == 2 ? p.dCre : p.dCim);
  if (outp) *reinterpret_cast<float4*>(outp + row * p.N + n) = acc;
}

// ------------------------------------------------------------------------ host side
int ng_for(int64_t N) {
  const int64_t ng = semx::cdiv(N, kGM);
  if (ng <= 1) return 1;
  if (ng <= 2) return 2;
  if (ng <= 4) return 4;
  return 8;
}

struct Geometry {
  int ng, cb, nblocks, ncl, nclusters, grid_x;
};

Geometry geometry(const SemxSelectiveLruArgs* a) {
  Geometry g;
  g.ng = ng_for(a->N);
  g.cb = kThreads / g.ng;
  g.nblocks = (int)semx::cdiv(a->C, g.cb);
  g.ncl = g.nblocks < kMaxClusterCTAs ? g.nblocks : kMaxClusterCTAs;
  if (g.ncl < 1) g.ncl = 1;
  g.nclusters = (int)semx::cdiv(g.nblocks, g.ncl);
  g.grid_x = g.nclusters * g.ncl;
  return g;
}

size_t bwd_smem(const SemxSelectiveLruArgs* a, int ng) {
  const bool real = a->real != 0;
  switch (ng) {
#define SEMX_CASE(NGV)                                                                \
  case NGV:                                                                           \
    return real ? BwdLayout<true, NGV>::bytes(a->chunk) : BwdLayout<false, NGV>::bytes(a->chunk);
    SEMX_CASE(1)
    SEMX_CASE(2)
    SEMX_CASE(4)
    SEMX_CASE(8)
#undef SEMX_CASE
  }
  return 0;
}

int validate(const SemxSelectiveLruArgs* a, bool bwd) {
  SEMX_REQUIRE(a->S >= 0 && a->L >= 0 && a->C >= 0 && a->N >= 0, SEMX_ERR_SHAPE,
               "selective_lru: negative size");
  SEMX_REQUIRE(a->N <= 32, SEMX_ERR_UNSUPPORTED, "selective_lru: N=%lld > 32",
               (long long)a->N);
  SEMX_REQUIRE(a->S <= 65535, SEMX_ERR_SHAPE, "selective_lru: S=%lld > 65535 (grid.y)",
               (long long)a->S);
  SEMX_REQUIRE(a->input_gain >= SEMX_GAIN_GAMMA && a->input_gain <= SEMX_GAIN_ZOH,
               SEMX_ERR_UNSUPPORTED, "selective_lru: input_gain=%d", a->input_gain);
  SEMX_REQUIRE(a->chunk >= kR && a->chunk <= 256 && a->chunk % kR == 0, SEMX_ERR_UNSUPPORTED,
               "selective_lru: chunk=%d must be a multiple of %d in [%d, 256]", a->chunk, kR, kR);
  semx::RowMap rm;
  const int rc = semx::make_rowmap(a->S, a->L, a->reverse, a->seq_group, a->group_stride, a->seq_stride,
                                   a->step_stride, &rm, "selective_lru");
  if (rc != SEMX_OK) return rc;
  const bool real = a->real != 0;
  const bool any = a->S * a->C > 0;
  if (any && a->N > 0) {
    SEMX_REQUIRE(a->a != nullptr && (real || a->omega != nullptr), SEMX_ERR_NULL,
                 "selective_lru: a/omega is NULL");
  }
  if (any) SEMX_REQUIRE(a->D != nullptr, SEMX_ERR_NULL, "selective_lru: D is NULL");
  if (a->S * a->L * a->C > 0) {
    SEMX_REQUIRE(a->delta_nu && a->x && (real || a->delta_theta), SEMX_ERR_NULL,
                 "selective_lru: delta_nu/delta_theta/x is NULL");
    if (a->N > 0) {
      SEMX_REQUIRE(a->B_re && a->C_re && (real || (a->B_im && a->C_im)), SEMX_ERR_NULL,
                   "selective_lru: B/C is NULL");
      if (a->N % 4 == 0) {
        SEMX_REQUIRE(semx::aligned(a->B_re, 16) && semx::aligned(a->C_re, 16) &&
                         (real || (semx::aligned(a->B_im, 16) && semx::aligned(a->C_im, 16))),
                     SEMX_ERR_ALIGN, "selective_lru: B/C must be 16-byte aligned when N %% 4 == 0");
      }
    }
    if (!bwd) SEMX_REQUIRE(a->y != nullptr, SEMX_ERR_NULL, "selective_lru: y is NULL");
    if (bwd) SEMX_REQUIRE(a->dy != nullptr, SEMX_ERR_NULL, "selective_lru bwd: dy is NULL");
  }
  if (!real) {
    SEMX_REQUIRE(!a->ckpt || semx::aligned(a->ckpt, 8), SEMX_ERR_ALIGN,
                 "selective_lru: ckpt must be 8-byte aligned");
  }
  if (bwd && a->S * a->C * a->N > 0) {
    SEMX_REQUIRE(a->ckpt != nullptr || a->L == 0, SEMX_ERR_NULL,
                 "selective_lru bwd: ckpt is NULL");
    SEMX_REQUIRE(a->workspace != nullptr, SEMX_ERR_WORKSPACE, "selective_lru bwd: workspace");
  }
  if (bwd) {
    const Geometry g = geometry(a);
    const size_t smem = bwd_smem(a, g.ng);
    SEMX_REQUIRE(smem <= 227 * 1024, SEMX_ERR_UNSUPPORTED,
                 "selective_lru bwd: chunk=%d needs %zu B of shared memory (> 227 KB)",
                 a->chunk, smem);
  }
  return SEMX_OK;
}

SParams to_params(const SemxSelectiveLruArgs* a) {
  SParams p = {};
  semx::make_rowmap(a->S, a->L, a->reverse, a->seq_group, a->group_stride, a->seq_stride, a->step_stride, &p.rm,
                    "selective_lru");
  const Geometry g = geometry(a);
  p.real = a->real != 0;
  p.gain = a->input_gain;
  p.chunk = a->chunk;
  p.nchunks = (int)semx::cdiv(a->L, a->chunk);
  p.S = a->S;
  p.L = a->L;
  p.C = a->C;
  p.N = a->N;
  p.detune = (!p.real && a->s != nullptr) ? 1 : 0;
  p.envelope = a->g != nullptr ? 1 : 0;
  p.ncl = g.ncl;
  p.nclusters = g.nclusters;
  p.dnu = a->delta_nu;
  p.dth = a->delta_theta;
  p.a = a->a;
  p.om = a->omega;
  p.Bre = a->B_re;
  p.Bim = a->B_im;
  p.Cre = a->C_re;
  p.Cim = a->C_im;
  p.x = a->x;
  p.D = a->D;
  p.g = a->g;
  p.sdet = a->s;
  p.h0r = a->h0_re;
  p.h0i = a->h0_im;
  p.y = a->y;
  p.hfr = a->hf_re;
  p.hfi = a->hf_im;
  p.ckpt = a->ckpt;
  p.dy = a->dy;
  p.dhfr = a->dhf_re;
  p.dhfi = a->dhf_im;
  p.d_dnu = a->d_delta_nu;
  p.d_dth = a->d_delta_theta;
  p.dx = a->dx;
  p.dBre = a->dB_re;
  p.dBim = a->dB_im;
  p.dCre = a->dC_re;
  p.dCim = a->dC_im;
  p.dh0r = a->dh0_re;
  p.dh0i = a->dh0_im;
  return p;
}

size_t part_floats(const SemxSelectiveLruArgs* a) {
  return (size_t)a->S * (size_t)(4 * a->C * a->N + a->C);
}
size_t group_floats(const SemxSelectiveLruArgs* a) {
  return semx::colsum_group_floats(a->S, 4 * a->C * a->N + a->C);
}
size_t dbc_floats(const SemxSelectiveLruArgs* a) {
  const Geometry g = geometry(a);
  if (g.nclusters <= 1) return 0;
  return (size_t)a->S * a->L * g.nclusters * (a->real ? 2 : 4) * a->N;
}

template <bool REAL, int GAIN, int NG, bool EXTRA>
int launch_fwd(const SParams& p, const Geometry& g, cudaStream_t st) {
  const dim3 grid((unsigned)g.nblocks, (unsigned)p.S);
  const size_t smem = Tiles<REAL, NG, tile_f<REAL>(), false>::bytes();
  auto kern = slru_fwd_kernel<REAL, GAIN, NG, EXTRA>;
  if (!semx::allow_smem(kern, smem)) return SEMX_ERR_LAUNCH;
  kern<<<grid, kThreads, smem, st>>>(p);
  return semx::check_launch("slru_fwd_kernel");
}

template <int GAIN, bool EXTRA>
int launch_fwd_rm(const SParams& p, cudaStream_t st) {
  const dim3 grid((unsigned)semx::cdiv(p.C, kRmCB), (unsigned)p.S);
  const size_t smem = TilesRM::bytes();
  auto kern = slru_fwd_real16_kernel<GAIN, EXTRA>;
  if (!semx::allow_smem(kern, smem)) return SEMX_ERR_LAUNCH;
  kern<<<grid, kRmCB, smem, st>>>(p);
  return semx::check_launch("slru_fwd_real16_kernel");
}

// The real forward with N <= 16 modes (slru_fwd_real16_kernel), specialised on the gain
// and the envelope readout.
int launch_fwd_real16(const SemxSelectiveLruArgs* a, const SParams& p, cudaStream_t st) {
  const bool env = p.envelope != 0;
  switch (a->input_gain) {
    case SEMX_GAIN_GAMMA:
      return env ? launch_fwd_rm<SEMX_GAIN_GAMMA, true>(p, st) : launch_fwd_rm<SEMX_GAIN_GAMMA, false>(p, st);
    case SEMX_GAIN_MAMBA:
      return env ? launch_fwd_rm<SEMX_GAIN_MAMBA, true>(p, st) : launch_fwd_rm<SEMX_GAIN_MAMBA, false>(p, st);
    default:
      return env ? launch_fwd_rm<SEMX_GAIN_ZOH, true>(p, st) : launch_fwd_rm<SEMX_GAIN_ZOH, false>(p, st);
  }
}

template <bool REAL, int GAIN, int NG, bool EXTRA>
int launch_bwd(const SParams& p, const Geometry& g, size_t smem, cudaStream_t st) {
  auto kern = slru_bwd_kernel<REAL, GAIN, NG, EXTRA>;
  if (!semx::allow_smem(kern, smem)) return SEMX_ERR_LAUNCH;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)g.grid_x, (unsigned)p.S);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)g.ncl;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
  if (e != cudaSuccess)
    return semx::fail(SEMX_ERR_LAUNCH, "slru_bwd_kernel launch: %s", cudaGetErrorString(e));
  return semx::check_launch("slru_bwd_kernel");
}

template <bool REAL, int GAIN, bool EXTRA>
int dispatch_ng(bool bwd, const SParams& p, const Geometry& g, size_t smem, cudaStream_t st) {
  switch (g.ng) {
#define SEMX_CASE(NGV) \
  case NGV:            \
    return bwd ? launch_bwd<REAL, GAIN, NGV, EXTRA>(p, g, smem, st)  \
               : launch_fwd<REAL, GAIN, NGV, EXTRA>(p, g, st);
    SEMX_CASE(1)
    SEMX_CASE(2)
    SEMX_CASE(4)
    SEMX_CASE(8)
#undef SEMX_CASE
  }
  return semx::fail(SEMX_ERR_UNSUPPORTED, "selective_lru: no kernel for NG=%d", g.ng);
}

template <int GAIN, bool EXTRA>
int dispatch_real(bool bwd, bool real, const SParams& p, const Geometry& g, size_t smem,
                  cudaStream_t st) {
  return real ? dispatch_ng<true, GAIN, EXTRA>(bwd, p, g, smem, st)
              : dispatch_ng<false, GAIN, EXTRA>(bwd, p, g, smem, st);
}

// Kernels are specialised on the element type, the input gain, the lanes per channel and
// whether the per-mode detune or the envelope readout is on (EXTRA).
int dispatch(bool bwd, const SemxSelectiveLruArgs* a, const SParams& p, const Geometry& g,
             size_t smem, cudaStream_t st) {
  const bool real = a->real != 0;
  const bool extra = p.detune || p.envelope;
  switch (a->input_gain) {
    case SEMX_GAIN_GAMMA:
      return extra ? dispatch_real<SEMX_GAIN_GAMMA, true>(bwd, real, p, g, smem, st)
                   : dispatch_real<SEMX_GAIN_GAMMA, false>(bwd, real, p, g, smem, st);
    case SEMX_GAIN_MAMBA:
      return extra ? dispatch_real<SEMX_GAIN_MAMBA, true>(bwd, real, p, g, smem, st)
                   : dispatch_real<SEMX_GAIN_MAMBA, false>(bwd, real, p, g, smem, st);
    default:
      return extra ? dispatch_real<SEMX_GAIN_ZOH, true>(bwd, real, p, g, smem, st)
                   : dispatch_real<SEMX_GAIN_ZOH, false>(bwd, real, p, g, smem, st);
  }
}

}  // namespace

extern "C" {

size_t semx_selective_lru_args_size(void) { return sizeof(SemxSelectiveLruArgs); }

size_t semx_selective_lru_ckpt_bytes(const SemxSelectiveLruArgs* a) {
  if (a == nullptr || a->chunk <= 0 || a->S < 0 || a->L < 0 || a->C < 0 || a->N < 0) return 0;
  return (size_t)a->S * (size_t)semx::cdiv(a->L, a->chunk) * (size_t)a->C * (size_t)a->N *
         (a->real ? 1 : 2) * sizeof(float);
}

size_t semx_selective_lru_workspace_bytes(const SemxSelectiveLruArgs* a) {
  if (a == nullptr || a->S < 0 || a->L < 0 || a->C < 0 || a->N < 0) return 0;
  return (part_floats(a) + group_floats(a) + dbc_floats(a)) * sizeof(float);
}

int semx_selective_lru_fwd(const SemxSelectiveLruArgs* a, semx_stream_t stream) {
  SEMX_CHECK_ARGS(a, SemxSelectiveLruArgs);
  int rc = validate(a, false);
  if (rc != SEMX_OK) return rc;
  if (a->S * a->C == 0) return SEMX_OK;
  rc = semx::bind_device({a->y, a->delta_nu, a->D});
  if (rc != SEMX_OK) return rc;
  const SParams p = to_params(a);
  if (a->real && a->N <= kRmNM) return launch_fwd_real16(a, p, semx::as_stream(stream));
  const Geometry g = geometry(a);
  return dispatch(false, a, p, g, 0, semx::as_stream(stream));
}

int semx_selective_lru_bwd(const SemxSelectiveLruArgs* a, semx_stream_t stream) {
  SEMX_CHECK_ARGS(a, SemxSelectiveLruArgs);
  int rc = validate(a, true);
  if (rc != SEMX_OK) return rc;
  rc = semx::bind_device({a->dy, a->D, a->workspace});
  if (rc != SEMX_OK) return rc;
  cudaStream_t st = semx::as_stream(stream);
  SParams p = to_params(a);
  const Geometry g = geometry(a);
  const int64_t K = 4 * a->C * a->N + a->C;
  if (a->S * a->C > 0) {
    float* ws = reinterpret_cast<float*>(a->workspace);
    p.part = ws;
    p.dbc_part = ws + part_floats(a) + group_floats(a);
    rc = dispatch(true, a, p, g, bwd_smem(a, g.ng), st);
    if (rc != SEMX_OK) return rc;
    if (g.nclusters > 1 && a->S * a->L * a->N > 0) {
      const int narr = a->real ? 2 : 4;
      const int64_t total = a->S * a->L * narr * a->N;
      const bool vec = a->N % 4 == 0 && semx::aligned(p.dbc_part, 16) && semx::aligned(p.dBre, 16) &&
                       semx::aligned(p.dBim, 16) && semx::aligned(p.dCre, 16) && semx::aligned(p.dCim, 16);
      if (vec) dbc_sum4_kernel<<<(unsigned)semx::cdiv(total / 4, 256), 256, 0, st>>>(p, narr);
      else dbc_sum_kernel<<<(unsigned)semx::cdiv(total, 256), 256, 0, st>>>(p, narr);
      rc = semx::check_launch("dbc_sum_kernel");
      if (rc != SEMX_OK) return rc;
    }
    float* gsum = ws + part_floats(a);
    semx::Segments seg = {};
    const int64_t CN = a->C * a->N;
    seg.n = 5;
    seg.out[0] = a->da;
    seg.out[1] = a->real ? nullptr : a->domega;
    seg.out[2] = (a->real || a->s == nullptr) ? nullptr : a->ds;
    seg.out[3] = a->g ? a->dg : nullptr;
    seg.out[4] = a->dD;
    seg.len[0] = seg.len[1] = seg.len[2] = seg.len[3] = CN;
    seg.len[4] = a->C;
    return semx::colsum(ws, a->S, K, gsum, seg, st);
  }
  return SEMX_OK;
}

}  // extern "C"
