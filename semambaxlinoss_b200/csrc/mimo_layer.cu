// Fused SelectiveLRUMIMO layer (after its token projections), for sm_100a.
//
// Reference behaviour (paths relative to the reference project):
//   models/selective_lru/selective_lru.py:488-587  SelectiveLRUMIMO.forward
//   models/selective_lru/selective_lru.py:590-599  _selective_recurrence
//
// One CTA per (sequence s, head h); time in kTC-token chunks. Per chunk, all of the
// head's token operands (x, the projection columns of the head) are staged in shared
// memory, then:
//   forward  1. per (t, n): pole lam and gain from (delta_nu, delta_theta), raw drive
//               sum_f B[n,f] x[f] + sum_r s_b[r] b_t[r,n], gained drive;
//            2. per mode n (one thread each): h_t = lam h_{t-1} + Bu over the chunk;
//            3. per (t, r): the rank read s_c Re(<c_t, h>);
//            4. per (t, f): y = Re(C h) + D x + <env, |h|^2> + rank feedthrough.
//   backward (chunks last first) recomputes 1-2 from the chunk's checkpoint, forms the
//            readout adjoint g per (t, n), runs G_t = g_t + conj(lam_{t+1}) G_{t+1} per
//            mode, and back-propagates through the gain, the pole and the drive. Token
//            gradients (dx, dproj) are written directly; parameter gradients are summed
//            per CTA in a fixed order, written as per-sequence partial rows and reduced
//            over sequences by the two-stage column sum.
// Every parallel loop distributes (t, n) or (t, f) items so that a warp's shared-memory
// reads of the per-head matrices are consecutive (both storage orders of B, C and
// env_gain are kept where both access orders occur).
#include <cuda_bf16.h>

#include "semx_common.cuh"
#include "semx_math.cuh"
#include "semx_reduce.cuh"

namespace {

constexpr int kT = 128;   // threads per CTA
constexpr int kTC = 32;   // tokens per chunk
constexpr int kMaxNh = 64;
constexpr int kMaxFh = 256;
constexpr int kMaxR = 16;
constexpr float kLog2e = 1.4426950408889634f;

struct LParams {
  int64_t S, L, H, Nh, Fh, R, P;  // P = projection row width
  int gain, detune, envelope, nchunks;
  float rs;
  const void* x;
  const void* proj;
  const float* A_log;
  const float* omega;
  const float* sdet;
  const float* B;
  const float* C;
  const float* D;
  const float* cout;
  const float* env;
  float* y;
  float* ckpt;
  const float* dy;
  float* dx;
  void* dproj;
  float* part;  // (S, K) partial parameter-gradient rows
  int64_t K;
};

// Shared-memory layout in floats (every offset a multiple of 4).
struct Lay {
  int Bt, Bn, Cn, Cf, En, Ef, Co, Dp, prm;
  int xs, raw, dnu, dth, sb, bt, sc, ct;
  int lam, gn, bu, hs, sr;
  int dys, dr, gs, db, tn, acc;
  int total;
};

__host__ __device__ inline int al4(int v) { return (v + 3) & ~3; }

__host__ __device__ inline Lay make_lay(int Nh, int Fh, int R, bool bwd, bool env) {
  Lay l = {};
  int o = 0;
  auto take = [&](int n) {
    const int at = o;
    o += al4(n);
    return at;
  };
  l.Bt = take(Fh * Nh * 2);
  l.Bn = bwd ? take(Nh * Fh * 2) : -1;
  l.Cn = take(Nh * Fh * 2);
  l.Cf = bwd ? take(Fh * Nh * 2) : -1;
  l.En = env ? take(Nh * Fh) : -1;
  l.Ef = (env && bwd) ? take(Fh * Nh) : -1;
  l.Co = take(R * Fh);
  l.Dp = take(Fh);
  l.prm = take(3 * Nh);
  l.xs = take(kTC * Fh);
  l.raw = take(kTC);
  l.dnu = take(kTC);
  l.dth = take(kTC);
  l.sb = take(kTC * R);
  l.bt = take(kTC * R * Nh);
  l.sc = take(kTC * R);
  l.ct = take(kTC * 2 * R * Nh);
  l.lam = take(kTC * Nh * 2);
  l.gn = take(kTC * Nh * 2);
  l.bu = take(kTC * Nh * 2);
  l.hs = take((kTC + 1) * Nh * 2);
  l.sr = take(kTC * R);
  if (bwd) {
    l.dys = take(kTC * Fh);
    l.dr = take(kTC * R);
    l.gs = take(kTC * Nh * 2);
    l.db = take(kTC * Nh * 2);
    l.tn = take(5 * kTC * Nh);
    l.acc = take(Nh * Fh * 2 + Fh * Nh * 2 + (env ? Fh * Nh : 0) + R * Fh + Fh);
  } else {
    l.dys = l.dr = l.gs = l.db = l.tn = l.acc = -1;
  }
  l.total = o;
  return l;
}

// Column offsets of head h's operands in a projection row.
struct Cols {
  int64_t dnu, dth, sb, bt, sc, ct;
};
__device__ __forceinline__ Cols cols_of(const LParams& p, int h) {
  const int64_t H = p.H, R = p.R, Nh = p.Nh;
  Cols c;
  c.dnu = h;
  c.dth = H + h;
  c.sb = 2 * H + (int64_t)h * R;
  c.bt = 2 * H + H * R + (int64_t)h * R * Nh;
  c.sc = 2 * H + H * R + H * R * Nh + (int64_t)h * R;
  c.ct = 2 * H + 2 * H * R + H * R * Nh + (int64_t)h * R * 2 * Nh;
  return c;
}

template <bool BF16>
__device__ __forceinline__ float ld(const void* base, int64_t i) {
  if (BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[i]);
  return reinterpret_cast<const float*>(base)[i];
}
template <bool BF16>
__device__ __forceinline__ void st(void* base, int64_t i, float v) {
  if (BF16) reinterpret_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16(v);
  else reinterpret_cast<float*>(base)[i] = v;
}

// Pole, gain and their intermediates for one (token, head, mode).
struct MDisc {
  float nu, cs, sn, base, lre, lim, gr, gi, rs, inv_den;
};

__device__ __forceinline__ MDisc mdisc(int gain, float a, float om, float sd, bool detune,
                                       float dnu, float dth) {
  MDisc d;
  d.nu = semx::ex2_approx(-dnu * (a * kLog2e));
  d.base = om + (detune ? sd * dth : dth);
  semx::sincos_reduced(dnu * d.base, &d.sn, &d.cs);
  d.lre = d.nu * d.cs;
  d.lim = d.nu * d.sn;
  d.gr = 1.f;
  d.gi = 0.f;
  d.rs = 1.f;
  d.inv_den = 1.f;
  if (gain == SEMX_GAIN_GAMMA) {
    const float q = fmaxf(1.f - d.nu * d.nu, 1e-6f);
    d.rs = semx::rsqrt_approx(q);
    d.gr = q * d.rs;
  } else if (gain == SEMX_GAIN_MAMBA) {
    d.gr = dnu;
  } else if (gain == SEMX_GAIN_ZOH) {
    const float em1 = expm1f(-dnu * a);
    const float sh = semx::sin_reduced(0.5f * (dnu * d.base));
    const float lm1r = em1 * d.cs - 2.f * sh * sh;
    const float lm1i = d.lim;
    d.inv_den = semx::rcp_approx(fmaxf(a * a + d.base * d.base, 1e-8f));
    d.gr = (d.base * lm1i - a * lm1r) * d.inv_den;
    d.gi = -(a * lm1i + d.base * lm1r) * d.inv_den;
  }
  return d;
}

// Loads the head's parameters into shared memory (both storage orders where needed).
__device__ void load_head_params(const LParams& p, const Lay& l, float* sm, int h, bool bwd) {
  const int Nh = (int)p.Nh, Fh = (int)p.Fh, R = (int)p.R;
  for (int i = threadIdx.x; i < Nh * Fh; i += kT) {
    const int n = i / Fh, f = i % Fh;
    const float2 b = reinterpret_cast<const float2*>(p.B)[((int64_t)h * Nh + n) * Fh + f];
    reinterpret_cast<float2*>(sm + l.Bt)[f * Nh + n] = b;
    if (bwd) reinterpret_cast<float2*>(sm + l.Bn)[n * Fh + f] = b;
    const int f2 = i / Nh, n2 = i % Nh;
    const float2 c = reinterpret_cast<const float2*>(p.C)[((int64_t)h * Fh + f2) * Nh + n2];
    reinterpret_cast<float2*>(sm + l.Cn)[n2 * Fh + f2] = c;
    if (bwd) reinterpret_cast<float2*>(sm + l.Cf)[f2 * Nh + n2] = c;
    if (p.envelope) {
      const float e = p.env[((int64_t)h * Fh + f2) * Nh + n2];
      sm[l.En + n2 * Fh + f2] = e;
      if (bwd) sm[l.Ef + f2 * Nh + n2] = e;
    }
  }
  for (int i = threadIdx.x; i < R * Fh; i += kT) sm[l.Co + i] = p.cout[(int64_t)h * R * Fh + i];
  for (int i = threadIdx.x; i < Fh; i += kT) sm[l.Dp + i] = p.D[(int64_t)h * Fh + i];
  for (int n = threadIdx.x; n < Nh; n += kT) {
    sm[l.prm + n] = expf(p.A_log[(int64_t)h * Nh + n]);
    sm[l.prm + Nh + n] = p.omega[(int64_t)h * Nh + n];
    sm[l.prm + 2 * Nh + n] = p.detune ? p.sdet[(int64_t)h * Nh + n] : 1.f;
  }
}

// Stages the chunk's token operands of head h (and dy in the backward).
template <bool BF16>
__device__ void stage_chunk(const LParams& p, const Lay& l, float* sm, int64_t s, int h, int t0,
                            int nt, bool bwd) {
  const int Nh = (int)p.Nh, Fh = (int)p.Fh, R = (int)p.R;
  const Cols c = cols_of(p, h);
  const int64_t Fd = p.H * p.Fh;
  for (int i = threadIdx.x; i < nt * Fh; i += kT) {
    const int t = i / Fh, f = i % Fh;
    const int64_t row = s * p.L + t0 + t;
    sm[l.xs + i] = ld<BF16>(p.x, row * Fd + (int64_t)h * Fh + f);
    if (bwd) sm[l.dys + i] = p.dy[row * Fd + (int64_t)h * Fh + f];
  }
  for (int t = threadIdx.x; t < nt; t += kT) {
    const int64_t row = (s * p.L + t0 + t) * p.P;
    const float raw = ld<BF16>(p.proj, row + c.dnu);
    sm[l.raw + t] = raw;
    sm[l.dnu + t] = semx::softplus(raw) * p.rs;
    sm[l.dth + t] = ld<BF16>(p.proj, row + c.dth);
  }
  if (R > 0) {
    for (int i = threadIdx.x; i < nt * R; i += kT) {
      const int t = i / R, r = i % R;
      const int64_t row = (s * p.L + t0 + t) * p.P;
      sm[l.sb + i] = ld<BF16>(p.proj, row + c.sb + r);
      sm[l.sc + i] = ld<BF16>(p.proj, row + c.sc + r);
    }
    const int wb = R * Nh;
    for (int i = threadIdx.x; i < nt * wb; i += kT) {
      const int t = i / wb, j = i % wb;
      sm[l.bt + i] = ld<BF16>(p.proj, (s * p.L + t0 + t) * p.P + c.bt + j);
    }
    const int wc = 2 * R * Nh;
    for (int i = threadIdx.x; i < nt * wc; i += kT) {
      const int t = i / wc, j = i % wc;
      sm[l.ct + i] = ld<BF16>(p.proj, (s * p.L + t0 + t) * p.P + c.ct + j);
    }
  }
}

// Pole, gain and raw drive per (t, n) of the chunk; `gained` stores gain * drive.
__device__ void poles_and_drive(const LParams& p, const Lay& l, float* sm, int nt, bool gained) {
  const int Nh = (int)p.Nh, Fh = (int)p.Fh, R = (int)p.R;
  const float2* Bt = reinterpret_cast<const float2*>(sm + l.Bt);
  for (int i = threadIdx.x; i < nt * Nh; i += kT) {
    const int t = i / Nh, n = i % Nh;
    const MDisc d = mdisc(p.gain, sm[l.prm + n], sm[l.prm + Nh + n], sm[l.prm + 2 * Nh + n],
                          p.detune != 0, sm[l.dnu + t], sm[l.dth + t]);
    float br = 0.f, bi = 0.f;
    const float* xr = sm + l.xs + t * Fh;
    for (int f = 0; f < Fh; ++f) {
      const float2 b = Bt[f * Nh + n];
      br = fmaf(b.x, xr[f], br);
      bi = fmaf(b.y, xr[f], bi);
    }
    for (int r = 0; r < R; ++r) br = fmaf(sm[l.sb + t * R + r], sm[l.bt + (t * R + r) * Nh + n], br);
    reinterpret_cast<float2*>(sm + l.lam)[i] = make_float2(d.lre, d.lim);
    reinterpret_cast<float2*>(sm + l.gn)[i] = make_float2(d.gr, d.gi);
    reinterpret_cast<float2*>(sm + l.bu)[i] =
        gained ? make_float2(d.gr * br - d.gi * bi, d.gr * bi + d.gi * br) : make_float2(br, bi);
  }
}

// ----------------------------------------------------------------------------- forward
template <bool BF16>
__global__ void __launch_bounds__(kT) mimo_layer_fwd_kernel(const LParams p) {
  extern __shared__ float4 smem4[];
  float* sm = reinterpret_cast<float*>(smem4);
  const int Nh = (int)p.Nh, Fh = (int)p.Fh, R = (int)p.R, L = (int)p.L;
  const Lay l = make_lay(Nh, Fh, R, false, p.envelope != 0);
  const int64_t s = blockIdx.x / p.H;
  const int h = (int)(blockIdx.x % p.H);
  const int tid = threadIdx.x;
  const int64_t Fd = p.H * p.Fh;
  load_head_params(p, l, sm, h, false);
  float2* hs = reinterpret_cast<float2*>(sm + l.hs);
  float2 state = make_float2(0.f, 0.f);  // thread n < Nh: the mode's state
  for (int k = 0; k < p.nchunks; ++k) {
    const int t0 = k * kTC, nt = min(kTC, L - t0);
    __syncthreads();
    stage_chunk<BF16>(p, l, sm, s, h, t0, nt, false);
    __syncthreads();
    poles_and_drive(p, l, sm, nt, true);
    __syncthreads();
    if (tid < Nh) {
      if (p.ckpt) reinterpret_cast<float2*>(p.ckpt)[((s * p.nchunks + k) * p.H + h) * Nh + tid] = state;
      hs[tid] = state;
      const float2* lam = reinterpret_cast<const float2*>(sm + l.lam);
      const float2* bu = reinterpret_cast<const float2*>(sm + l.bu);
      for (int t = 0; t < nt; ++t) {
        const float2 a = lam[t * Nh + tid], u = bu[t * Nh + tid];
        const float nr = fmaf(a.x, state.x, fmaf(-a.y, state.y, u.x));
        const float ni = fmaf(a.x, state.y, fmaf(a.y, state.x, u.y));
        state = make_float2(nr, ni);
        hs[(t + 1) * Nh + tid] = state;
      }
    }
    __syncthreads();
    if (R > 0) {
      for (int i = tid; i < nt * R; i += kT) {
        const int t = i / R, r = i % R;
        const float* cr = sm + l.ct + (t * R + r) * 2 * Nh;
        float acc = 0.f;
        for (int n = 0; n < Nh; ++n) {
          const float2 hv = hs[(t + 1) * Nh + n];
          acc = fmaf(cr[n], hv.x, fmaf(-cr[Nh + n], hv.y, acc));
        }
        sm[l.sr + i] = sm[l.sc + i] * acc;
      }
      __syncthreads();
    }
    const float2* Cn = reinterpret_cast<const float2*>(sm + l.Cn);
    for (int i = tid; i < nt * Fh; i += kT) {
      const int t = i / Fh, f = i % Fh;
      float acc = sm[l.Dp + f] * sm[l.xs + i];
      for (int n = 0; n < Nh; ++n) {
        const float2 hv = hs[(t + 1) * Nh + n];
        const float2 c = Cn[n * Fh + f];
        acc = fmaf(c.x, hv.x, fmaf(-c.y, hv.y, acc));
        if (p.envelope) acc = fmaf(sm[l.En + n * Fh + f], hv.x * hv.x + hv.y * hv.y, acc);
      }
      for (int r = 0; r < R; ++r) acc = fmaf(sm[l.sr + t * R + r], sm[l.Co + r * Fh + f], acc);
      p.y[(s * p.L + t0 + t) * Fd + (int64_t)h * Fh + f] = acc;
    }
  }
}

// ---------------------------------------------------------------------------- backward
template <bool BF16>
__global__ void __launch_bounds__(kT) mimo_layer_bwd_kernel(const LParams p) {
  extern __shared__ float4 smem4[];
  float* sm = reinterpret_cast<float*>(smem4);
  const int Nh = (int)p.Nh, Fh = (int)p.Fh, R = (int)p.R, L = (int)p.L;
  const bool env = p.envelope != 0;
  const Lay l = make_lay(Nh, Fh, R, true, env);
  const int64_t s = blockIdx.x / p.H;
  const int h = (int)(blockIdx.x % p.H);
  const int tid = threadIdx.x;
  const int64_t Fd = p.H * p.Fh;
  const Cols cols = cols_of(p, h);
  load_head_params(p, l, sm, h, true);
  // Parameter accumulators: [dB (Nh,Fh,2) | dC (Fh,Nh,2) | denv (Fh,Nh) | dcout (R,Fh) | dD (Fh)]
  const int oB = 0, oC = oB + Nh * Fh * 2, oE = oC + Fh * Nh * 2, oO = oE + (env ? Fh * Nh : 0),
            oD = oO + R * Fh, nacc = oD + Fh;
  for (int i = tid; i < nacc; i += kT) sm[l.acc + i] = 0.f;
  float2* hs = reinterpret_cast<float2*>(sm + l.hs);
  float2* gs = reinterpret_cast<float2*>(sm + l.gs);
  float2* db = reinterpret_cast<float2*>(sm + l.db);
  const float2* lam = reinterpret_cast<const float2*>(sm + l.lam);
  const float2* gn = reinterpret_cast<const float2*>(sm + l.gn);
  const float2* braw = reinterpret_cast<const float2*>(sm + l.bu);
  float* tn = sm + l.tn;  // [5][kTC][Nh]: d_dnu, d_dth, da, domega, dsd per (t, n)
  // Per-mode state of the threads kT/2 + n: carry conj(lam_{t+1}) G_{t+1} and the
  // parameter sums over time.
  const int nthr = tid - kT / 2;
  const bool mode_thr = nthr >= 0 && nthr < Nh;
  float2 carry = make_float2(0.f, 0.f);
  float acc_a = 0.f, acc_om = 0.f, acc_sd = 0.f;

  for (int k = p.nchunks - 1; k >= 0; --k) {
    const int t0 = k * kTC, nt = min(kTC, L - t0);
    __syncthreads();
    stage_chunk<BF16>(p, l, sm, s, h, t0, nt, true);
    __syncthreads();
    poles_and_drive(p, l, sm, nt, false);
    __syncthreads();
    // Recompute the chunk's states from its checkpoint (row 0 = state entering it).
    if (tid < Nh) {
      float2 hv = reinterpret_cast<const float2*>(p.ckpt)[((s * p.nchunks + k) * p.H + h) * Nh + tid];
      hs[tid] = hv;
      for (int t = 0; t < nt; ++t) {
        const float2 a = lam[t * Nh + tid], g = gn[t * Nh + tid], b = braw[t * Nh + tid];
        const float ur = g.x * b.x - g.y * b.y, ui = g.x * b.y + g.y * b.x;
        const float nr = fmaf(a.x, hv.x, fmaf(-a.y, hv.y, ur));
        const float ni = fmaf(a.x, hv.y, fmaf(a.y, hv.x, ui));
        hv = make_float2(nr, ni);
        hs[(t + 1) * Nh + tid] = hv;
      }
    }
    __syncthreads();
    // Rank read and its adjoint per (t, r).
    if (R > 0) {
      for (int i = tid; i < nt * R; i += kT) {
        const int t = i / R, r = i % R;
        const float* cr = sm + l.ct + (t * R + r) * 2 * Nh;
        float rd = 0.f;
        for (int n = 0; n < Nh; ++n) {
          const float2 hv = hs[(t + 1) * Nh + n];
          rd = fmaf(cr[n], hv.x, fmaf(-cr[Nh + n], hv.y, rd));
        }
        float dyc = 0.f;
        for (int f = 0; f < Fh; ++f) dyc = fmaf(sm[l.dys + t * Fh + f], sm[l.Co + r * Fh + f], dyc);
        const float scv = sm[l.sc + i];
        sm[l.sr + i] = scv * rd;
        sm[l.dr + i] = scv * dyc;
        st<BF16>(p.dproj, (s * p.L + t0 + t) * p.P + cols.sc + r, rd * dyc);
      }
      __syncthreads();
    }
    // Readout adjoint g[t][n] = dL/dh_t (conjugate convention), and d c_t.
    {
      const float2* Cf = reinterpret_cast<const float2*>(sm + l.Cf);
      for (int i = tid; i < nt * Nh; i += kT) {
        const int t = i / Nh, n = i % Nh;
        const float2 hv = hs[(t + 1) * Nh + n];
        float gr = 0.f, gi = 0.f, e = 0.f;
        const float* dyr = sm + l.dys + t * Fh;
        for (int f = 0; f < Fh; ++f) {
          const float2 c = Cf[f * Nh + n];
          gr = fmaf(dyr[f], c.x, gr);
          gi = fmaf(-dyr[f], c.y, gi);
          if (env) e = fmaf(dyr[f], sm[l.Ef + f * Nh + n], e);
        }
        if (env) {
          gr = fmaf(2.f * e, hv.x, gr);
          gi = fmaf(2.f * e, hv.y, gi);
        }
        for (int r = 0; r < R; ++r) {
          const float drv = sm[l.dr + t * R + r];
          const float* cr = sm + l.ct + (t * R + r) * 2 * Nh;
          gr = fmaf(drv, cr[n], gr);
          gi = fmaf(-drv, cr[Nh + n], gi);
          const int64_t row = (s * p.L + t0 + t) * p.P + cols.ct + (int64_t)r * 2 * Nh;
          st<BF16>(p.dproj, row + n, drv * hv.x);
          st<BF16>(p.dproj, row + Nh + n, -drv * hv.y);
        }
        gs[i] = make_float2(gr, gi);
      }
    }
    __syncthreads();
    // Adjoint scan per mode: G_t = g_t + carry, carry = conj(lam_t) G_t.
    if (mode_thr) {
      for (int t = nt - 1; t >= 0; --t) {
        const float2 g = gs[t * Nh + nthr], a = lam[t * Nh + nthr];
        const float Gr = g.x + carry.x, Gi = g.y + carry.y;
        gs[t * Nh + nthr] = make_float2(Gr, Gi);
        carry = make_float2(a.x * Gr + a.y * Gi, a.x * Gi - a.y * Gr);
      }
    }
    __syncthreads();
    // Through the gain and the pole, per (t, n).
    for (int i = tid; i < nt * Nh; i += kT) {
      const int t = i / Nh, n = i % Nh;
      const float a = sm[l.prm + n], om = sm[l.prm + Nh + n], sd = sm[l.prm + 2 * Nh + n];
      const float dnu = sm[l.dnu + t], dth = sm[l.dth + t];
      const MDisc d = mdisc(p.gain, a, om, sd, p.detune != 0, dnu, dth);
      const float2 G = gs[i], b = braw[i], hp = hs[t * Nh + n];
      // d raw drive = conj(gain) G; d gain = conj(raw drive) G.
      db[i] = make_float2(d.gr * G.x + d.gi * G.y, d.gr * G.y - d.gi * G.x);
      const float dgr = b.x * G.x + b.y * G.y, dgi = b.x * G.y - b.y * G.x;
      // d lam = G conj(h_{t-1}); P = nu dL/dnu, d_th = dL/d(angle).
      const float dlre = G.x * hp.x + G.y * hp.y, dlim = G.y * hp.x - G.x * hp.y;
      float P = dlre * d.lre + dlim * d.lim;
      const float d_th = dlim * d.lre - dlre * d.lim;
      float d_dnu = 0.f, da_extra = 0.f, dbase_extra = 0.f;
      if (p.gain == SEMX_GAIN_GAMMA) {
        const float nu2 = d.nu * d.nu;
        P -= ((1.f - nu2) >= 1e-6f) ? dgr * nu2 * d.rs : 0.f;
      } else if (p.gain == SEMX_GAIN_MAMBA) {
        d_dnu = dgr;
      } else if (p.gain == SEMX_GAIN_ZOH) {
        d_dnu = dgr * d.lre + dgi * d.lim;
        const float pr = dnu * d.lre - d.gr, pi = dnu * d.lim - d.gi;
        const float qr = (d.base * pi - a * pr) * d.inv_den;
        const float qi = -(a * pi + d.base * pr) * d.inv_den;
        da_extra = -(dgr * qr + dgi * qi);
        dbase_extra = dgi * qr - dgr * qi;
      }
      d_dnu += d_th * d.base - a * P;
      const float dbase = d_th * dnu + dbase_extra;
      tn[0 * kTC * Nh + i] = d_dnu;
      tn[1 * kTC * Nh + i] = p.detune ? dbase * sd : dbase;
      tn[2 * kTC * Nh + i] = da_extra - dnu * P;
      tn[3 * kTC * Nh + i] = dbase;
      tn[4 * kTC * Nh + i] = p.detune ? dbase * dth : 0.f;
    }
    __syncthreads();
    // Per-token sums over modes (dnu / dth columns) and per-mode sums over time.
    if (tid < nt) {
      float sn = 0.f, st_ = 0.f;
      for (int n = 0; n < Nh; ++n) {
        sn += tn[tid * Nh + n];
        st_ += tn[kTC * Nh + tid * Nh + n];
      }
      const int64_t row = (s * p.L + t0 + tid) * p.P;
      st<BF16>(p.dproj, row + cols.dnu, sn * p.rs * semx::softplus_grad(sm[l.raw + tid]));
      st<BF16>(p.dproj, row + cols.dth, st_);
    }
    if (mode_thr) {
      for (int t = nt - 1; t >= 0; --t) {
        acc_a += tn[2 * kTC * Nh + t * Nh + nthr];
        acc_om += tn[3 * kTC * Nh + t * Nh + nthr];
        acc_sd += tn[4 * kTC * Nh + t * Nh + nthr];
      }
    }
    // dx = B^H d(raw drive) + D dy per (t, f).
    {
      const float2* Bn = reinterpret_cast<const float2*>(sm + l.Bn);
      for (int i = tid; i < nt * Fh; i += kT) {
        const int t = i / Fh, f = i % Fh;
        float acc = sm[l.Dp + f] * sm[l.dys + i];
        for (int n = 0; n < Nh; ++n) {
          const float2 b = Bn[n * Fh + f], g = db[t * Nh + n];
          acc = fmaf(b.x, g.x, fmaf(b.y, g.y, acc));
        }
        p.dx[(s * p.L + t0 + t) * Fd + (int64_t)h * Fh + f] = acc;
      }
    }
    // Rank write: d s_b, d b_t.
    if (R > 0) {
      for (int i = tid; i < nt * R; i += kT) {
        const int t = i / R, r = i % R;
        float acc = 0.f;
        for (int n = 0; n < Nh; ++n) acc = fmaf(sm[l.bt + (t * R + r) * Nh + n], db[t * Nh + n].x, acc);
        st<BF16>(p.dproj, (s * p.L + t0 + t) * p.P + cols.sb + r, acc);
      }
      const int wb = R * Nh;
      for (int i = tid; i < nt * wb; i += kT) {
        const int t = i / wb, j = i % wb, r = j / Nh, n = j % Nh;
        st<BF16>(p.dproj, (s * p.L + t0 + t) * p.P + cols.bt + j, sm[l.sb + t * R + r] * db[t * Nh + n].x);
      }
    }
    // Parameter sums over the chunk (each item owned by one thread, fixed order in t).
    for (int i = tid; i < Nh * Fh; i += kT) {
      {  // dB[n, f] += x[t, f] d(raw drive)[t, n]
        const int n = i / Fh, f = i % Fh;
        float ar = 0.f, ai = 0.f;
        for (int t = 0; t < nt; ++t) {
          const float xv = sm[l.xs + t * Fh + f];
          const float2 g = db[t * Nh + n];
          ar = fmaf(xv, g.x, ar);
          ai = fmaf(xv, g.y, ai);
        }
        sm[l.acc + oB + 2 * i] += ar;
        sm[l.acc + oB + 2 * i + 1] += ai;
      }
      {  // dC[f, n] += dy[t, f] (h_re, -h_im)[t, n]; denv[f, n] += dy |h|^2
        const int f = i / Nh, n = i % Nh;
        float ar = 0.f, ai = 0.f, ae = 0.f;
        for (int t = 0; t < nt; ++t) {
          const float dv = sm[l.dys + t * Fh + f];
          const float2 hv = hs[(t + 1) * Nh + n];
          ar = fmaf(dv, hv.x, ar);
          ai = fmaf(-dv, hv.y, ai);
          if (env) ae = fmaf(dv, hv.x * hv.x + hv.y * hv.y, ae);
        }
        sm[l.acc + oC + 2 * i] += ar;
        sm[l.acc + oC + 2 * i + 1] += ai;
        if (env) sm[l.acc + oE + i] += ae;
      }
    }
    for (int i = tid; i < R * Fh + Fh; i += kT) {
      float acc = 0.f;
      if (i < R * Fh) {  // dcout[r, f] += s_c read dy
        const int r = i / Fh, f = i % Fh;
        for (int t = 0; t < nt; ++t) acc = fmaf(sm[l.sr + t * R + r], sm[l.dys + t * Fh + f], acc);
        sm[l.acc + oO + i] += acc;
      } else {  // dD[f] += dy x
        const int f = i - R * Fh;
        for (int t = 0; t < nt; ++t) acc = fmaf(sm[l.dys + t * Fh + f], sm[l.xs + t * Fh + f], acc);
        sm[l.acc + oD + f] += acc;
      }
    }
  }
  __syncthreads();
  // Partial row of sequence s, parameter-major so every segment is in output order:
  // [dB | dC | denv | dcout | dD | dA_log | domega | ddetune], each over all heads.
  {
    const int64_t H = p.H;
    float* row = p.part + s * p.K;
    int64_t off = 0;
    auto put = [&](int64_t seg_per_head, int src, int cnt) {
      for (int i = tid; i < cnt; i += kT) row[off + (int64_t)h * seg_per_head + i] = sm[l.acc + src + i];
      off += H * seg_per_head;
    };
    put(Nh * Fh * 2, oB, Nh * Fh * 2);
    put(Fh * Nh * 2, oC, Fh * Nh * 2);
    if (env) put(Fh * Nh, oE, Fh * Nh);
    if (R > 0) put(R * Fh, oO, R * Fh);
    put(Fh, oD, Fh);
    if (mode_thr) {
      row[off + (int64_t)h * Nh + nthr] = acc_a * sm[l.prm + nthr];  // d/dA_log = a d/da
      row[off + H * Nh + (int64_t)h * Nh + nthr] = acc_om;
      row[off + 2 * H * Nh + (int64_t)h * Nh + nthr] = acc_sd;
    }
  }
}

// ------------------------------------------------------------------------ host side
int64_t proj_width(const SemxMimoLayerArgs* a) {
  return 2 * a->H + (a->rank > 0 ? 2 * a->H * a->rank + 3 * a->H * a->rank * a->Nh : 0);
}

int64_t part_row(const SemxMimoLayerArgs* a) {
  const int64_t H = a->H, Nh = a->Nh, Fh = a->Fh, R = a->rank;
  return H * (4 * Nh * Fh + (a->envelope ? Fh * Nh : 0) + R * Fh + Fh + 3 * Nh);
}

size_t layer_smem(const SemxMimoLayerArgs* a, bool bwd) {
  return (size_t)make_lay((int)a->Nh, (int)a->Fh, a->rank, bwd, a->envelope != 0).total * sizeof(float);
}

int layer_validate(const SemxMimoLayerArgs* a, bool bwd) {
  SEMX_REQUIRE(a->S >= 0 && a->L >= 0 && a->H >= 0 && a->Nh >= 0 && a->Fh >= 0 && a->rank >= 0,
               SEMX_ERR_SHAPE, "mimo_layer: negative size");
  SEMX_REQUIRE(a->Nh <= kMaxNh && a->Fh <= kMaxFh && a->rank <= kMaxR, SEMX_ERR_UNSUPPORTED,
               "mimo_layer: Nh=%lld (max %d), Fh=%lld (max %d), rank=%d (max %d)", (long long)a->Nh,
               kMaxNh, (long long)a->Fh, kMaxFh, a->rank, kMaxR);
  SEMX_REQUIRE(a->input_gain >= SEMX_GAIN_GAMMA && a->input_gain <= SEMX_GAIN_NONE, SEMX_ERR_UNSUPPORTED,
               "mimo_layer: input_gain=%d", a->input_gain);
  SEMX_REQUIRE(a->S * a->H <= 0x7fffffffLL, SEMX_ERR_SHAPE, "mimo_layer: S*H too large");
  const size_t smem = layer_smem(a, bwd);
  SEMX_REQUIRE(smem <= 227 * 1024, SEMX_ERR_UNSUPPORTED,
               "mimo_layer: head of Nh=%lld, Fh=%lld, rank=%d needs %zu B of shared memory",
               (long long)a->Nh, (long long)a->Fh, a->rank, smem);
  if (a->S * a->H > 0) {
    SEMX_REQUIRE(a->A_log && a->omega && a->B && a->C && a->D, SEMX_ERR_NULL,
                 "mimo_layer: NULL parameter");
    SEMX_REQUIRE(!a->detune || a->detune_gain, SEMX_ERR_NULL, "mimo_layer: detune_gain is NULL");
    SEMX_REQUIRE(!a->envelope || a->env_gain, SEMX_ERR_NULL, "mimo_layer: env_gain is NULL");
    SEMX_REQUIRE(a->rank == 0 || a->c_out, SEMX_ERR_NULL, "mimo_layer: c_out is NULL");
    SEMX_REQUIRE(semx::aligned(a->B, 8) && semx::aligned(a->C, 8), SEMX_ERR_ALIGN,
                 "mimo_layer: B and C must be 8-byte aligned");
  }
  if (a->S * a->L * a->H > 0) {
    SEMX_REQUIRE(a->x && a->proj, SEMX_ERR_NULL, "mimo_layer: x/proj is NULL");
    if (!bwd) SEMX_REQUIRE(a->y, SEMX_ERR_NULL, "mimo_layer: y is NULL");
    if (bwd) {
      SEMX_REQUIRE(a->ckpt && a->dy && a->dx && a->dproj, SEMX_ERR_NULL,
                   "mimo_layer bwd: ckpt/dy/dx/dproj is NULL");
    }
    SEMX_REQUIRE(!a->ckpt || semx::aligned(a->ckpt, 8), SEMX_ERR_ALIGN, "mimo_layer: ckpt alignment");
  }
  return SEMX_OK;
}

LParams to_lparams(const SemxMimoLayerArgs* a) {
  LParams p = {};
  p.S = a->S; p.L = a->L; p.H = a->H; p.Nh = a->Nh; p.Fh = a->Fh; p.R = a->rank;
  p.P = proj_width(a);
  p.gain = a->input_gain;
  p.detune = a->detune ? 1 : 0;
  p.envelope = a->envelope ? 1 : 0;
  p.nchunks = (int)semx::cdiv(a->L, kTC);
  p.rs = a->rate_scale;
  p.x = a->x; p.proj = a->proj;
  p.A_log = a->A_log; p.omega = a->omega; p.sdet = a->detune_gain; p.B = a->B; p.C = a->C; p.D = a->D;
  p.cout = a->c_out; p.env = a->env_gain;
  p.y = a->y; p.ckpt = a->ckpt; p.dy = a->dy; p.dx = a->dx; p.dproj = a->dproj;
  p.K = part_row(a);
  return p;
}

template <typename K>
int launch_layer(K kern, const LParams& p, size_t smem, cudaStream_t st, const char* name) {
  if (!semx::allow_smem(kern, smem)) return SEMX_ERR_LAUNCH;
  kern<<<(unsigned)(p.S * p.H), kT, smem, st>>>(p);
  return semx::check_launch(name);
}

}  // namespace

extern "C" {

size_t semx_mimo_layer_args_size(void) { return sizeof(SemxMimoLayerArgs); }

size_t semx_mimo_layer_ckpt_bytes(const SemxMimoLayerArgs* a) {
  if (a == nullptr || a->S < 0 || a->L < 0 || a->H < 0 || a->Nh < 0) return 0;
  return (size_t)a->S * (size_t)semx::cdiv(a->L, kTC) * (size_t)(a->H * a->Nh) * 2 * sizeof(float);
}

size_t semx_mimo_layer_workspace_bytes(const SemxMimoLayerArgs* a) {
  if (a == nullptr || a->S < 0 || a->H < 0 || a->Nh < 0 || a->Fh < 0 || a->rank < 0) return 0;
  const int64_t K = part_row(a);
  return ((size_t)a->S * K + semx::colsum_group_floats(a->S, K)) * sizeof(float);
}

int semx_mimo_layer_fwd(const SemxMimoLayerArgs* a, semx_stream_t stream) {
  SEMX_CHECK_ARGS(a, SemxMimoLayerArgs);
  int rc = layer_validate(a, false);
  if (rc != SEMX_OK) return rc;
  if (a->S * a->H == 0 || a->L == 0) return SEMX_OK;
  rc = semx::bind_device({a->y});
  if (rc != SEMX_OK) return rc;
  const LParams p = to_lparams(a);
  const size_t smem = layer_smem(a, false);
  cudaStream_t st = semx::as_stream(stream);
  return a->bf16 ? launch_layer(mimo_layer_fwd_kernel<true>, p, smem, st, "mimo_layer_fwd_kernel")
                 : launch_layer(mimo_layer_fwd_kernel<false>, p, smem, st, "mimo_layer_fwd_kernel");
}

int semx_mimo_layer_bwd(const SemxMimoLayerArgs* a, semx_stream_t stream) {
  SEMX_CHECK_ARGS(a, SemxMimoLayerArgs);
  int rc = layer_validate(a, true);
  if (rc != SEMX_OK) return rc;
  if (a->S * a->H == 0) return SEMX_OK;
  SEMX_REQUIRE(a->workspace != nullptr, SEMX_ERR_WORKSPACE, "mimo_layer bwd: workspace is NULL");
  rc = semx::bind_device({a->workspace});
  if (rc != SEMX_OK) return rc;
  cudaStream_t st = semx::as_stream(stream);
  LParams p = to_lparams(a);
  float* ws = reinterpret_cast<float*>(a->workspace);
  p.part = ws;
  if (a->L > 0) {
    const size_t smem = layer_smem(a, true);
    rc = a->bf16 ? launch_layer(mimo_layer_bwd_kernel<true>, p, smem, st, "mimo_layer_bwd_kernel")
                 : launch_layer(mimo_layer_bwd_kernel<false>, p, smem, st, "mimo_layer_bwd_kernel");
    if (rc != SEMX_OK) return rc;
  } else {
    cudaMemsetAsync(ws, 0, (size_t)a->S * p.K * sizeof(float), st);
  }
  const int64_t H = a->H, Nh = a->Nh, Fh = a->Fh, R = a->rank;
  semx::Segments seg = {};
  int n = 0;
  auto add = [&](float* out, int64_t len) {
    seg.out[n] = out;
    seg.len[n] = len;
    ++n;
  };
  add(a->dB, H * Nh * Fh * 2);
  add(a->dC, H * Fh * Nh * 2);
  if (a->envelope) add(a->denv, H * Fh * Nh);
  if (R > 0) add(a->dc_out, H * R * Fh);
  add(a->dD, H * Fh);
  add(a->dA_log, H * Nh);
  add(a->domega, H * Nh);
  add(a->detune ? a->ddetune : nullptr, H * Nh);
  seg.n = n;
  return semx::colsum(ws, a->S, p.K, ws + (size_t)a->S * p.K, seg, st);
}

}  // extern "C"
