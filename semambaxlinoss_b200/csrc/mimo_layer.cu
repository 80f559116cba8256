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
//               (B x)[n] + sum_r s_b[r] b_t[r,n], gained drive;
//            2. per mode n (one thread each): h_t = lam h_{t-1} + Bu over the chunk;
//            3. per (t, r): the rank read s_c Re(<c_t, h>);
//            4. per (t, f): y = Re(C h) + D x + <env, |h|^2> + rank feedthrough.
//   backward (chunks last first) recomputes 1-2 from the chunk's checkpoint, forms the
//            readout adjoint g per (t, n), runs G_t = g_t + conj(lam_{t+1}) G_{t+1} per
//            mode, and back-propagates through the gain, the pole and the drive. Token
//            gradients (dx, dproj) are written directly; parameter gradients are summed
//            per CTA in a fixed order, written as per-sequence partial rows and reduced
//            over sequences by the two-stage column sum.
// The static drive (B x)[n] of every head is a column pair of the projection rows: the
// block-diagonal B is part of the input projection GEMM, so its forward product, its
// x-gradient B^H d(drive) and its weight gradient run on the tensor cores in that GEMM
// and its backward, and the layer kernels read and write the drive columns like the
// other token operands (dproj of the drive = d(raw drive)).
// Every parallel loop distributes (t, n) or (t, f) items so that a warp's shared-memory
// reads of the per-head matrices are consecutive (both storage orders of C and env_gain
// are kept where both access orders occur).
#include <cuda_bf16.h>

#include <type_traits>

#include "semx_common.cuh"
#include "semx_math.cuh"
#include "semx_reduce.cuh"
#include "semx_tc.cuh"

namespace {

constexpr int kT = 128;   // threads per CTA
constexpr int kTC = 32;   // tokens per chunk
constexpr int kCk = 16;   // tokens per checkpoint
constexpr int kMaxNh = 64;
constexpr int kMaxFh = 256;
constexpr int kMaxR = 16;
constexpr float kLog2e = 1.4426950408889634f;

struct LParams {
  int64_t S, L, H, Nh, Fh, R, P;  // P = projection row width
  int gain, detune, envelope, nchunks;
  int nck;  // checkpoints: one per kCk tokens
  int vec;  // 16-byte aligned rows: bit 0 x, bit 1 b_t / c_t, bit 2 dy, bit 3 dx,
            // bit 4 the drive columns (proj and dproj), bit 5 the b_t / c_t columns of dproj
  float rs;
  const void* x;
  const void* proj;
  const float* A_log;
  const float* omega;
  const float* sdet;
  const float* C;
  const float* D;
  const float* cout;
  const float* env;
  const float* dtb;  // [b_nu (H) | b_th (H)] added to the dnu_raw / dth columns, or null
  float* y;
  float* ckpt;
  const float* dy;
  void* dx;          // the dtype of x
  void* dproj;
  float* part;  // (S, K) partial parameter-gradient rows
  int64_t K;
};

// Shared-memory layout in floats (every offset a multiple of 4).
struct Lay {
  int Cn, Cf, En, Ef, Co, Dp, prm;
  int xs, bx, raw, dnu, dth, sb, bt, sc, ct;
  int lam, gn, bu, hs, sr;
  int dys, dr, gs, db, tn, acc, rb;
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
  l.Cn = take(Nh * Fh * 2);
  l.Cf = bwd ? take(Fh * Nh * 2) : -1;
  l.En = env ? take(Nh * Fh) : -1;
  l.Ef = (env && bwd) ? take(Fh * Nh) : -1;
  l.Co = take(R * Fh);
  l.Dp = take(Fh);
  l.prm = take(3 * Nh);
  l.xs = take(kTC * Fh);
  l.bx = take(kTC * Nh * 2);
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
    l.acc = take(Fh * Nh * 2 + (env ? Fh * Nh : 0) + R * Fh + Fh);
    l.rb = take(2 * kTC);
  } else {
    l.dys = l.dr = l.gs = l.db = l.tn = l.acc = l.rb = -1;
  }
  l.total = o;
  return l;
}

// Column offsets of head h's operands in a projection row.
struct Cols {
  int64_t dnu, dth, sb, bt, sc, ct, bx;
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
  c.bx = 2 * H + 2 * H * R + 3 * H * R * Nh + (int64_t)h * 2 * Nh;
  return c;
}

// The dt_nu / dt_theta biases of head h (zero without them).
__device__ __forceinline__ float2 dt_bias(const LParams& p, int h) {
  return p.dtb ? make_float2(p.dtb[h], p.dtb[p.H + h]) : make_float2(0.f, 0.f);
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
  const float2 bias = dt_bias(p, h);
  for (int t = threadIdx.x; t < nt; t += kT) {
    const int64_t row = (s * p.L + t0 + t) * p.P;
    const float raw = ld<BF16>(p.proj, row + c.dnu) + bias.x;
    sm[l.raw + t] = raw;
    sm[l.dnu + t] = semx::softplus(raw) * p.rs;
    sm[l.dth + t] = ld<BF16>(p.proj, row + c.dth) + bias.y;
  }
  for (int i = threadIdx.x; i < nt * 2 * Nh; i += kT) {
    const int t = i / (2 * Nh), j = i % (2 * Nh);
    sm[l.bx + i] = ld<BF16>(p.proj, (s * p.L + t0 + t) * p.P + c.bx + j);
  }
  if (R > 0) {
    for (int i = threadIdx.x; i < nt * R; i += kT) {
      const int t = i / (R > 0 ? R : 1), r = i % (R > 0 ? R : 1);
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
  const int Nh = (int)p.Nh, R = (int)p.R;
  const float2* bx = reinterpret_cast<const float2*>(sm + l.bx);
  for (int i = threadIdx.x; i < nt * Nh; i += kT) {
    const int t = i / Nh, n = i % Nh;
    const MDisc d = mdisc(p.gain, sm[l.prm + n], sm[l.prm + Nh + n], sm[l.prm + 2 * Nh + n],
                          p.detune != 0, sm[l.dnu + t], sm[l.dth + t]);
    float br = bx[i].x;
    const float bi = bx[i].y;
    for (int r = 0; r < R; ++r) br = fmaf(sm[l.sb + t * R + r], sm[l.bt + (t * R + r) * Nh + n], br);
    reinterpret_cast<float2*>(sm + l.lam)[i] = make_float2(d.lre, d.lim);
    reinterpret_cast<float2*>(sm + l.gn)[i] = make_float2(d.gr, d.gi);
    reinterpret_cast<float2*>(sm + l.bu)[i] =
        gained ? make_float2(d.gr * br - d.gi * bi, d.gr * bi + d.gi * br) : make_float2(br, bi);
  }
}

// ----------------------------------------------------------------------------- forward
// Shared-memory layout of the forward (floats; staging buffers hold the input dtype).
struct FLay {
  int Cr, Ci, En, Co, Dp, prm, cin;
  int stg[2], sml[2];  // staged x | drive | b_t | c_t (input dtype); small operands (fp32)
  int lam, bu, hs, sr;
  int xw, bxw, btw, ctw;  // staged row widths in elements; x, b_t and c_t rows are padded
                          // so rows two tokens apart fall in different shared-memory banks
                          // (drive rows are read two consecutive tokens per warp and are
                          // not padded)
  int hw;              // row width of lam / bu / hs in float2 (Nh + 1, same reason)
  int tc;              // tokens per chunk
  int total;
};

__host__ __device__ inline FLay make_flay(int Nh, int Fh, int R, bool env, int es, int tc = kTC) {
  FLay l = {};
  l.tc = tc;
  int o = 0;
  auto take = [&](int n) {
    const int at = o;
    o += al4(n);
    return at;
  };
  l.Cr = take(Nh * Fh);
  l.Ci = take(Nh * Fh);
  l.En = env ? take(Nh * Fh) : -1;
  l.Co = take(R * Fh);
  l.Dp = take(Fh);
  l.prm = take(3 * Nh);
  l.cin = take(Nh * 2);
  const int pad = 16 / es;
  l.xw = ((Fh * es + 15) / 16) * 16 / es + pad;
  l.bxw = ((2 * Nh * es + 15) / 16) * 16 / es;
  l.btw = R > 0 ? ((R * Nh * es + 15) / 16) * 16 / es + pad : 0;
  l.ctw = R > 0 ? ((2 * R * Nh * es + 15) / 16) * 16 / es + pad : 0;
  const int stg_elems = tc * (l.xw + l.bxw + l.btw + l.ctw);
  for (int b = 0; b < 2; ++b) l.stg[b] = take((stg_elems * es + 3) / 4);
  for (int b = 0; b < 2; ++b) l.sml[b] = take(tc * (3 + 2 * R));
  l.hw = Nh + 1;
  l.lam = take(tc * l.hw * 2);
  l.bu = take(tc * l.hw * 2);
  l.hs = take(tc * l.hw * 2);
  l.sr = take(tc * R);
  l.total = o;
  return l;
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }

// Copies rows [t0, t0 + nt) of one column segment (width elements at column col of rows
// row_stride apart) into d (rows dw elements apart).
template <typename T>
__device__ __forceinline__ void stage_segment(T* d, int dw, const T* src, int64_t row0, int64_t row_stride,
                                              int64_t col, int width, int nt, bool vec) {
  constexpr int kPer = 16 / sizeof(T);
  if (vec) {
    const int q = width / kPer;
    for (int i = threadIdx.x; i < nt * q; i += kT) {
      const int t = i / q, j = i - (i / q) * q;
      cp_async16(d + t * dw + j * kPer, src + (row0 + t) * row_stride + col + j * kPer);
    }
  } else {
    for (int i = threadIdx.x; i < nt * width; i += kT) {
      const int t = i / width, j = i - (i / width) * width;
      d[t * dw + j] = src[(row0 + t) * row_stride + col + j];
    }
  }
}

// Issues the staging of chunk [t0, t0 + nt) of head h: x [tc][Fh], drive [tc][2 Nh],
// b_t [tc][R Nh], c_t [tc][2 R Nh] in the input dtype, rows l.xw / l.bxw / l.btw /
// l.ctw apart; 16-byte cp.async where the host found the rows aligned (p.vec bit 0: x,
// bit 1: b_t and c_t, bit 4: drive), otherwise plain loads.
template <bool BF16, int NH, int FH, int RK>
__device__ __forceinline__ void stage_bulk(const LParams& p, const FLay& l, void* dst, int64_t s, int h,
                                           int t0, int nt) {
  using T = typename std::conditional<BF16, __nv_bfloat16, float>::type;
  const int Nh = NH > 0 ? NH : (int)p.Nh, Fh = FH > 0 ? FH : (int)p.Fh, R = RK >= 0 ? RK : (int)p.R;
  T* xs = reinterpret_cast<T*>(dst);
  T* bxs = xs + l.tc * l.xw;
  T* bts = bxs + l.tc * l.bxw;
  T* cts = bts + l.tc * l.btw;
  const T* X = reinterpret_cast<const T*>(p.x);
  const T* Pj = reinterpret_cast<const T*>(p.proj);
  const int64_t row0 = s * p.L + t0;
  const Cols c = cols_of(p, h);
  stage_segment<T>(xs, l.xw, X, row0, p.H * p.Fh, (int64_t)h * Fh, Fh, nt, (p.vec & 1) != 0);
  stage_segment<T>(bxs, l.bxw, Pj, row0, p.P, c.bx, 2 * Nh, nt, (p.vec & 16) != 0);
  if (R > 0) {
    stage_segment<T>(bts, l.btw, Pj, row0, p.P, c.bt, R * Nh, nt, (p.vec & 2) != 0);
    stage_segment<T>(cts, l.ctw, Pj, row0, p.P, c.ct, 2 * R * Nh, nt, (p.vec & 2) != 0);
  }
}

// Small per-token operands [dnu_raw, dth, s_b (R), s_c (R)] of chunk [t0, t0 + nt): item q
// of this thread is i = tid + q kT over nt (2 + 2R) values.
constexpr int kPre = 9;
template <bool BF16, int RK>
__device__ __forceinline__ void load_small(const LParams& p, int64_t s, int h, int t0, int nt, float2 bias,
                                           float (&pre)[kPre]) {
  const int R = RK >= 0 ? RK : (int)p.R, w = 2 + 2 * R;
  const Cols c = cols_of(p, h);
#pragma unroll
  for (int q = 0; q < kPre; ++q) {
    const int i = threadIdx.x + q * kT;
    if (i < nt * w) {
      const int t = i / w, j = i % w;
      const int64_t col = j == 0 ? c.dnu : j == 1 ? c.dth : j < 2 + R ? c.sb + (j - 2) : c.sc + (j - 2 - R);
      pre[q] = ld<BF16>(p.proj, (s * p.L + t0 + t) * p.P + col) + (j == 0 ? bias.x : j == 1 ? bias.y : 0.f);
    }
  }
}
// Writes them as [raw (CT) | dnu (CT) | dth (CT) | s_b (CT R) | s_c (CT R)] for a chunk of
// CT tokens.
template <int RK, int CT = kTC>
__device__ __forceinline__ void store_small(const LParams& p, float* sml, int nt, const float (&pre)[kPre]) {
  const int R = RK >= 0 ? RK : (int)p.R, w = 2 + 2 * R;
#pragma unroll
  for (int q = 0; q < kPre; ++q) {
    const int i = threadIdx.x + q * kT;
    if (i < nt * w) {
      const int t = i / w, j = i % w;
      if (j == 0) {
        sml[t] = pre[q];
        sml[CT + t] = semx::softplus(pre[q]) * p.rs;
      } else if (j == 1) {
        sml[2 * CT + t] = pre[q];
      } else if (j < 2 + R) {
        sml[3 * CT + t * R + (j - 2)] = pre[q];
      } else {
        sml[3 * CT + CT * R + t * R + (j - 2 - R)] = pre[q];
      }
    }
  }
}

// Four consecutive staged values (8-byte aligned for bf16, 16-byte aligned for fp32).
__device__ __forceinline__ float4 ld4(const __nv_bfloat16* q) {
  const uint2 u = *reinterpret_cast<const uint2*>(q);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ float4 ld4(const float* q) { return *reinterpret_cast<const float4*>(q); }
// Two consecutive staged values (4-byte aligned for bf16, 8-byte aligned for fp32).
__device__ __forceinline__ float2 ld2(const __nv_bfloat16* q) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(q));
}
__device__ __forceinline__ float2 ld2(const float* q) { return *reinterpret_cast<const float2*>(q); }

__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
  return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}

// Scan of the chunk: h_t = lam_t h_{t-1} + bu_t from cin[n]; writes hs[t][n] and the
// chunk's final state back to cin[n]. With SEG > 1 (Nh * SEG == kT), thread (n, seg)
// composes kTC / SEG steps, the segments are combined by an inclusive shuffle scan of the
// affine maps, and each segment is replayed from its entry state; SEG == 1 runs one
// thread per mode over the whole chunk.
// Rows of lam / bu / hs are hw float2 apart. Lanes are segment-major inside a warp
// (lane = seg * (32 / SEG) + mode), so the shuffles step by 32 / SEG lanes and the
// shared-memory rows touched by one instruction fall in distinct banks.
// chunk_scan_to: the same scan with each state h_t of mode n handed to store(t, n, h_t).
template <int SEG, int CT, typename Store>
__device__ __forceinline__ void chunk_scan_to(const float2* lam, const float2* bu, float2* cin, int Nh, int hw,
                                              int nt, Store store);

template <int SEG, int CT = kTC>
__device__ __forceinline__ void chunk_scan(const float2* lam, const float2* bu, float2* hs, float2* cin,
                                           int Nh, int hw, int nt) {
  chunk_scan_to<SEG, CT>(lam, bu, cin, Nh, hw, nt, [&](int t, int n, float2 v) { hs[t * hw + n] = v; });
}

template <int SEG, int CT, typename Store>
__device__ __forceinline__ void chunk_scan_to(const float2* lam, const float2* bu, float2* cin, int Nh, int hw,
                                              int nt, Store store) {
  if (SEG == 1) {
    const int n = threadIdx.x;
    if (n < Nh) {
      float2 st = cin[n];
      for (int t = 0; t < nt; ++t) {
        st = cmul(lam[t * hw + n], st);
        st.x += bu[t * hw + n].x;
        st.y += bu[t * hw + n].y;
        store(t, n, st);
      }
      cin[n] = st;
    }
    return;
  }
  constexpr int TS = CT / SEG;
  constexpr int MPW = 32 / SEG;  // modes per warp
  const int lane = threadIdx.x & 31;
  const int n = (threadIdx.x >> 5) * MPW + lane % MPW, seg = lane / MPW;
  const int t0 = seg * TS;
  float2 A = make_float2(1.f, 0.f), b = make_float2(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < TS; ++i) {
    const int t = t0 + i;
    if (t < nt) {
      const float2 a = lam[t * hw + n];
      b = cmul(a, b);
      b.x += bu[t * hw + n].x;
      b.y += bu[t * hw + n].y;
      A = cmul(a, A);
    }
  }
  // Inclusive scan over the segments of mode n: (A, b) after (Ap, bp) = (A Ap, A bp + b).
#pragma unroll
  for (int off = 1; off < SEG; off <<= 1) {
    const float apr = __shfl_up_sync(0xffffffffu, A.x, off * MPW);
    const float api = __shfl_up_sync(0xffffffffu, A.y, off * MPW);
    const float bpr = __shfl_up_sync(0xffffffffu, b.x, off * MPW);
    const float bpi = __shfl_up_sync(0xffffffffu, b.y, off * MPW);
    if (seg >= off) {
      const float2 nb = cmul(A, make_float2(bpr, bpi));
      b = make_float2(nb.x + b.x, nb.y + b.y);
      A = cmul(A, make_float2(apr, api));
    }
  }
  const float2 c0 = cin[n];
  // Entry state of this segment: the inclusive map of the previous segment applied to c0.
  const float epr = __shfl_up_sync(0xffffffffu, A.x, MPW);
  const float epi = __shfl_up_sync(0xffffffffu, A.y, MPW);
  const float ebr = __shfl_up_sync(0xffffffffu, b.x, MPW);
  const float ebi = __shfl_up_sync(0xffffffffu, b.y, MPW);
  float2 st = c0;
  if (seg > 0) {
    st = cmul(make_float2(epr, epi), c0);
    st.x += ebr;
    st.y += ebi;
  }
#pragma unroll
  for (int i = 0; i < TS; ++i) {
    const int t = t0 + i;
    if (t < nt) {
      st = cmul(lam[t * hw + n], st);
      st.x += bu[t * hw + n].x;
      st.y += bu[t * hw + n].y;
      store(t, n, st);
    }
  }
  __syncwarp();
  if (seg == SEG - 1) {  // final state of the chunk: the last segment's map applied to c0
    const float2 e = cmul(A, c0);
    cin[n] = make_float2(e.x + b.x, e.y + b.y);
  }
}

// NH, FH, RK > 0 (RK >= 0) fix the head's modes, channels and rank at compile time;
// 0 (-1) takes them from the parameters. CT tokens per chunk (a multiple of the 16-token
// checkpoint interval): 16 for the 16-mode, 32-channel heads, whose 31 KB of shared memory
// then lets 7 CTAs share an SM; 32 otherwise.
template <bool BF16, int SEG, int NH, int FH, int RK, int CT = kTC>
__global__ void __launch_bounds__(kT) mimo_layer_fwd_kernel(const LParams p) {
  using T = typename std::conditional<BF16, __nv_bfloat16, float>::type;
  extern __shared__ float4 smem4[];
  float* sm = reinterpret_cast<float*>(smem4);
  const int Nh = NH > 0 ? NH : (int)p.Nh, Fh = FH > 0 ? FH : (int)p.Fh, R = RK >= 0 ? RK : (int)p.R;
  const int L = (int)p.L;
  const bool env = p.envelope != 0;
  static_assert(CT % kCk == 0 && CT % SEG == 0, "chunk must hold whole checkpoint blocks and segments");
  constexpr int CPC = CT / kCk;  // checkpoints per chunk
  const FLay l = make_flay(Nh, Fh, R, env, (int)sizeof(T), CT);
  const int nchunks = (L + CT - 1) / CT;
  const int64_t s = blockIdx.x / p.H;
  const int h = (int)(blockIdx.x % p.H);
  const int tid = threadIdx.x;
  const int64_t Fd = p.H * p.Fh;
  // Head parameters.
  for (int i = tid; i < Nh * Fh; i += kT) {
    const int f2 = i / Nh, n2 = i % Nh;
    const float2 cv = reinterpret_cast<const float2*>(p.C)[((int64_t)h * Fh + f2) * Nh + n2];
    sm[l.Cr + n2 * Fh + f2] = cv.x;
    sm[l.Ci + n2 * Fh + f2] = cv.y;
    if (env) sm[l.En + n2 * Fh + f2] = p.env[((int64_t)h * Fh + f2) * Nh + n2];
  }
  for (int i = tid; i < R * Fh; i += kT) sm[l.Co + i] = p.cout[(int64_t)h * R * Fh + i];
  for (int i = tid; i < Fh; i += kT) sm[l.Dp + i] = p.D[(int64_t)h * Fh + i];
  for (int n = tid; n < Nh; n += kT) {
    sm[l.prm + n] = expf(p.A_log[(int64_t)h * Nh + n]);
    sm[l.prm + Nh + n] = p.omega[(int64_t)h * Nh + n];
    sm[l.prm + 2 * Nh + n] = p.detune ? p.sdet[(int64_t)h * Nh + n] : 1.f;
    reinterpret_cast<float2*>(sm + l.cin)[n] = make_float2(0.f, 0.f);
  }
  float2* lam = reinterpret_cast<float2*>(sm + l.lam);
  float2* bu = reinterpret_cast<float2*>(sm + l.bu);
  float2* hs = reinterpret_cast<float2*>(sm + l.hs);
  float2* cin = reinterpret_cast<float2*>(sm + l.cin);
  const float* Cr = sm + l.Cr;
  const float* Ci = sm + l.Ci;
  const int hw = l.hw;
  const float2 bias = dt_bias(p, h);
  float pre[kPre];
  if (nchunks > 0) {
    const int nt0 = min(CT, L);
    stage_bulk<BF16, NH, FH, RK>(p, l, sm + l.stg[0], s, h, 0, nt0);
    load_small<BF16, RK>(p, s, h, 0, nt0, bias, pre);
    store_small<RK, CT>(p, sm + l.sml[0], nt0, pre);
  }
  cp_async_commit();
  for (int k = 0; k < nchunks; ++k) {
    const int b = k & 1;
    const int t0 = k * CT, nt = min(CT, L - t0);
    const int t0n = t0 + CT, ntn = min(CT, L - t0n);
    cp_async_wait_all();
    __syncthreads();
    if (k + 1 < nchunks) {
      stage_bulk<BF16, NH, FH, RK>(p, l, sm + l.stg[b ^ 1], s, h, t0n, ntn);
      load_small<BF16, RK>(p, s, h, t0n, ntn, bias, pre);
    }
    cp_async_commit();
    const T* xs = reinterpret_cast<const T*>(sm + l.stg[b]);
    const T* bxs = xs + CT * l.xw;
    const T* bts = bxs + CT * l.bxw;
    const T* cts = bts + CT * l.btw;
    const int xw = l.xw, bxw = l.bxw, btw = l.btw, ctw = l.ctw;
    const float* sml = sm + l.sml[b];
    const float* dnus = sml + CT;
    const float* dths = sml + 2 * CT;
    const float* sbs = sml + 3 * CT;
    const float* scs = sbs + CT * R;
    // Poles and gained drive per (token, mode).
    for (int i = tid; i < nt * Nh; i += kT) {
      const int t = i / Nh, n = i - (i / Nh) * Nh;
      const float2 bq = ld2(bxs + t * bxw + 2 * n);
      float rr = bq.x;
      const float bi = bq.y;
      for (int r = 0; r < R; ++r) rr = fmaf(sbs[t * R + r], static_cast<float>(bts[t * btw + r * Nh + n]), rr);
      const MDisc d = mdisc(p.gain, sm[l.prm + n], sm[l.prm + Nh + n], sm[l.prm + 2 * Nh + n],
                            p.detune != 0, dnus[t], dths[t]);
      lam[t * hw + n] = make_float2(d.lre, d.lim);
      bu[t * hw + n] = make_float2(d.gr * rr - d.gi * bi, d.gr * bi + d.gi * rr);
    }
    __syncthreads();
    if (p.ckpt != nullptr && tid < Nh)
      reinterpret_cast<float2*>(p.ckpt)[((s * p.nck + CPC * k) * p.H + h) * Nh + tid] = cin[tid];
    __syncthreads();
    chunk_scan<SEG, CT>(lam, bu, hs, cin, Nh, hw, nt);
    __syncthreads();
#pragma unroll
    for (int m = 1; m < CPC; ++m)  // the state entering token t0 + 16 m
      if (p.ckpt != nullptr && tid < Nh && t0 + m * kCk < L)
        reinterpret_cast<float2*>(p.ckpt)[((s * p.nck + CPC * k + m) * p.H + h) * Nh + tid] =
            hs[(m * kCk - 1) * hw + tid];
    if (R > 0) {
      for (int i = tid; i < nt * R; i += kT) {
        const int t = i / (R > 0 ? R : 1), r = i % (R > 0 ? R : 1);
        const T* cr = cts + t * ctw + r * 2 * Nh;
        float acc = 0.f;
        for (int n = 0; n < Nh; ++n) {
          const float2 hv = hs[t * hw + n];
          acc = fmaf(static_cast<float>(cr[n]), hv.x, fmaf(-static_cast<float>(cr[Nh + n]), hv.y, acc));
        }
        sm[l.sr + i] = scs[i] * acc;
      }
      __syncthreads();
    }
    // Readout, TPI tokens x 4 channels per item (one item per thread for 16 x 32 heads).
    constexpr int TPI = CT >= 32 ? 2 : 1;
    const int fq = (Fh + 3) / 4;
    for (int it = tid; it < (CT / TPI) * fq; it += kT) {
      const int ta = (it / fq) * TPI, fa = (it % fq) * 4;
      if (ta >= nt) continue;
      bool tok[TPI];
#pragma unroll
      for (int dt = 0; dt < TPI; ++dt) tok[dt] = ta + dt < nt;
      float acc[TPI][4];
#pragma unroll
      for (int dt = 0; dt < TPI; ++dt)
#pragma unroll
        for (int df = 0; df < 4; ++df) {
          const int f = min(fa + df, Fh - 1);
          const int t = min(ta + dt, nt - 1);
          acc[dt][df] = sm[l.Dp + f] * static_cast<float>(xs[t * xw + f]);
        }
#pragma unroll 4
      for (int n = 0; n < Nh; ++n) {
        float2 hv[TPI];
        float pw[TPI];
#pragma unroll
        for (int dt = 0; dt < TPI; ++dt) {
          hv[dt] = tok[dt] ? hs[(ta + dt) * hw + n] : make_float2(0.f, 0.f);
          pw[dt] = hv[dt].x * hv[dt].x + hv[dt].y * hv[dt].y;
        }
#pragma unroll
        for (int df = 0; df < 4; ++df) {
          const int f = min(fa + df, Fh - 1);
          const float cre = Cr[n * Fh + f], cim = Ci[n * Fh + f];
#pragma unroll
          for (int dt = 0; dt < TPI; ++dt) acc[dt][df] = fmaf(cre, hv[dt].x, fmaf(-cim, hv[dt].y, acc[dt][df]));
          if (env) {
            const float e = sm[l.En + n * Fh + f];
#pragma unroll
            for (int dt = 0; dt < TPI; ++dt) acc[dt][df] = fmaf(e, pw[dt], acc[dt][df]);
          }
        }
      }
      for (int r = 0; r < R; ++r) {
        float sv[TPI];
#pragma unroll
        for (int dt = 0; dt < TPI; ++dt) sv[dt] = tok[dt] ? sm[l.sr + (ta + dt) * R + r] : 0.f;
#pragma unroll
        for (int df = 0; df < 4; ++df) {
          const float co = sm[l.Co + r * Fh + min(fa + df, Fh - 1)];
#pragma unroll
          for (int dt = 0; dt < TPI; ++dt) acc[dt][df] = fmaf(sv[dt], co, acc[dt][df]);
        }
      }
#pragma unroll
      for (int dt = 0; dt < TPI; ++dt) {
        if (!tok[dt]) continue;
        float* yr = p.y + (s * p.L + t0 + ta + dt) * Fd + (int64_t)h * Fh + fa;
#pragma unroll
        for (int df = 0; df < 4; ++df)
          if (fa + df < Fh) yr[df] = acc[dt][df];
      }
    }
    if (k + 1 < nchunks) store_small<RK, CT>(p, sm + l.sml[b ^ 1], ntn, pre);
  }
}

// ------------------------------------------------- forward, tensor-core readout (bf16)
// The forward of 16-mode, 32-channel heads with bf16 operands and no envelope readout,
// with the readout Re(C h) on the tensor cores: the chunk scan writes each state straight
// into a 64-token A tile [h_re (16) | h_im (16)] (fp32, 128-byte swizzled, K-major); once
// four 16-token chunks are in, one thread issues four kind::tf32 MMAs (M 64, N 32, K 8
// each) against the B tile [C_re | -C_im] of the head, accumulating in tensor memory. The
// epilogue (D skip and rank feedthrough added, y stored) of a tile runs during the next
// chunk, after its poles, so the MMA never stalls the CTA. tf32 operands (10-bit mantissa)
// keep the readout well inside the bf16-input tolerance; the fp32 layer keeps the fp32
// CUDA-core readout of mimo_layer_fwd_kernel.
//
// Shared memory (floats, from a 1024-byte aligned base): A tile, B tile, head parameters,
// double-buffered unpadded staging of x / drive / b_t / c_t and of the small operands,
// poles and gained drive of a chunk, rank reads of a tile, the mbarrier and the
// tensor-memory address: 35.6 KB, 6 CTAs per SM.
constexpr int kTcM = 64;                    // tokens per tensor-core tile (the MMA's M)
constexpr uint32_t kTcWaitLimit = 1u << 22;  // mbarrier polls before a wait gives up
__device__ unsigned int g_tc_timeouts;       // waits that gave up (semx_tc_timeouts)

struct TcLay {
  static constexpr int at = 0;                        // 64 x 32 fp32, swizzled
  static constexpr int bt2 = at + kTcM * 32;          // 32 x 32 fp32, swizzled
  static constexpr int Co = bt2 + 32 * 32;            // c_out (4 x 32)
  static constexpr int Dp = Co + 4 * 32;              // D (32)
  static constexpr int prm = Dp + 32;                 // a, omega, detune (3 x 16)
  static constexpr int cin = prm + 48;                // chunk entry state (16 float2)
  static constexpr int stg_floats = 16 * (32 + 32 + 64 + 128) / 2;  // bf16 x | drive | b_t | c_t
  static constexpr int stg0 = cin + 32;
  static constexpr int stg1 = stg0 + stg_floats;
  static constexpr int sml_floats = 16 * (3 + 2 * 4);
  static constexpr int sml0 = stg1 + stg_floats;
  static constexpr int sml1 = sml0 + sml_floats;
  static constexpr int hw = 17;                       // lam / bu rows (float2)
  static constexpr int lam = sml1 + sml_floats;
  static constexpr int bu = lam + 16 * hw * 2;
  static constexpr int srk = bu + 16 * hw * 2;        // rank reads of the tile (64 x 4)
  static constexpr int bar = srk + kTcM * 4;          // 8-byte mbarrier
  static constexpr int tslot = bar + 2;               // tensor-memory address
  static constexpr int total = tslot + 2;
};
static_assert(TcLay::bt2 % 256 == 0 && TcLay::bar % 2 == 0, "tile / mbarrier alignment");

// Epilogue of the tile whose MMA was committed: lanes 0..15 of warp w <= last hold the rows
// of its chunk w (tensor-memory lanes 32 w + i); y = acc + D x + sum_r rank read_r c_out_r.
template <int RK>
__device__ __forceinline__ void tc_epilogue(const LParams& p, const float* sm, uint32_t taddr, int64_t s,
                                            int h, int tile_t0, int last, int L) {
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  if (w > last) return;  // warp-uniform
  const int64_t Fd = p.H * 32;
  const int j = 16 * w + lane, tg = tile_t0 + j;
  const bool live = lane < 16 && tg < L;
  uint4 xu[4];
  if (live) {
    const uint4* xg = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p.x) +
                                                     (s * p.L + tg) * Fd + (int64_t)h * 32);
#pragma unroll
    for (int c = 0; c < 4; ++c) xu[c] = __ldg(xg + c);
  }
  float acc[32];
  semx::tc::tmem_ld32(taddr + ((uint32_t)(32 * w) << 16), acc);
  if (!live) return;
  const __nv_bfloat16* xr = reinterpret_cast<const __nv_bfloat16*>(xu);
  float sv[RK > 0 ? RK : 1];
#pragma unroll
  for (int r = 0; r < RK; ++r) sv[r] = sm[TcLay::srk + j * 4 + r];
  float* yr = p.y + (s * p.L + tg) * Fd + (int64_t)h * 32;
#pragma unroll
  for (int f4 = 0; f4 < 8; ++f4) {
    const float4 xv = ld4(xr + 4 * f4);
    const float xa[4] = {xv.x, xv.y, xv.z, xv.w};
    float o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int f = 4 * f4 + e;
      o[e] = fmaf(sm[TcLay::Dp + f], xa[e], acc[f]);
#pragma unroll
      for (int r = 0; r < RK; ++r) o[e] = fmaf(sv[r], sm[TcLay::Co + r * 32 + f], o[e]);
    }
    *reinterpret_cast<float4*>(yr + 4 * f4) = make_float4(o[0], o[1], o[2], o[3]);
  }
}

template <int RK>
__global__ void __launch_bounds__(kT, 6) mimo_layer_fwd_tc_kernel(const LParams p) {
  using T = __nv_bfloat16;
  constexpr int NH = 16, FH = 32, CT = 16, SEG = 8, R = RK, hw = TcLay::hw;
  extern __shared__ __align__(1024) float4 smem4[];
  float* sm = reinterpret_cast<float*>(smem4);
  const int L = (int)p.L;
  const int nchunks = (L + CT - 1) / CT;
  const int64_t s = blockIdx.x / p.H;
  const int h = (int)(blockIdx.x % p.H);
  const int tid = threadIdx.x;
  // The staging helpers read the row widths of an FLay: unpadded rows here.
  FLay l = {};
  l.tc = CT;
  l.xw = FH;
  l.bxw = 2 * NH;
  l.btw = R * NH;
  l.ctw = 2 * R * NH;
  // The tiles' swizzle pattern assumes a 1024-byte aligned base (declared above); a
  // misaligned base is counted like a timed-out wait and the CTA writes nothing.
  if ((semx::tc::smem_addr(smem4) & 1023u) != 0) {
    if (tid == 0) atomicAdd(&g_tc_timeouts, 1u);
    return;
  }
  // Head parameters; B tile row f = [C_re[f, 0..15] | -C_im[f, 0..15]].
  for (int i = tid; i < 32 * 8; i += kT) {
    const int f2 = i >> 3, c = i & 7;
    const float2* cr = reinterpret_cast<const float2*>(p.C) + ((int64_t)h * FH + f2) * NH + (c & 3) * 4;
    const float2 c0 = cr[0], c1 = cr[1], c2 = cr[2], c3 = cr[3];
    const float4 v = c < 4 ? make_float4(c0.x, c1.x, c2.x, c3.x) : make_float4(-c0.y, -c1.y, -c2.y, -c3.y);
    *reinterpret_cast<float4*>(reinterpret_cast<char*>(sm + TcLay::bt2) + semx::tc::sw128(f2, c)) = v;
  }
  for (int i = tid; i < R * FH; i += kT) sm[TcLay::Co + i] = p.cout[(int64_t)h * R * FH + i];
  for (int i = tid; i < FH; i += kT) sm[TcLay::Dp + i] = p.D[(int64_t)h * FH + i];
  if (tid < NH) {
    sm[TcLay::prm + tid] = expf(p.A_log[(int64_t)h * NH + tid]);
    sm[TcLay::prm + NH + tid] = p.omega[(int64_t)h * NH + tid];
    sm[TcLay::prm + 2 * NH + tid] = p.detune ? p.sdet[(int64_t)h * NH + tid] : 1.f;
    reinterpret_cast<float2*>(sm + TcLay::cin)[tid] = make_float2(0.f, 0.f);
  }
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + TcLay::bar);
  if (tid < 32) semx::tc::tmem_alloc(reinterpret_cast<uint32_t*>(sm + TcLay::tslot), 32);
  if (tid == 0) semx::tc::mbar_init(bar, 1);
  semx::tc::fence_smem_to_async();
  semx::tc::fence_before_sync();
  __syncthreads();
  semx::tc::fence_after_sync();
  const uint32_t taddr = *reinterpret_cast<const uint32_t*>(sm + TcLay::tslot);

  float2* lam = reinterpret_cast<float2*>(sm + TcLay::lam);
  float2* bu = reinterpret_cast<float2*>(sm + TcLay::bu);
  float2* cin = reinterpret_cast<float2*>(sm + TcLay::cin);
  char* atile = reinterpret_cast<char*>(sm + TcLay::at);
  const int stg[2] = {TcLay::stg0, TcLay::stg1}, sml_off[2] = {TcLay::sml0, TcLay::sml1};
  const float2 bias = dt_bias(p, h);
  float pre[kPre];
  uint32_t phase = 0;
  int pending = -1;     // chunk index of the last chunk of a committed, not yet read-out tile
  bool bail = false;
  if (nchunks > 0) {
    const int nt0 = min(CT, L);
    stage_bulk<true, NH, FH, RK>(p, l, sm + stg[0], s, h, 0, nt0);
    load_small<true, RK>(p, s, h, 0, nt0, bias, pre);
    store_small<RK, CT>(p, sm + sml_off[0], nt0, pre);
  }
  cp_async_commit();
  for (int k = 0; k < nchunks; ++k) {
    const int b = k & 1, q = k & 3;
    const int t0 = k * CT, nt = min(CT, L - t0);
    const int t0n = t0 + CT, ntn = min(CT, L - t0n);
    cp_async_wait_all();
    __syncthreads();
    if (k + 1 < nchunks) {
      stage_bulk<true, NH, FH, RK>(p, l, sm + stg[b ^ 1], s, h, t0n, ntn);
      load_small<true, RK>(p, s, h, t0n, ntn, bias, pre);
    }
    cp_async_commit();
    const T* xs = reinterpret_cast<const T*>(sm + stg[b]);
    const T* bxs = xs + CT * l.xw;
    const T* bts = bxs + CT * l.bxw;
    const T* cts = bts + CT * l.btw;
    const float* sml = sm + sml_off[b];
    const float* dnus = sml + CT;
    const float* dths = sml + 2 * CT;
    const float* sbs = sml + 3 * CT;
    const float* scs = sbs + CT * R;
    // Poles and gained drive per (token, mode).
    for (int i = tid; i < nt * NH; i += kT) {
      const int t = i >> 4, n = i & 15;
      const float2 bq = ld2(bxs + t * l.bxw + 2 * n);
      float rr = bq.x;
      const float bi = bq.y;
#pragma unroll
      for (int r = 0; r < R; ++r) rr = fmaf(sbs[t * R + r], static_cast<float>(bts[t * l.btw + r * NH + n]), rr);
      const MDisc d = mdisc(p.gain, sm[TcLay::prm + n], sm[TcLay::prm + NH + n], sm[TcLay::prm + 2 * NH + n],
                            p.detune != 0, dnus[t], dths[t]);
      lam[t * hw + n] = make_float2(d.lre, d.lim);
      bu[t * hw + n] = make_float2(d.gr * rr - d.gi * bi, d.gr * bi + d.gi * rr);
    }
    if (p.ckpt != nullptr && tid < NH)
      reinterpret_cast<float2*>(p.ckpt)[((s * p.nck + k) * p.H + h) * NH + tid] = cin[tid];
    __syncthreads();
    if (q == 0 && pending >= 0) {
      // The previous tile: its MMA was committed a whole chunk ago; read it out before
      // this chunk's states overwrite the A rows 0..15 and its rank reads.
      const bool ok = semx::tc::mbar_wait(bar, phase, kTcWaitLimit);
      phase ^= 1u;
      if (__syncthreads_or(!ok)) {
        if (tid == 0) atomicAdd(&g_tc_timeouts, 1u);
        bail = true;
        break;
      }
      semx::tc::fence_after_sync();
      tc_epilogue<RK>(p, sm, taddr, s, h, (pending - 3) * CT, 3, L);
      semx::tc::fence_before_sync();
      pending = -1;
    }
    // The chunk's states, straight into A rows 16 q + t.
    const int row0 = 16 * q;
    chunk_scan_to<SEG, CT>(lam, bu, cin, NH, hw, nt, [&](int t, int n, float2 v) {
      const int row = row0 + t;
      char* base = atile + row * 128 + 4 * (n & 3);
      *reinterpret_cast<float*>(base + (((n >> 2) ^ (row & 7)) << 4)) = v.x;
      *reinterpret_cast<float*>(base + ((((n >> 2) + 4) ^ (row & 7)) << 4)) = v.y;
    });
    __syncthreads();
    // Rank reads s_c Re(<c_t, h_t>) per (token, rank), from the A rows; a thread pair per
    // item (modes 0-7 / 8-15), the halves added with one shuffle.
    if (R > 0) {
      static_assert(R == 0 || kT >= 2 * CT * R, "two threads per (token, rank)");
      const int item = tid >> 1, half = tid & 1;
      const bool act = item < nt * R;
      const int t = item / (R > 0 ? R : 1), r = item % (R > 0 ? R : 1);
      const int row = row0 + t;
      float acc = 0.f;
      if (act) {
        const T* cr = cts + t * l.ctw + r * 2 * NH;
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const int c = 2 * half + cc;
          const float4 hre = *reinterpret_cast<const float4*>(atile + semx::tc::sw128(row, c));
          const float4 him = *reinterpret_cast<const float4*>(atile + semx::tc::sw128(row, c + 4));
          const float4 cre = ld4(cr + 4 * c), cim = ld4(cr + NH + 4 * c);
          acc = fmaf(cre.x, hre.x, fmaf(-cim.x, him.x, acc));
          acc = fmaf(cre.y, hre.y, fmaf(-cim.y, him.y, acc));
          acc = fmaf(cre.z, hre.z, fmaf(-cim.z, him.z, acc));
          acc = fmaf(cre.w, hre.w, fmaf(-cim.w, him.w, acc));
        }
      }
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      if (act && half == 0) sm[TcLay::srk + row * 4 + r] = scs[item] * acc;
    }
    if (q == 3 || k == nchunks - 1) {
      // The tile is complete: one thread issues its MMAs (the accumulator is free: the
      // previous tile was read out before this tile's first chunk).
      semx::tc::fence_smem_to_async();
      semx::tc::fence_before_sync();
      __syncthreads();
      semx::tc::fence_after_sync();
      if (tid == 0) {
        constexpr uint32_t idesc = semx::tc::idesc_tf32(kTcM, 32);
        const uint32_t a0 = semx::tc::smem_addr(atile), b0 = semx::tc::smem_addr(sm + TcLay::bt2);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          semx::tc::mma_tf32(taddr, semx::tc::desc_sw128_kmajor(a0 + 32 * kk),
                             semx::tc::desc_sw128_kmajor(b0 + 32 * kk), idesc, kk > 0);
        semx::tc::mma_commit(bar);
      }
      pending = k;
    }
    if (k + 1 < nchunks) store_small<RK, CT>(p, sm + sml_off[b ^ 1], ntn, pre);
  }
  if (!bail && pending >= 0) {  // the last tile (possibly partial)
    const bool ok = semx::tc::mbar_wait(bar, phase, kTcWaitLimit);
    phase ^= 1u;
    if (__syncthreads_or(!ok)) {
      if (tid == 0) atomicAdd(&g_tc_timeouts, 1u);
      bail = true;
    } else {
      semx::tc::fence_after_sync();
      tc_epilogue<RK>(p, sm, taddr, s, h, (pending & ~3) * CT, pending & 3, L);
    }
  }
  cp_async_wait_all();
  // After a give-up, one more bounded wait for the outstanding MMA before its tensor
  // memory is released.
  if (bail) semx::tc::mbar_wait(bar, phase ^ 1u, kTcWaitLimit);
  semx::tc::fence_before_sync();
  __syncthreads();
  if (tid < 32) semx::tc::tmem_dealloc(taddr, 32);
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
  // Parameter accumulators: [dC (Fh,Nh,2) | denv (Fh,Nh) | dcout (R,Fh) | dD (Fh)]
  const int oC = 0, oE = oC + Fh * Nh * 2, oO = oE + (env ? Fh * Nh : 0), oD = oO + R * Fh, nacc = oD + Fh;
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
  float acc_bnu = 0.f, acc_bth = 0.f;  // dt bias sums of token lane tid < kTC

  for (int k = p.nchunks - 1; k >= 0; --k) {
    const int t0 = k * kTC, nt = min(kTC, L - t0);
    __syncthreads();
    stage_chunk<BF16>(p, l, sm, s, h, t0, nt, true);
    __syncthreads();
    poles_and_drive(p, l, sm, nt, false);
    __syncthreads();
    // Recompute the chunk's states from its checkpoint (row 0 = state entering it).
    if (tid < Nh) {
      float2 hv = reinterpret_cast<const float2*>(p.ckpt)[((s * p.nck + 2 * k) * p.H + h) * Nh + tid];
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
        const int t = i / (R > 0 ? R : 1), r = i % (R > 0 ? R : 1);
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
      const float draw = sn * p.rs * semx::softplus_grad(sm[l.raw + tid]);
      st<BF16>(p.dproj, row + cols.dnu, draw);
      st<BF16>(p.dproj, row + cols.dth, st_);
      acc_bnu += draw;
      acc_bth += st_;
    }
    if (mode_thr) {
      for (int t = nt - 1; t >= 0; --t) {
        acc_a += tn[2 * kTC * Nh + t * Nh + nthr];
        acc_om += tn[3 * kTC * Nh + t * Nh + nthr];
        acc_sd += tn[4 * kTC * Nh + t * Nh + nthr];
      }
    }
    // dx = D dy per (t, f) (the drive's part B^H d(raw drive) reaches x through the
    // projection's backward); d(drive columns) = d(raw drive) per (t, n).
    for (int i = tid; i < nt * Fh; i += kT) {
      const int t = i / Fh, f = i % Fh;
      st<BF16>(p.dx, (s * p.L + t0 + t) * Fd + (int64_t)h * Fh + f, sm[l.Dp + f] * sm[l.dys + i]);
    }
    for (int i = tid; i < nt * 2 * Nh; i += kT) {
      const int t = i / (2 * Nh), j = i % (2 * Nh);
      st<BF16>(p.dproj, (s * p.L + t0 + t) * p.P + cols.bx + j, sm[l.db + t * 2 * Nh + j]);
    }
    // Rank write: d s_b, d b_t.
    if (R > 0) {
      for (int i = tid; i < nt * R; i += kT) {
        const int t = i / (R > 0 ? R : 1), r = i % (R > 0 ? R : 1);
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
  if (tid < kTC) {
    sm[l.rb + tid] = acc_bnu;
    sm[l.rb + kTC + tid] = acc_bth;
  }
  __syncthreads();
  // Partial row of sequence s, parameter-major so every segment is in output order:
  // [dC | denv | dcout | dD | dA_log | domega | ddetune | d dt bias], each over all heads.
  {
    const int64_t H = p.H;
    float* row = p.part + s * p.K;
    int64_t off = 0;
    auto put = [&](int64_t seg_per_head, int src, int cnt) {
      for (int i = tid; i < cnt; i += kT) row[off + (int64_t)h * seg_per_head + i] = sm[l.acc + src + i];
      off += H * seg_per_head;
    };
    put(Fh * Nh * 2, oC, Fh * Nh * 2);
    if (env) put(Fh * Nh, oE, Fh * Nh);
    if (R > 0) put(R * Fh, oO, R * Fh);
    put(Fh, oD, Fh);
    if (mode_thr) {
      row[off + (int64_t)h * Nh + nthr] = acc_a * sm[l.prm + nthr];  // d/dA_log = a d/da
      row[off + H * Nh + (int64_t)h * Nh + nthr] = acc_om;
      row[off + 2 * H * Nh + (int64_t)h * Nh + nthr] = acc_sd;
    }
    off += 3 * H * Nh;
    if (tid < 2) {  // over the token lanes in a fixed order
      float acc = 0.f;
      for (int q = 0; q < kTC; ++q) acc += sm[l.rb + tid * kTC + q];
      row[off + tid * H + h] = acc;
    }
  }
}

// ------------------------------------------------------------- backward, 16 x 32 heads
// The backward of the 16-mode, 32-channel heads (rank RK = 0 or 4), 16-token chunks:
// everything a thread sums over time lives in its registers with a fixed ownership, so
// the shared-memory footprint (about 52 KB) leaves room for 4 CTAs per SM.
constexpr int kB_NH = 16, kB_FH = 32, kB_CT = 16, kB_SEG = 8;
constexpr int kB_HW = kB_NH + 2;  // float2 row width of lam / gain / drive / h / G / db

// Reverse adjoint scan of a chunk: G_t = g_t + c_{t+1}, c_t = conj(lam_t) G_t, starting
// from cadj[n] (the carry of the token after the chunk); writes G over g and the carry at
// the chunk start back to cadj[n]. Thread (mode, segment) as in chunk_scan; segments are
// combined by an inclusive scan from the last segment down.
template <int SEG, int CT>
__device__ __forceinline__ void chunk_scan_rev(const float2* lam, float2* gs, float2* cadj, int hw, int nt) {
  constexpr int TS = CT / SEG, MPW = 32 / SEG;
  const int lane = threadIdx.x & 31;
  const int n = (threadIdx.x >> 5) * MPW + lane % MPW, seg = lane / MPW;
  const int t0 = seg * TS;
  float2 A = make_float2(1.f, 0.f), b = make_float2(0.f, 0.f);  // c_start = A c_end + b
#pragma unroll
  for (int i = TS - 1; i >= 0; --i) {
    const int t = t0 + i;
    if (t < nt) {
      const float2 l = lam[t * hw + n];
      const float2 g = gs[t * hw + n];
      const float2 G = make_float2(g.x + b.x, g.y + b.y);
      b = make_float2(l.x * G.x + l.y * G.y, l.x * G.y - l.y * G.x);
      A = make_float2(l.x * A.x + l.y * A.y, l.x * A.y - l.y * A.x);
    }
  }
  // Inclusive maps over segments seg .. SEG-1: (A, b) o (An, bn) = (A An, A bn + b).
#pragma unroll
  for (int off = 1; off < SEG; off <<= 1) {
    const float anr = __shfl_down_sync(0xffffffffu, A.x, off * MPW);
    const float ani = __shfl_down_sync(0xffffffffu, A.y, off * MPW);
    const float bnr = __shfl_down_sync(0xffffffffu, b.x, off * MPW);
    const float bni = __shfl_down_sync(0xffffffffu, b.y, off * MPW);
    if (seg + off < SEG) {
      const float2 nb = cmul(A, make_float2(bnr, bni));
      b = make_float2(nb.x + b.x, nb.y + b.y);
      A = cmul(A, make_float2(anr, ani));
    }
  }
  const float2 c0 = cadj[n];
  const float enr = __shfl_down_sync(0xffffffffu, A.x, MPW);
  const float eni = __shfl_down_sync(0xffffffffu, A.y, MPW);
  const float ebr = __shfl_down_sync(0xffffffffu, b.x, MPW);
  const float ebi = __shfl_down_sync(0xffffffffu, b.y, MPW);
  float2 c = c0;
  if (seg < SEG - 1) {
    c = cmul(make_float2(enr, eni), c0);
    c.x += ebr;
    c.y += ebi;
  }
#pragma unroll
  for (int i = TS - 1; i >= 0; --i) {
    const int t = t0 + i;
    if (t < nt) {
      const float2 l = lam[t * hw + n];
      const float2 g = gs[t * hw + n];
      const float2 G = make_float2(g.x + c.x, g.y + c.y);
      gs[t * hw + n] = G;
      c = make_float2(l.x * G.x + l.y * G.y, l.x * G.y - l.y * G.x);
    }
  }
  __syncwarp();
  if (seg == 0) {
    const float2 e = cmul(A, c0);
    cadj[n] = make_float2(e.x + b.x, e.y + b.y);
  }
}

struct BLay {
  int Cfr, Cfi, Ef, Co, Dp, prm, cin, cadj;
  int stg[2], dys[2], sml[2];
  int lam, gn, braw, hs, gs, db, sr, dr, red, rb;
  int xw, bxw, btw, ctw, dyw;
  int total;
};

__host__ __device__ inline BLay make_blay(int R, bool env, int es) {
  constexpr int NH = kB_NH, FH = kB_FH, CT = kB_CT, HW = kB_HW;
  BLay l = {};
  int o = 0;
  auto take = [&](int n) {
    const int at = o;
    o += al4(n);
    return at;
  };
  l.Cfr = take(FH * NH);
  l.Cfi = take(FH * NH);
  l.Ef = env ? take(FH * NH) : -1;
  l.Co = take(R * FH);
  l.Dp = take(FH);
  l.prm = take(3 * NH);
  l.cin = take(2 * NH);
  l.cadj = take(2 * NH);
  const int pad = 16 / es;
  l.xw = FH + pad;
  l.bxw = 2 * NH;
  l.btw = R > 0 ? R * NH + pad : 0;
  l.ctw = R > 0 ? 2 * R * NH + pad : 0;
  l.dyw = FH + 4;
  for (int b = 0; b < 2; ++b) l.stg[b] = take((CT * (l.xw + l.bxw + l.btw + l.ctw) * es + 3) / 4);
  for (int b = 0; b < 2; ++b) l.dys[b] = take(CT * l.dyw);
  for (int b = 0; b < 2; ++b) l.sml[b] = take(CT * (3 + 2 * R));
  l.lam = take(CT * HW * 2);
  l.gn = take(CT * HW * 2);
  l.braw = take(CT * HW * 2);
  l.hs = take((CT + 1) * HW * 2);
  l.gs = take(CT * HW * 2);
  l.db = take(CT * HW * 2);
  l.sr = take(CT * R);
  l.dr = take(CT * R);
  // The end-of-kernel sums reuse lam and gn (contiguous, 2 CT HW 2 >= 3 NH kT/8 + 2 kT/8
  // floats), which are dead after the last chunk: 3 KB less per CTA is what lets 5 CTAs
  // share an SM.
  l.red = l.lam;
  l.rb = l.lam + 3 * NH * (kT / 8);
  static_assert(2 * kB_CT * kB_HW * 2 >= 3 * kB_NH * (kT / 8) + 2 * (kT / 8), "red / rb must fit in lam + gn");
  l.total = o;
  return l;
}

template <bool BF16, int RK>
__global__ void __launch_bounds__(kT) mimo_layer_bwd16_kernel(const LParams p) {
  using T = typename std::conditional<BF16, __nv_bfloat16, float>::type;
  constexpr int NH = kB_NH, FH = kB_FH, CT = kB_CT, HW = kB_HW, R = RK;
  extern __shared__ float4 smem4[];
  float* sm = reinterpret_cast<float*>(smem4);
  const bool env = p.envelope != 0, det = p.detune != 0;
  const BLay l = make_blay(R, env, (int)sizeof(T));
  const int64_t s = blockIdx.x / p.H;
  const int h = (int)(blockIdx.x % p.H);
  const int tid = threadIdx.x;
  const int L = (int)p.L;
  const int64_t Fd = p.H * p.Fh;
  const Cols cols = cols_of(p, h);
  // Head parameters in the storage orders the loops read.
  for (int i = tid; i < NH * FH; i += kT) {
    const int f2 = i / NH, n2 = i % NH;
    const float2 cv = reinterpret_cast<const float2*>(p.C)[((int64_t)h * FH + f2) * NH + n2];
    sm[l.Cfr + f2 * NH + n2] = cv.x;
    sm[l.Cfi + f2 * NH + n2] = cv.y;
    if (env) sm[l.Ef + f2 * NH + n2] = p.env[((int64_t)h * FH + f2) * NH + n2];
  }
  for (int i = tid; i < R * FH; i += kT) sm[l.Co + i] = p.cout[(int64_t)h * R * FH + i];
  for (int i = tid; i < FH; i += kT) sm[l.Dp + i] = p.D[(int64_t)h * FH + i];
  for (int n = tid; n < NH; n += kT) {
    sm[l.prm + n] = expf(p.A_log[(int64_t)h * NH + n]);
    sm[l.prm + NH + n] = p.omega[(int64_t)h * NH + n];
    sm[l.prm + 2 * NH + n] = det ? p.sdet[(int64_t)h * NH + n] : 1.f;
    reinterpret_cast<float2*>(sm + l.cadj)[n] = make_float2(0.f, 0.f);
  }
  float2* lam = reinterpret_cast<float2*>(sm + l.lam);
  float2* gn = reinterpret_cast<float2*>(sm + l.gn);
  float2* braw = reinterpret_cast<float2*>(sm + l.braw);
  float2* hs = reinterpret_cast<float2*>(sm + l.hs);
  float2* gs = reinterpret_cast<float2*>(sm + l.gs);
  float2* db = reinterpret_cast<float2*>(sm + l.db);
  float2* cin = reinterpret_cast<float2*>(sm + l.cin);
  float2* cadj = reinterpret_cast<float2*>(sm + l.cadj);

  // Thread roles (fixed for the whole kernel).
  const int tA = tid / 8, npA = tid % 8;        // (token, mode pair) items
  const int fC = tid / 4, nqC = tid % 4;        // dC / denv items (channel, 4 modes)
  const int rO = tid / FH, fO = tid % FH;       // dcout items (rank, channel) when R = 4
  float acc_a[2] = {0.f, 0.f}, acc_om[2] = {0.f, 0.f}, acc_sd[2] = {0.f, 0.f};
  float aCr[4] = {}, aCi[4] = {}, aE[4] = {};
  float aO = 0.f, aD = 0.f;
  float aBnu = 0.f, aBth = 0.f;  // dt bias sums of token lane tA (threads with npA == 0)
  const float2 bias = dt_bias(p, h);

  const int nck = p.nck;
  float pre[kPre];
  auto stage = [&](int k, int b) {
    const int t0 = k * CT, nt = min(CT, L - t0);
    T* xs = reinterpret_cast<T*>(sm + l.stg[b]);
    const int64_t row0 = s * p.L + t0;
    const T* Pj = reinterpret_cast<const T*>(p.proj);
    stage_segment<T>(xs, l.xw, reinterpret_cast<const T*>(p.x), row0, Fd, (int64_t)h * FH, FH, nt,
                     (p.vec & 1) != 0);
    stage_segment<T>(xs + CT * l.xw, l.bxw, Pj, row0, p.P, cols.bx, 2 * NH, nt, (p.vec & 16) != 0);
    if (R > 0) {
      stage_segment<T>(xs + CT * (l.xw + l.bxw), l.btw, Pj, row0, p.P, cols.bt, R * NH, nt, (p.vec & 2) != 0);
      stage_segment<T>(xs + CT * (l.xw + l.bxw + l.btw), l.ctw, Pj, row0, p.P, cols.ct, 2 * R * NH, nt,
                       (p.vec & 2) != 0);
    }
    stage_segment<float>(sm + l.dys[b], l.dyw, p.dy, row0, Fd, (int64_t)h * FH, FH, nt, (p.vec & 4) != 0);
  };
  if (nck > 0) {
    const int k = nck - 1, nt = min(CT, L - k * CT);
    stage(k, 0);
    load_small<BF16, RK>(p, s, h, k * CT, nt, bias, pre);
    store_small<RK, CT>(p, sm + l.sml[0], nt, pre);
  }
  cp_async_commit();
  int b = 0;
  for (int k = nck - 1; k >= 0; --k, b ^= 1) {
    const int t0 = k * CT, nt = min(CT, L - t0);
    cp_async_wait_all();
    __syncthreads();
    if (k > 0) {
      stage(k - 1, b ^ 1);
      load_small<BF16, RK>(p, s, h, (k - 1) * CT, CT, bias, pre);
    }
    cp_async_commit();
    const T* xs = reinterpret_cast<const T*>(sm + l.stg[b]);
    const T* bxs = xs + CT * l.xw;
    const T* bts = bxs + CT * l.bxw;
    const T* cts = bts + CT * l.btw;
    const float* dys = sm + l.dys[b];
    const float* sml = sm + l.sml[b];
    const float* raws = sml;
    const float* dnus = sml + CT;
    const float* dths = sml + 2 * CT;
    const float* sbs = sml + 3 * CT;
    const float* scs = sbs + CT * R;
    const int xw = l.xw, bxw = l.bxw, btw = l.btw, ctw = l.ctw, dyw = l.dyw;

    // A. Poles, gains, raw and gained drive per (token, mode pair); entry state.
    if (tid < NH) {
      const float2 c = reinterpret_cast<const float2*>(p.ckpt)[((s * nck + k) * p.H + h) * NH + tid];
      cin[tid] = c;
      hs[tid] = c;
    }
    if (tA < nt) {
      const int t = tA, na = 2 * npA;
      const float4 bq = ld4(bxs + t * bxw + 2 * na);
      float br0 = bq.x, bi0 = bq.y, br1 = bq.z, bi1 = bq.w;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float sbv = sbs[t * R + r];
        br0 = fmaf(sbv, static_cast<float>(bts[t * btw + r * NH + na]), br0);
        br1 = fmaf(sbv, static_cast<float>(bts[t * btw + r * NH + na + 1]), br1);
      }
#pragma unroll
      for (int dn = 0; dn < 2; ++dn) {
        const int n = na + dn;
        const float brv = dn ? br1 : br0, biv = dn ? bi1 : bi0;
        const MDisc d = mdisc(p.gain, sm[l.prm + n], sm[l.prm + NH + n], sm[l.prm + 2 * NH + n], det,
                              dnus[t], dths[t]);
        lam[t * HW + n] = make_float2(d.lre, d.lim);
        gn[t * HW + n] = make_float2(d.gr, d.gi);
        braw[t * HW + n] = make_float2(brv, biv);
        gs[t * HW + n] = make_float2(d.gr * brv - d.gi * biv, d.gr * biv + d.gi * brv);
      }
    }
    __syncthreads();
    // B. States of the chunk (rows 1..nt of hs) from the checkpoint.
    chunk_scan<kB_SEG, CT>(lam, gs, hs + HW, cin, NH, HW, nt);
    __syncthreads();
    // C. Rank read and its adjoint per (token, rank).
    if (R > 0) {
      if (tid < nt * R) {
        const int t = tid / (R > 0 ? R : 1), r = tid % (R > 0 ? R : 1);
        const T* cr = cts + t * ctw + r * 2 * NH;
        float rd = 0.f;
#pragma unroll
        for (int n = 0; n < NH; ++n) {
          const float2 hv = hs[(t + 1) * HW + n];
          rd = fmaf(static_cast<float>(cr[n]), hv.x, fmaf(-static_cast<float>(cr[NH + n]), hv.y, rd));
        }
        float dyc = 0.f;
#pragma unroll 8
        for (int f = 0; f < FH; ++f) dyc = fmaf(dys[t * dyw + f], sm[l.Co + r * FH + f], dyc);
        const float scv = scs[t * R + r];
        sm[l.sr + tid] = scv * rd;
        sm[l.dr + tid] = scv * dyc;
        st<BF16>(p.dproj, (s * p.L + t0 + t) * p.P + cols.sc + r, rd * dyc);
      }
      __syncthreads();
    }
    // D. Readout adjoint g per (token, mode pair), and the c_t gradient.
    if (tA < nt) {
      const int t = tA, na = 2 * npA;
      float g0r = 0.f, g0i = 0.f, g1r = 0.f, g1i = 0.f, e0 = 0.f, e1 = 0.f;
#pragma unroll 8
      for (int f = 0; f < FH; ++f) {
        const float dv = dys[t * dyw + f];
        const float2 cr = *reinterpret_cast<const float2*>(sm + l.Cfr + f * NH + na);
        const float2 ci = *reinterpret_cast<const float2*>(sm + l.Cfi + f * NH + na);
        g0r = fmaf(dv, cr.x, g0r);
        g0i = fmaf(-dv, ci.x, g0i);
        g1r = fmaf(dv, cr.y, g1r);
        g1i = fmaf(-dv, ci.y, g1i);
        if (env) {
          const float2 ev = *reinterpret_cast<const float2*>(sm + l.Ef + f * NH + na);
          e0 = fmaf(dv, ev.x, e0);
          e1 = fmaf(dv, ev.y, e1);
        }
      }
      const float2 h0 = hs[(t + 1) * HW + na], h1 = hs[(t + 1) * HW + na + 1];
      if (env) {
        g0r = fmaf(2.f * e0, h0.x, g0r);
        g0i = fmaf(2.f * e0, h0.y, g0i);
        g1r = fmaf(2.f * e1, h1.x, g1r);
        g1i = fmaf(2.f * e1, h1.y, g1i);
      }
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float drv = sm[l.dr + t * R + r];
        const T* cr = cts + t * ctw + r * 2 * NH;
        g0r = fmaf(drv, static_cast<float>(cr[na]), g0r);
        g1r = fmaf(drv, static_cast<float>(cr[na + 1]), g1r);
        g0i = fmaf(-drv, static_cast<float>(cr[NH + na]), g0i);
        g1i = fmaf(-drv, static_cast<float>(cr[NH + na + 1]), g1i);
        const int64_t row = (s * p.L + t0 + t) * p.P + cols.ct + (int64_t)r * 2 * NH;
        st<BF16>(p.dproj, row + na, drv * h0.x);
        st<BF16>(p.dproj, row + na + 1, drv * h1.x);
        st<BF16>(p.dproj, row + NH + na, -drv * h0.y);
        st<BF16>(p.dproj, row + NH + na + 1, -drv * h1.y);
      }
      gs[t * HW + na] = make_float2(g0r, g0i);
      gs[t * HW + na + 1] = make_float2(g1r, g1i);
    }
    __syncthreads();
    // E. Adjoint scan: G over g, carry across chunks in cadj.
    chunk_scan_rev<kB_SEG, CT>(lam, gs, cadj, HW, nt);
    __syncthreads();
    // F. Through the gain and the pole per (token, mode pair).
    {
      float sdnu = 0.f, sdth = 0.f;
      if (tA < nt) {
        const int t = tA;
#pragma unroll
        for (int dn = 0; dn < 2; ++dn) {
          const int n = 2 * npA + dn;
          const float a = sm[l.prm + n], om = sm[l.prm + NH + n], sd = sm[l.prm + 2 * NH + n];
          const float dnu = dnus[t], dth = dths[t];
          const MDisc d = mdisc(p.gain, a, om, sd, det, dnu, dth);
          const float2 G = gs[t * HW + n], bv = braw[t * HW + n], hp = hs[t * HW + n];
          db[t * HW + n] = make_float2(d.gr * G.x + d.gi * G.y, d.gr * G.y - d.gi * G.x);
          const float dgr = bv.x * G.x + bv.y * G.y, dgi = bv.x * G.y - bv.y * G.x;
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
          sdnu += d_dnu;
          sdth += det ? dbase * sd : dbase;
          acc_a[dn] += da_extra - dnu * P;
          acc_om[dn] += dbase;
          acc_sd[dn] += det ? dbase * dth : 0.f;
        }
      }
      // Per-token sums over the 8 mode pairs (consecutive lanes), fixed order.
#pragma unroll
      for (int m = 1; m < 8; m <<= 1) {
        sdnu += __shfl_xor_sync(0xffffffffu, sdnu, m);
        sdth += __shfl_xor_sync(0xffffffffu, sdth, m);
      }
      if (npA == 0 && tA < nt) {
        const int64_t row = (s * p.L + t0 + tA) * p.P;
        const float draw = sdnu * p.rs * semx::softplus_grad(raws[tA]);
        st<BF16>(p.dproj, row + cols.dnu, draw);
        st<BF16>(p.dproj, row + cols.dth, sdth);
        aBnu += draw;
        aBth += sdth;
      }
    }
    __syncthreads();
    // G. dx = D dy per (token, 4 channels); the drive's part B^H d(raw drive) reaches x
    // through the projection's backward. d(drive columns) = d(raw drive) of the token's
    // mode pair.
    if (tA < nt) {
      const int t = tA, f0 = 4 * npA, na = 2 * npA;
      float4 acc;
      acc.x = sm[l.Dp + f0] * dys[t * dyw + f0];
      acc.y = sm[l.Dp + f0 + 1] * dys[t * dyw + f0 + 1];
      acc.z = sm[l.Dp + f0 + 2] * dys[t * dyw + f0 + 2];
      acc.w = sm[l.Dp + f0 + 3] * dys[t * dyw + f0 + 3];
      const float2 g0 = db[t * HW + na], g1 = db[t * HW + na + 1];
      const int64_t drow = (s * p.L + t0 + t) * p.P + cols.bx + 2 * na;
      if ((p.vec & 16) != 0) {
        if (BF16) {
          __nv_bfloat162 q[2] = {__floats2bfloat162_rn(g0.x, g0.y), __floats2bfloat162_rn(g1.x, g1.y)};
          *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p.dproj) + drow) =
              *reinterpret_cast<const uint2*>(q);
        } else {
          *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.dproj) + drow) = make_float4(g0.x, g0.y, g1.x, g1.y);
        }
      } else {
        st<BF16>(p.dproj, drow, g0.x);
        st<BF16>(p.dproj, drow + 1, g0.y);
        st<BF16>(p.dproj, drow + 2, g1.x);
        st<BF16>(p.dproj, drow + 3, g1.y);
      }
      const int64_t xo = (s * p.L + t0 + t) * Fd + (int64_t)h * FH + f0;
      if ((p.vec & 8) != 0) {
        if (BF16) {
          __nv_bfloat162 q[2] = {__floats2bfloat162_rn(acc.x, acc.y), __floats2bfloat162_rn(acc.z, acc.w)};
          *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p.dx) + xo) = *reinterpret_cast<const uint2*>(q);
        } else {
          *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.dx) + xo) = acc;
        }
      } else {
        st<BF16>(p.dx, xo, acc.x);
        st<BF16>(p.dx, xo + 1, acc.y);
        st<BF16>(p.dx, xo + 2, acc.z);
        st<BF16>(p.dx, xo + 3, acc.w);
      }
    }
    // H. Rank write: d s_b, d b_t.
    if (R > 0 && tid < nt * R) {
      const int t = tid / (R > 0 ? R : 1), r = tid % (R > 0 ? R : 1);
      const float sbv = sbs[t * R + r];
      const int64_t row = (s * p.L + t0 + t) * p.P;
      float acc = 0.f;
#pragma unroll
      for (int n = 0; n < NH; ++n) {
        const float g = db[t * HW + n].x;
        acc = fmaf(static_cast<float>(bts[t * btw + r * NH + n]), g, acc);
        st<BF16>(p.dproj, row + cols.bt + r * NH + n, sbv * g);
      }
      st<BF16>(p.dproj, row + cols.sb + r, acc);
    }
    // I. Parameter sums over the chunk, fixed ownership.
    for (int t = 0; t < nt; ++t) {
      {  // dC[fC, 4 nqC .. +3] += dy (h_re, -h_im); denv += dy |h|^2
        const float dv = dys[t * dyw + fC];
        const float4 ha = *reinterpret_cast<const float4*>(hs + (t + 1) * HW + 4 * nqC);
        const float4 hb = *reinterpret_cast<const float4*>(hs + (t + 1) * HW + 4 * nqC + 2);
        const float hr[4] = {ha.x, ha.z, hb.x, hb.z}, hi[4] = {ha.y, ha.w, hb.y, hb.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          aCr[j] = fmaf(dv, hr[j], aCr[j]);
          aCi[j] = fmaf(-dv, hi[j], aCi[j]);
          if (env) aE[j] = fmaf(dv, hr[j] * hr[j] + hi[j] * hi[j], aE[j]);
        }
      }
      if (R > 0) aO = fmaf(sm[l.sr + t * R + rO], dys[t * dyw + fO], aO);
      if (tid < FH) aD = fmaf(dys[t * dyw + tid], static_cast<float>(xs[t * xw + tid]), aD);
    }
    // Small operands of the next chunk (its buffer was last read two chunks ago).
    if (k > 0) store_small<RK, CT>(p, sm + l.sml[b ^ 1], CT, pre);
  }
  __syncthreads();
  // Per-mode sums over the 16 token lanes that share a mode pair, fixed order.
  float* red = sm + l.red;  // [3][NH][kT / 8]
#pragma unroll
  for (int dn = 0; dn < 2; ++dn) {
    const int n = 2 * npA + dn;
    red[(0 * NH + n) * (kT / 8) + tA] = acc_a[dn];
    red[(1 * NH + n) * (kT / 8) + tA] = acc_om[dn];
    red[(2 * NH + n) * (kT / 8) + tA] = acc_sd[dn];
  }
  if (npA == 0) {
    sm[l.rb + tA] = aBnu;
    sm[l.rb + kT / 8 + tA] = aBth;
  }
  __syncthreads();
  // Partial row of sequence s: [dC | denv | dcout | dD | dA_log | domega | ddetune | d dt bias].
  const int64_t H = p.H;
  float* row = p.part + s * p.K;
  int64_t off = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int64_t i = ((int64_t)h * FH + fC) * NH + 4 * nqC + j;
    row[off + 2 * i] = aCr[j];
    row[off + 2 * i + 1] = aCi[j];
  }
  off += H * FH * NH * 2;
  if (env) {
#pragma unroll
    for (int j = 0; j < 4; ++j) row[off + ((int64_t)h * FH + fC) * NH + 4 * nqC + j] = aE[j];
    off += H * FH * NH;
  }
  if (R > 0) {
    row[off + (int64_t)h * R * FH + rO * FH + fO] = aO;
    off += H * R * FH;
  }
  if (tid < FH) row[off + (int64_t)h * FH + tid] = aD;
  off += H * FH;
  if (tid < 3 * NH) {
    const int which = tid / NH, n = tid % NH;
    float acc = 0.f;
    for (int q = 0; q < kT / 8; ++q) acc += red[(which * NH + n) * (kT / 8) + q];
    if (which == 0) acc *= sm[l.prm + n];  // d/dA_log = a d/da
    row[off + which * H * NH + (int64_t)h * NH + n] = acc;
  }
  off += 3 * H * NH;
  if (tid < 2) {  // dt bias: over the token lanes in a fixed order
    float acc = 0.f;
    for (int q = 0; q < kT / 8; ++q) acc += sm[l.rb + tid * (kT / 8) + q];
    row[off + tid * H + h] = acc;
  }
}

// ------------------------------------------------ backward, tensor-core readout adjoint (bf16)
// mimo_layer_bwd16_kernel with the readout adjoint on the tensor cores (bf16 operands,
// 16 x 32 heads, no envelope readout): per 64-token tile, one thread issues four
// kind::tf32 MMAs, D (64 x 32, tensor memory) = dy tile (K-major, rows = tokens) x
// [C_re | -C_im]^T (K-major, rows = modes), i.e. g[t, n] = sum_f dy[t, f] conj(C[f, n]);
// warp q moves the rows of chunk q into shared memory when the backward reaches that
// chunk. The dy tile holds the current 64-token tile; each chunk's 16 rows are refilled
// with the previous tile's (cp.async) as soon as the chunk is done. The chunk's states
// live in a swizzled h tile ([h_re | -h_im], rows = tokens) plus the entry state. dC stays
// a per-thread register sum: the tf32 MMA with an MN-major operand (the token-major h and
// dy tiles read as K = tokens) returned zeros in the 128-byte-swizzled layout used here.
// 43 KB of shared memory, at most 96 registers: 5 CTAs per SM, as for bwd16.
struct TcBLay {
  static constexpr int dyt = 0;                          // 64 x 32 fp32, swizzled
  static constexpr int bwt = dyt + 64 * 32;              // 32 x 32 fp32, swizzled
  // The chunk's states, row t = [h_re | -h_im], and its dy rows, both 16 x 32 fp32 in the
  // 32-byte-based swizzle: the MN-major A operand (h; the dy rows behind it fill the
  // accumulator rows 32-63, which are not read) and B operand (dy) of the dC sums.
  static constexpr int ht = bwt + 32 * 32;
  static constexpr int dy32 = ht + 16 * 32;
  static constexpr int Co = dy32 + 16 * 32;              // c_out (4 x 32)
  static constexpr int Dp = Co + 4 * 32;
  static constexpr int prm = Dp + 32;                    // a, omega, detune (3 x 16)
  static constexpr int cin = prm + 48;                   // scan carry (16 float2)
  static constexpr int cadj = cin + 32;                  // adjoint carry (16 float2)
  static constexpr int hent = cadj + 32;                 // chunk entry state (16 float2)
  static constexpr int stg_floats = 16 * (32 + 32 + 64 + 128) / 2;
  static constexpr int stg0 = hent + 32;
  static constexpr int stg1 = stg0 + stg_floats;
  static constexpr int sml_floats = 16 * (3 + 2 * 4);
  static constexpr int sml0 = stg1 + stg_floats;
  static constexpr int sml1 = sml0 + sml_floats;
  static constexpr int lam = sml1 + sml_floats;          // 16 x kB_HW float2 each
  static constexpr int braw = lam + 16 * kB_HW * 2;
  static constexpr int gs = braw + 16 * kB_HW * 2;
  static constexpr int db = gs + 16 * kB_HW * 2;
  static constexpr int sr = db + 16 * kB_HW * 2;
  static constexpr int dr = sr + 64;
  static constexpr int bar = dr + 64;                    // two 8-byte mbarriers: readout adjoint, dC
  static constexpr int tslot = bar + 4;
  static constexpr int total = tslot + 4;
  static constexpr int red = lam;                        // end-of-kernel sums reuse lam + braw
  static constexpr int rb = lam + 3 * 16 * (kT / 8);
};
static_assert(TcBLay::bwt % 256 == 0 && TcBLay::ht % 256 == 0 && TcBLay::dy32 == TcBLay::ht + 512 &&
                  TcBLay::stg0 % 4 == 0 &&
                  TcBLay::bar % 2 == 0 && TcBLay::rb + 2 * (kT / 8) <= TcBLay::gs,
              "tensor-core backward layout");

// Copies dy rows [t0g, t0g + nt) of head h into dy-tile rows row0.. (zeros for rows
// nt..15 of a partial chunk).
__device__ __forceinline__ void tcb_load_dy(const LParams& p, float* sm, int64_t s, int h, int row0, int t0g,
                                            int nt) {
  char* dyt = reinterpret_cast<char*>(sm + TcBLay::dyt);
  const int64_t Fd = p.H * 32;
  for (int i = threadIdx.x; i < 16 * 8; i += kT) {
    const int r = i >> 3, c = i & 7;
    float* dst = reinterpret_cast<float*>(dyt + semx::tc::sw128(row0 + r, c));
    if (r < nt) {
      const float* src = p.dy + (s * p.L + t0g + r) * Fd + (int64_t)h * 32 + 4 * c;
      if ((p.vec & 4) != 0) {
        cp_async16(dst, src);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) dst[e] = src[e];
      }
    } else {
      *reinterpret_cast<float4*>(dst) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
}

// dy[t, f] and a float4 of it from the dy tile (row = tile row of token t).
__device__ __forceinline__ float tcb_dy(const float* sm, int row, int f) {
  return *reinterpret_cast<const float*>(reinterpret_cast<const char*>(sm + TcBLay::dyt) +
                                         semx::tc::sw128(row, f >> 2) + 4 * (f & 3));
}
// h_t[n] from the h tile, which stores [h_re | -h_im].
__device__ __forceinline__ float2 tcb_h(const float* sm, int t, int n) {
  const char* ht = reinterpret_cast<const char*>(sm + TcBLay::ht);
  const float re = *reinterpret_cast<const float*>(ht + semx::tc::sw128_32b(t, n));
  const float nim = *reinterpret_cast<const float*>(ht + semx::tc::sw128_32b(t, n + 16));
  return make_float2(re, -nim);
}

template <int RK>
__global__ void __launch_bounds__(kT, 5) mimo_layer_bwd_tc_kernel(const LParams p) {
  using T = __nv_bfloat16;
  constexpr int NH = kB_NH, FH = kB_FH, CT = kB_CT, HW = kB_HW, R = RK;
  extern __shared__ __align__(1024) float4 smem4[];
  float* sm = reinterpret_cast<float*>(smem4);
  const bool det = p.detune != 0;
  const int64_t s = blockIdx.x / p.H;
  const int h = (int)(blockIdx.x % p.H);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int L = (int)p.L;
  const int64_t Fd = p.H * p.Fh;
  const Cols cols = cols_of(p, h);
  // Unpadded staging rows (the staging helpers read these widths).
  FLay fl = {};
  fl.tc = CT;
  fl.xw = FH;
  fl.bxw = 2 * NH;
  fl.btw = R * NH;
  fl.ctw = 2 * R * NH;
  if ((semx::tc::smem_addr(smem4) & 1023u) != 0) {  // the swizzled tiles need a 1 KB base
    if (tid == 0) atomicAdd(&g_tc_timeouts, 1u);
    return;
  }
  // Head parameters; B tile row n = [C_re[0..31, n]] (n < 16) or [-C_im[0..31, n - 16]].
  for (int i = tid; i < 32 * 8; i += kT) {
    const int n2 = i >> 3, c = i & 7;
    const float2* cp = reinterpret_cast<const float2*>(p.C) + ((int64_t)h * FH + 4 * c) * NH + (n2 & 15);
    float v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 cv = cp[e * NH];
      v[e] = n2 < 16 ? cv.x : -cv.y;
    }
    *reinterpret_cast<float4*>(reinterpret_cast<char*>(sm + TcBLay::bwt) + semx::tc::sw128(n2, c)) =
        make_float4(v[0], v[1], v[2], v[3]);
  }
  // h and dy32 tiles: rows past a partial chunk stay 0.
  for (int i = tid; i < 2 * 16 * 32; i += kT) sm[TcBLay::ht + i] = 0.f;
  for (int i = tid; i < R * FH; i += kT) sm[TcBLay::Co + i] = p.cout[(int64_t)h * R * FH + i];
  for (int i = tid; i < FH; i += kT) sm[TcBLay::Dp + i] = p.D[(int64_t)h * FH + i];
  if (tid < NH) {
    sm[TcBLay::prm + tid] = expf(p.A_log[(int64_t)h * NH + tid]);
    sm[TcBLay::prm + NH + tid] = p.omega[(int64_t)h * NH + tid];
    sm[TcBLay::prm + 2 * NH + tid] = det ? p.sdet[(int64_t)h * NH + tid] : 1.f;
    reinterpret_cast<float2*>(sm + TcBLay::cadj)[tid] = make_float2(0.f, 0.f);
  }
  uint64_t* bar_adj = reinterpret_cast<uint64_t*>(sm + TcBLay::bar);
  uint64_t* bar_dc = bar_adj + 1;
  // Tensor memory: columns 0-31 the readout adjoint of a 64-token tile, 32-63 the dC /
  // dc_out sums over the whole sequence.
  if (tid < 32) semx::tc::tmem_alloc(reinterpret_cast<uint32_t*>(sm + TcBLay::tslot), 64);
  if (tid == 0) {
    semx::tc::mbar_init(bar_adj, 1);
    semx::tc::mbar_init(bar_dc, 1);
  }
  semx::tc::fence_before_sync();
  __syncthreads();
  semx::tc::fence_after_sync();
  const uint32_t taddr = *reinterpret_cast<const uint32_t*>(sm + TcBLay::tslot);

  float2* lam = reinterpret_cast<float2*>(sm + TcBLay::lam);
  float2* braw = reinterpret_cast<float2*>(sm + TcBLay::braw);
  float2* gs = reinterpret_cast<float2*>(sm + TcBLay::gs);
  float2* db = reinterpret_cast<float2*>(sm + TcBLay::db);
  float2* cin = reinterpret_cast<float2*>(sm + TcBLay::cin);
  float2* cadj = reinterpret_cast<float2*>(sm + TcBLay::cadj);
  float2* hent = reinterpret_cast<float2*>(sm + TcBLay::hent);
  char* htile = reinterpret_cast<char*>(sm + TcBLay::ht);
  const int stg[2] = {TcBLay::stg0, TcBLay::stg1}, smlo[2] = {TcBLay::sml0, TcBLay::sml1};

  // Thread roles (fixed for the whole kernel).
  const int tA = tid / 8, npA = tid % 8;   // (token, mode pair) items
  const int rO = tid / FH, fO = tid % FH;  // dcout items (rank, channel) when R = 4
  float acc_a[2] = {0.f, 0.f}, acc_om[2] = {0.f, 0.f}, acc_sd[2] = {0.f, 0.f};
  float aO = 0.f, aD = 0.f;
  float aBnu = 0.f, aBth = 0.f;
  const float2 bias = dt_bias(p, h);
  const int nck = p.nck;
  uint32_t ph_adj = 0, ph_dc = 0;
  bool bail = false, adj_pending = false, dc_pending = false;
  float pre[kPre];
  auto stage = [&](int k, int b) {
    const int t0 = k * CT, nt = min(CT, L - t0);
    stage_bulk<true, 16, 32, RK>(p, fl, sm + stg[b], s, h, t0, nt);
  };
  if (nck > 0) {
    const int k = nck - 1, nt = min(CT, L - k * CT);
    stage(k, 0);
    load_small<true, RK>(p, s, h, k * CT, nt, bias, pre);
    store_small<RK, CT>(p, sm + smlo[0], nt, pre);
    // dy of the last tile, and of the previous tile's chunks whose rows the last tile
    // does not use.
    const int qlast = k & 3;
    for (int q = 0; q <= qlast; ++q) {
      const int kk = k - qlast + q;
      tcb_load_dy(p, sm, s, h, 16 * q, kk * CT, min(CT, L - kk * CT));
    }
    for (int q = qlast + 1; q < 4 && k - qlast - 4 + q >= 0; ++q) tcb_load_dy(p, sm, s, h, 16 * q, (k - qlast - 4 + q) * CT, CT);
  }
  cp_async_commit();
  int b = 0;
  for (int k = nck - 1; k >= 0; --k, b ^= 1) {
    const int q = k & 3;
    const int t0 = k * CT, nt = min(CT, L - t0);
    const bool tile_start = (k == nck - 1) || q == 3;
    const int row0 = 16 * q;  // this chunk's rows in the dy tile
    if (tile_start) cp_async_wait_all();
    else asm volatile("cp.async.wait_group 1;\n" ::: "memory");
    semx::tc::fence_smem_to_async();
    __syncthreads();
    if (tile_start && tid == 0) {  // readout adjoint of the tile: dy x [C_re | -C_im]^T
      constexpr uint32_t idesc = semx::tc::idesc_tf32(64, 32);
      const uint32_t a0 = semx::tc::smem_addr(sm + TcBLay::dyt), b0 = semx::tc::smem_addr(sm + TcBLay::bwt);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        semx::tc::mma_tf32(taddr, semx::tc::desc_sw128_kmajor(a0 + 32 * kk), semx::tc::desc_sw128_kmajor(b0 + 32 * kk),
                           idesc, kk > 0);
      semx::tc::mma_commit(bar_adj);
    }
    adj_pending = adj_pending || tile_start;
    if (k > 0) {
      stage(k - 1, b ^ 1);
      load_small<true, RK>(p, s, h, (k - 1) * CT, CT, bias, pre);
    }
    cp_async_commit();
    const T* xs = reinterpret_cast<const T*>(sm + stg[b]);
    const T* bxs = xs + CT * fl.xw;
    const T* bts = bxs + CT * fl.bxw;
    const T* cts = bts + CT * fl.btw;
    const float* sml = sm + smlo[b];
    const float* raws = sml;
    const float* dnus = sml + CT;
    const float* dths = sml + 2 * CT;
    const float* sbs = sml + 3 * CT;
    const float* scs = sbs + CT * R;
    const int xw = fl.xw, bxw = fl.bxw, btw = fl.btw, ctw = fl.ctw;

    // A. Poles, raw and gained drive per (token, mode pair); entry state. The chunk's dy
    // rows into the dC operand tile, one 16-byte piece per thread.
    {
      static_assert(kT == 16 * 8, "one dy piece per thread");
      const int t = tid >> 3, c = tid & 7;
      *reinterpret_cast<float4*>(reinterpret_cast<char*>(sm + TcBLay::dy32) + semx::tc::sw128_32b(t, 4 * c)) =
          *reinterpret_cast<const float4*>(reinterpret_cast<const char*>(sm + TcBLay::dyt) +
                                           semx::tc::sw128(row0 + t, c));
    }
    if (tid < NH) {
      const float2 c = reinterpret_cast<const float2*>(p.ckpt)[((s * nck + k) * p.H + h) * NH + tid];
      cin[tid] = c;
      hent[tid] = c;
    }
    if (tA < nt) {
      const int t = tA, na = 2 * npA;
      const float4 bq = ld4(bxs + t * bxw + 2 * na);
      float br0 = bq.x, bi0 = bq.y, br1 = bq.z, bi1 = bq.w;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float sbv = sbs[t * R + r];
        br0 = fmaf(sbv, static_cast<float>(bts[t * btw + r * NH + na]), br0);
        br1 = fmaf(sbv, static_cast<float>(bts[t * btw + r * NH + na + 1]), br1);
      }
#pragma unroll
      for (int dn = 0; dn < 2; ++dn) {
        const int n = na + dn;
        const float brv = dn ? br1 : br0, biv = dn ? bi1 : bi0;
        const MDisc d = mdisc(p.gain, sm[TcBLay::prm + n], sm[TcBLay::prm + NH + n], sm[TcBLay::prm + 2 * NH + n],
                              det, dnus[t], dths[t]);
        lam[t * HW + n] = make_float2(d.lre, d.lim);
        braw[t * HW + n] = make_float2(brv, biv);
        gs[t * HW + n] = make_float2(d.gr * brv - d.gi * biv, d.gr * biv + d.gi * brv);
      }
    }
    // The readout adjoint rows of this chunk (warp q, lanes 0..15) into db, which is free
    // until phase F; at a tile start, after its MMA (issued above) completes.
    if (tile_start) {
      const bool ok = semx::tc::mbar_wait(bar_adj, ph_adj, kTcWaitLimit);
      if (__syncthreads_or(!ok)) {
        if (tid == 0) atomicAdd(&g_tc_timeouts, 1u);
        bail = true;
        break;
      }
      ph_adj ^= 1u;
      adj_pending = false;
      semx::tc::fence_after_sync();
    }
    if (warp == q) {
      float acc[32];
      semx::tc::tmem_ld32(taddr + ((uint32_t)(32 * q) << 16), acc);
      if (lane < nt) {
#pragma unroll
        for (int n = 0; n < NH; ++n) db[lane * HW + n] = make_float2(acc[n], acc[16 + n]);
      }
    }
    semx::tc::fence_before_sync();
    __syncthreads();
    // B. States of the chunk from the checkpoint, into the h tile as [h_re | -h_im].
    chunk_scan_to<kB_SEG, CT>(lam, gs, cin, NH, HW, nt, [&](int t, int n, float2 v) {
      *reinterpret_cast<float*>(htile + semx::tc::sw128_32b(t, n)) = v.x;
      *reinterpret_cast<float*>(htile + semx::tc::sw128_32b(t, n + 16)) = -v.y;
    });
    __syncthreads();
    // C. Rank read and its adjoint per (token, rank), each item split over a thread pair
    // (modes 0-7 / 8-15 of the read, channels 0-15 / 16-31 of the adjoint) so that all
    // four warps share the phase; the halves are added with one shuffle.
    if (R > 0) {
      static_assert(R == 0 || kT >= 2 * CT * R, "two threads per (token, rank)");
      const int item = tid >> 1, half = tid & 1;
      const bool act = item < nt * R;
      const int t = item / (R > 0 ? R : 1), r = item % (R > 0 ? R : 1);
      float rd = 0.f, dyc = 0.f;
      if (act) {
        const T* cr = cts + t * ctw + r * 2 * NH;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int c4 = 2 * half + c;
          const float4 hre = *reinterpret_cast<const float4*>(htile + semx::tc::sw128_32b(t, 4 * c4));
          const float4 hni = *reinterpret_cast<const float4*>(htile + semx::tc::sw128_32b(t, 4 * c4 + 16));
          const float4 cre = ld4(cr + 4 * c4), cim = ld4(cr + NH + 4 * c4);
          rd = fmaf(cre.x, hre.x, fmaf(cim.x, hni.x, rd));
          rd = fmaf(cre.y, hre.y, fmaf(cim.y, hni.y, rd));
          rd = fmaf(cre.z, hre.z, fmaf(cim.z, hni.z, rd));
          rd = fmaf(cre.w, hre.w, fmaf(cim.w, hni.w, rd));
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int c4 = 4 * half + c;
          const float4 dv = *reinterpret_cast<const float4*>(reinterpret_cast<const char*>(sm + TcBLay::dyt) +
                                                             semx::tc::sw128(row0 + t, c4));
          const float* co = sm + TcBLay::Co + r * FH + 4 * c4;
          dyc = fmaf(dv.x, co[0], fmaf(dv.y, co[1], fmaf(dv.z, co[2], fmaf(dv.w, co[3], dyc))));
        }
      }
      rd += __shfl_xor_sync(0xffffffffu, rd, 1);
      dyc += __shfl_xor_sync(0xffffffffu, dyc, 1);
      if (act && half == 0) {
        const float scv = scs[t * R + r];
        sm[TcBLay::sr + item] = scv * rd;
        sm[TcBLay::dr + item] = scv * dyc;
        st<true>(p.dproj, (s * p.L + t0 + t) * p.P + cols.sc + r, rd * dyc);
      }
    }
    // The chunk's dC terms on the tensor cores, accumulated in tensor memory over the whole
    // sequence: D[m, f] += sum_t h[t, m] dy[t, f] (m < 32: h_re, -h_im), both tiles read
    // MN-major; one MMA per 8 tokens. Waited for at the end of the chunk, before the tiles
    // change.
    semx::tc::fence_smem_to_async();
    __syncthreads();
    if (tid == 0) {
      constexpr uint32_t idesc = semx::tc::idesc_tf32(64, 32, true);
      const uint32_t a0 = semx::tc::smem_addr(sm + TcBLay::ht), b0 = semx::tc::smem_addr(sm + TcBLay::dy32);
#pragma unroll
      for (int kk = 0; kk < 2; ++kk)
        semx::tc::mma_tf32(taddr + 32u, semx::tc::desc_sw128b32_mnmajor(a0 + 1024u * kk, 2048u),
                           semx::tc::desc_sw128b32_mnmajor(b0 + 1024u * kk, 2048u), idesc,
                           k < nck - 1 || kk > 0);
      semx::tc::mma_commit(bar_dc);
    }
    dc_pending = true;
    // D. Readout adjoint (drained into db after phase A) plus the rank terms, and the c_t
    // gradient, per (token, mode pair).
    if (tA < nt) {
      const int t = tA, na = 2 * npA;
      float2 g0 = db[t * HW + na], g1 = db[t * HW + na + 1];
      const float2 h0 = tcb_h(sm, t, na), h1 = tcb_h(sm, t, na + 1);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float drv = sm[TcBLay::dr + t * R + r];
        const T* cr = cts + t * ctw + r * 2 * NH;
        g0.x = fmaf(drv, static_cast<float>(cr[na]), g0.x);
        g1.x = fmaf(drv, static_cast<float>(cr[na + 1]), g1.x);
        g0.y = fmaf(-drv, static_cast<float>(cr[NH + na]), g0.y);
        g1.y = fmaf(-drv, static_cast<float>(cr[NH + na + 1]), g1.y);
        const int64_t row = (s * p.L + t0 + t) * p.P + cols.ct + (int64_t)r * 2 * NH;
        if ((p.vec & 32) != 0) {  // the mode pair's two columns as one 4-byte store each
          __nv_bfloat16* dp = reinterpret_cast<__nv_bfloat16*>(p.dproj);
          *reinterpret_cast<__nv_bfloat162*>(dp + row + na) = __floats2bfloat162_rn(drv * h0.x, drv * h1.x);
          *reinterpret_cast<__nv_bfloat162*>(dp + row + NH + na) = __floats2bfloat162_rn(-drv * h0.y, -drv * h1.y);
        } else {
          st<true>(p.dproj, row + na, drv * h0.x);
          st<true>(p.dproj, row + na + 1, drv * h1.x);
          st<true>(p.dproj, row + NH + na, -drv * h0.y);
          st<true>(p.dproj, row + NH + na + 1, -drv * h1.y);
        }
      }
      gs[t * HW + na] = g0;
      gs[t * HW + na + 1] = g1;
    }
    __syncthreads();
    // E. Adjoint scan: G over g, carry across chunks in cadj.
    chunk_scan_rev<kB_SEG, CT>(lam, gs, cadj, HW, nt);
    __syncthreads();
    // F. Through the gain and the pole per (token, mode pair).
    {
      float sdnu = 0.f, sdth = 0.f;
      if (tA < nt) {
        const int t = tA;
#pragma unroll
        for (int dn = 0; dn < 2; ++dn) {
          const int n = 2 * npA + dn;
          const float a = sm[TcBLay::prm + n], om = sm[TcBLay::prm + NH + n], sd = sm[TcBLay::prm + 2 * NH + n];
          const float dnu = dnus[t], dth = dths[t];
          const MDisc d = mdisc(p.gain, a, om, sd, det, dnu, dth);
          const float2 G = gs[t * HW + n], bv = braw[t * HW + n];
          const float2 hp = t == 0 ? hent[n] : tcb_h(sm, t > 0 ? t - 1 : 0, n);
          db[t * HW + n] = make_float2(d.gr * G.x + d.gi * G.y, d.gr * G.y - d.gi * G.x);
          const float dgr = bv.x * G.x + bv.y * G.y, dgi = bv.x * G.y - bv.y * G.x;
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
          sdnu += d_dnu;
          sdth += det ? dbase * sd : dbase;
          acc_a[dn] += da_extra - dnu * P;
          acc_om[dn] += dbase;
          acc_sd[dn] += det ? dbase * dth : 0.f;
        }
      }
#pragma unroll
      for (int m = 1; m < 8; m <<= 1) {
        sdnu += __shfl_xor_sync(0xffffffffu, sdnu, m);
        sdth += __shfl_xor_sync(0xffffffffu, sdth, m);
      }
      if (npA == 0 && tA < nt) {
        const int64_t row = (s * p.L + t0 + tA) * p.P;
        const float draw = sdnu * p.rs * semx::softplus_grad(raws[tA]);
        st<true>(p.dproj, row + cols.dnu, draw);
        st<true>(p.dproj, row + cols.dth, sdth);
        aBnu += draw;
        aBth += sdth;
      }
    }
    __syncthreads();
    // G. dx = D dy per (token, 4 channels); d(drive columns) = d(raw drive) of the token's
    // mode pair.
    if (tA < nt) {
      const int t = tA, f0 = 4 * npA, na = 2 * npA;
      const float4 dv = *reinterpret_cast<const float4*>(reinterpret_cast<const char*>(sm + TcBLay::dyt) +
                                                         semx::tc::sw128(row0 + t, npA));
      float4 acc;
      acc.x = sm[TcBLay::Dp + f0] * dv.x;
      acc.y = sm[TcBLay::Dp + f0 + 1] * dv.y;
      acc.z = sm[TcBLay::Dp + f0 + 2] * dv.z;
      acc.w = sm[TcBLay::Dp + f0 + 3] * dv.w;
      const float2 g0 = db[t * HW + na], g1 = db[t * HW + na + 1];
      const int64_t drow = (s * p.L + t0 + t) * p.P + cols.bx + 2 * na;
      if ((p.vec & 16) != 0) {
        __nv_bfloat162 qv[2] = {__floats2bfloat162_rn(g0.x, g0.y), __floats2bfloat162_rn(g1.x, g1.y)};
        *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p.dproj) + drow) = *reinterpret_cast<const uint2*>(qv);
      } else {
        st<true>(p.dproj, drow, g0.x);
        st<true>(p.dproj, drow + 1, g0.y);
        st<true>(p.dproj, drow + 2, g1.x);
        st<true>(p.dproj, drow + 3, g1.y);
      }
      const int64_t xo = (s * p.L + t0 + t) * Fd + (int64_t)h * FH + f0;
      if ((p.vec & 8) != 0) {
        __nv_bfloat162 qv[2] = {__floats2bfloat162_rn(acc.x, acc.y), __floats2bfloat162_rn(acc.z, acc.w)};
        *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p.dx) + xo) = *reinterpret_cast<const uint2*>(qv);
      } else {
        st<true>(p.dx, xo, acc.x);
        st<true>(p.dx, xo + 1, acc.y);
        st<true>(p.dx, xo + 2, acc.z);
        st<true>(p.dx, xo + 3, acc.w);
      }
    }
    // H. Rank write: d s_b, d b_t; a thread pair per (token, rank), each thread 8 of the 16
    // b_t columns (one 16-byte store), the two halves of d s_b added with one shuffle.
    if (R > 0) {
      const int item = tid >> 1, half = tid & 1;
      const bool act = item < nt * R;
      const int t = item / (R > 0 ? R : 1), r = item % (R > 0 ? R : 1);
      float acc = 0.f;
      if (act) {
        const float sbv = sbs[t * R + r];
        const int64_t row = (s * p.L + t0 + t) * p.P;
        __nv_bfloat16* dp = reinterpret_cast<__nv_bfloat16*>(p.dproj) + row + cols.bt + r * NH;
        const int n8 = 8 * half;
        __nv_bfloat162 q[4];
#pragma unroll
        for (int n = n8; n < n8 + 8; n += 2) {
          const float g0 = db[t * HW + n].x, g1 = db[t * HW + n + 1].x;
          acc = fmaf(static_cast<float>(bts[t * btw + r * NH + n]), g0, acc);
          acc = fmaf(static_cast<float>(bts[t * btw + r * NH + n + 1]), g1, acc);
          q[(n - n8) / 2] = __floats2bfloat162_rn(sbv * g0, sbv * g1);
        }
        if ((p.vec & 32) != 0) {
          *reinterpret_cast<uint4*>(dp + n8) = *reinterpret_cast<const uint4*>(q);
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            dp[n8 + 2 * i] = q[i].x;
            dp[n8 + 2 * i + 1] = q[i].y;
          }
        }
      }
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      if (act && half == 0) st<true>(p.dproj, (s * p.L + t0 + t) * p.P + cols.sb + r, acc);
    }
    // I. dc_out and dD sums over the chunk, fixed ownership.
    for (int t = 0; t < nt; ++t) {
      if (R > 0) aO = fmaf(sm[TcBLay::sr + t * R + rO], tcb_dy(sm, row0 + t, fO), aO);
      if (tid < FH) aD = fmaf(tcb_dy(sm, row0 + t, tid), static_cast<float>(xs[t * xw + tid]), aD);
    }
    if (k > 0) store_small<RK, CT>(p, sm + smlo[b ^ 1], CT, pre);
    // Every thread is past its reads of the chunk's dy rows, and the dC MMA is done with
    // the h and dy32 tiles: refill the dy rows with the same chunk of the previous tile.
    {
      const bool ok = semx::tc::mbar_wait(bar_dc, ph_dc, kTcWaitLimit);
      if (__syncthreads_or(!ok)) {
        if (tid == 0) atomicAdd(&g_tc_timeouts, 1u);
        bail = true;
        break;
      }
      ph_dc ^= 1u;
      dc_pending = false;
    }
    if (k >= 4) tcb_load_dy(p, sm, s, h, row0, (k - 4) * CT, CT);
    cp_async_commit();
  }
  cp_async_wait_all();
  __syncthreads();
  const int64_t H = p.H;
  float* row = p.part + s * p.K;
  if (!bail) {
    // dC from tensor memory: accumulator row m is read by lane m % 16 of warp m / 16
    // (rows 0-15: dC_re, 16-31: dC_im of mode m % 16), its 32 columns being the channels.
    semx::tc::fence_after_sync();
    if (warp < 2) {
      float v[32];
      semx::tc::tmem_ld32(taddr + 32u + ((uint32_t)(32 * warp) << 16), v);
      if (lane < NH) {
#pragma unroll
        for (int f = 0; f < FH; ++f) row[2 * (((int64_t)h * FH + f) * NH + lane) + warp] = nck > 0 ? v[f] : 0.f;
      }
    }
    // Per-mode sums over the 16 token lanes that share a mode pair, fixed order.
    float* red = sm + TcBLay::red;  // [3][NH][kT / 8]
#pragma unroll
    for (int dn = 0; dn < 2; ++dn) {
      const int n = 2 * npA + dn;
      red[(0 * NH + n) * (kT / 8) + tA] = acc_a[dn];
      red[(1 * NH + n) * (kT / 8) + tA] = acc_om[dn];
      red[(2 * NH + n) * (kT / 8) + tA] = acc_sd[dn];
    }
    if (npA == 0) {
      sm[TcBLay::rb + tA] = aBnu;
      sm[TcBLay::rb + kT / 8 + tA] = aBth;
    }
    __syncthreads();
    // Partial row of sequence s: [dC | dcout | dD | dA_log | domega | ddetune | d dt bias].
    int64_t off = H * FH * NH * 2;
    if (R > 0) {
      row[off + (int64_t)h * R * FH + rO * FH + fO] = aO;
      off += H * R * FH;
    }
    if (tid < FH) row[off + (int64_t)h * FH + tid] = aD;
    off += H * FH;
    if (tid < 3 * NH) {
      const int which = tid / NH, n = tid % NH;
      float acc = 0.f;
      for (int qq = 0; qq < kT / 8; ++qq) acc += red[(which * NH + n) * (kT / 8) + qq];
      if (which == 0) acc *= sm[TcBLay::prm + n];  // d/dA_log = a d/da
      row[off + which * H * NH + (int64_t)h * NH + n] = acc;
    }
    off += 3 * H * NH;
    if (tid < 2) {
      float acc = 0.f;
      for (int qq = 0; qq < kT / 8; ++qq) acc += sm[TcBLay::rb + tid * (kT / 8) + qq];
      row[off + tid * H + h] = acc;
    }
  } else {
    // After a give-up, let the outstanding MMAs finish (bounded) before the tensor memory
    // they write is released.
    if (adj_pending) semx::tc::mbar_wait(bar_adj, ph_adj, kTcWaitLimit);
    if (dc_pending) semx::tc::mbar_wait(bar_dc, ph_dc, kTcWaitLimit);
  }
  semx::tc::fence_before_sync();
  __syncthreads();
  if (tid < 32) semx::tc::tmem_dealloc(taddr, 64);
}

// ------------------------------------------------------------------------ host side
int64_t proj_width(const SemxMimoLayerArgs* a) {
  return 2 * a->H + (a->rank > 0 ? 2 * a->H * a->rank + 3 * a->H * a->rank * a->Nh : 0) + 2 * a->H * a->Nh;
}

int64_t part_row(const SemxMimoLayerArgs* a) {
  const int64_t H = a->H, Nh = a->Nh, Fh = a->Fh, R = a->rank;
  return H * (2 * Nh * Fh + (a->envelope ? Fh * Nh : 0) + R * Fh + Fh + 3 * Nh + 2);
}

// The backward of 16-mode, 32-channel heads of rank 0 or 4 has its own kernel.
bool bwd16(const SemxMimoLayerArgs* a) { return a->Nh == 16 && a->Fh == 32 && (a->rank == 0 || a->rank == 4); }

// The forward of 16-mode, 32-channel heads (rank 0 or 4) runs 16-token chunks.
int fwd_chunk(const SemxMimoLayerArgs* a) { return bwd16(a) ? kCk : kTC; }

// The bf16 forward of those heads without the envelope readout reads out on the tensor
// cores (mimo_layer_fwd_tc_kernel: 16-byte aligned x and y rows).
bool fwd_tc(const SemxMimoLayerArgs* a) {
  return bwd16(a) && a->bf16 && !a->envelope && semx::aligned(a->y, 16) && semx::aligned(a->x, 16);
}

// The bf16 backward of those heads without the envelope readout runs its contractions on
// the tensor cores (mimo_layer_bwd_tc_kernel).
bool bwd_tc(const SemxMimoLayerArgs* a) { return bwd16(a) && a->bf16 && !a->envelope; }

size_t layer_smem(const SemxMimoLayerArgs* a, bool bwd) {
  if (bwd && bwd_tc(a)) return (size_t)TcBLay::total * sizeof(float);
  if (bwd && bwd16(a)) return (size_t)make_blay(a->rank, a->envelope != 0, a->bf16 ? 2 : 4).total * sizeof(float);
  if (!bwd && fwd_tc(a)) return (size_t)TcLay::total * sizeof(float);
  if (!bwd)
    return (size_t)make_flay((int)a->Nh, (int)a->Fh, a->rank, a->envelope != 0, a->bf16 ? 2 : 4, fwd_chunk(a))
               .total * sizeof(float);
  return (size_t)make_lay((int)a->Nh, (int)a->Fh, a->rank, bwd, a->envelope != 0).total * sizeof(float);
}

// Which operand rows allow 16-byte staging copies (LParams::vec).
int vec_flags(const SemxMimoLayerArgs* a) {
  const int64_t es = a->bf16 ? 2 : 4, H = a->H, R = a->rank, Nh = a->Nh, Fh = a->Fh;
  const int64_t P = proj_width(a);
  const bool vx = semx::aligned(a->x, 16) && (H * Fh * es) % 16 == 0 && (Fh * es) % 16 == 0;
  const bool vp = semx::aligned(a->proj, 16) && (P * es) % 16 == 0 && ((2 * H + H * R) * es) % 16 == 0 &&
                  ((R * Nh * es) % 16) == 0 && ((2 * H + 2 * H * R + H * R * Nh) * es) % 16 == 0;
  const bool vdy = semx::aligned(a->dy, 16) && (H * Fh * 4) % 16 == 0 && (Fh * 4) % 16 == 0;
  const bool vdx = semx::aligned(a->dx, 16) && Fh % 4 == 0;
  const int64_t bx0 = 2 * H + 2 * H * R + 3 * H * R * Nh;
  const bool vbx = semx::aligned(a->proj, 16) && (a->dproj == nullptr || semx::aligned(a->dproj, 16)) &&
                   (P * es) % 16 == 0 && (bx0 * es) % 16 == 0 && (2 * Nh * es) % 16 == 0;
  // dproj rows whose b_t columns of one (head, rank) start on 16 bytes and whose c_t mode
  // pairs start on 4 bytes (the tensor-core backward's vector stores).
  const int64_t bt0 = 2 * H + H * R, ct0 = 2 * H + 2 * H * R + H * R * Nh;
  const bool vdp = a->dproj != nullptr && semx::aligned(a->dproj, 16) && (P * es) % 16 == 0 &&
                   (bt0 * es) % 16 == 0 && (Nh * es) % 16 == 0 && (ct0 * es) % 4 == 0 && Nh % 2 == 0;
  return (vx ? 1 : 0) | (vp ? 2 : 0) | (vdy ? 4 : 0) | (vdx ? 8 : 0) | (vbx ? 16 : 0) | (vdp ? 32 : 0);
}

// Segments per mode of the forward's parallel chunk scan (1: one thread per mode).
int scan_segments(int64_t Nh) {
  if (Nh <= 0 || kT % Nh != 0) return 1;
  const int seg = kT / (int)Nh;
  return (seg <= 32 && kTC % seg == 0) ? seg : 1;
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
    SEMX_REQUIRE(a->A_log && a->omega && a->C && a->D, SEMX_ERR_NULL, "mimo_layer: NULL parameter");
    SEMX_REQUIRE(!a->detune || a->detune_gain, SEMX_ERR_NULL, "mimo_layer: detune_gain is NULL");
    SEMX_REQUIRE(!a->envelope || a->env_gain, SEMX_ERR_NULL, "mimo_layer: env_gain is NULL");
    SEMX_REQUIRE(a->rank == 0 || a->c_out, SEMX_ERR_NULL, "mimo_layer: c_out is NULL");
    SEMX_REQUIRE(semx::aligned(a->C, 8), SEMX_ERR_ALIGN, "mimo_layer: C must be 8-byte aligned");
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
  p.nck = (int)semx::cdiv(a->L, kCk);
  p.rs = a->rate_scale;
  p.x = a->x; p.proj = a->proj;
  p.A_log = a->A_log; p.omega = a->omega; p.sdet = a->detune_gain; p.C = a->C; p.D = a->D;
  p.cout = a->c_out; p.env = a->env_gain; p.dtb = a->dt_bias;
  p.y = a->y; p.ckpt = a->ckpt; p.dy = a->dy; p.dx = a->dx; p.dproj = a->dproj;
  p.K = part_row(a);
  p.vec = vec_flags(a);
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

int semx_tc_timeouts(uint32_t* count) {
  SEMX_REQUIRE(count != nullptr, SEMX_ERR_NULL, "semx_tc_timeouts: count is NULL");
  unsigned int v = 0;
  const cudaError_t e = cudaMemcpyFromSymbol(&v, g_tc_timeouts, sizeof(v));
  if (e != cudaSuccess) return semx::fail(SEMX_ERR_LAUNCH, "semx_tc_timeouts: %s", cudaGetErrorString(e));
  *count = v;
  return SEMX_OK;
}

size_t semx_mimo_layer_args_size(void) { return sizeof(SemxMimoLayerArgs); }

size_t semx_mimo_layer_ckpt_bytes(const SemxMimoLayerArgs* a) {
  if (a == nullptr || a->S < 0 || a->L < 0 || a->H < 0 || a->Nh < 0) return 0;
  return (size_t)a->S * (size_t)semx::cdiv(a->L, kCk) * (size_t)(a->H * a->Nh) * 2 * sizeof(float);
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
  const int seg = scan_segments(a->Nh);
  if (fwd_tc(a)) {
    static_assert(kCk == 16, "the tensor-core forward writes one checkpoint per 16-token chunk");
    return a->rank == 4 ? launch_layer(mimo_layer_fwd_tc_kernel<4>, p, smem, st, "mimo_layer_fwd_tc_kernel")
                        : launch_layer(mimo_layer_fwd_tc_kernel<0>, p, smem, st, "mimo_layer_fwd_tc_kernel");
  }
  if (bwd16(a)) {
    // The 16-mode, 32-channel heads, specialised at compile time, 16-token chunks.
    static_assert(kCk % 8 == 0, "16-token chunks hold whole 8-segment scans");
    if (a->rank == 4)
      return a->bf16 ? launch_layer(mimo_layer_fwd_kernel<true, 8, 16, 32, 4, kCk>, p, smem, st, "mimo_layer_fwd_kernel")
                     : launch_layer(mimo_layer_fwd_kernel<false, 8, 16, 32, 4, kCk>, p, smem, st, "mimo_layer_fwd_kernel");
    return a->bf16 ? launch_layer(mimo_layer_fwd_kernel<true, 8, 16, 32, 0, kCk>, p, smem, st, "mimo_layer_fwd_kernel")
                   : launch_layer(mimo_layer_fwd_kernel<false, 8, 16, 32, 0, kCk>, p, smem, st, "mimo_layer_fwd_kernel");
  }
  switch (seg) {
#define SEMX_SEG(SV)                                                                                  \
  case SV:                                                                                            \
    return a->bf16                                                                                    \
               ? launch_layer(mimo_layer_fwd_kernel<true, SV, 0, 0, -1>, p, smem, st, "mimo_layer_fwd_kernel") \
               : launch_layer(mimo_layer_fwd_kernel<false, SV, 0, 0, -1>, p, smem, st, "mimo_layer_fwd_kernel");
    SEMX_SEG(2)
    SEMX_SEG(4)
    SEMX_SEG(8)
    SEMX_SEG(16)
    SEMX_SEG(32)
#undef SEMX_SEG
    default:
      return a->bf16 ? launch_layer(mimo_layer_fwd_kernel<true, 1, 0, 0, -1>, p, smem, st, "mimo_layer_fwd_kernel")
                     : launch_layer(mimo_layer_fwd_kernel<false, 1, 0, 0, -1>, p, smem, st, "mimo_layer_fwd_kernel");
  }
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
    if (bwd_tc(a)) {
      rc = a->rank == 4 ? launch_layer(mimo_layer_bwd_tc_kernel<4>, p, smem, st, "mimo_layer_bwd_tc_kernel")
                        : launch_layer(mimo_layer_bwd_tc_kernel<0>, p, smem, st, "mimo_layer_bwd_tc_kernel");
    } else if (bwd16(a)) {
      if (a->rank == 4)
        rc = a->bf16 ? launch_layer(mimo_layer_bwd16_kernel<true, 4>, p, smem, st, "mimo_layer_bwd16_kernel")
                     : launch_layer(mimo_layer_bwd16_kernel<false, 4>, p, smem, st, "mimo_layer_bwd16_kernel");
      else
        rc = a->bf16 ? launch_layer(mimo_layer_bwd16_kernel<true, 0>, p, smem, st, "mimo_layer_bwd16_kernel")
                     : launch_layer(mimo_layer_bwd16_kernel<false, 0>, p, smem, st, "mimo_layer_bwd16_kernel");
    } else {
      rc = a->bf16 ? launch_layer(mimo_layer_bwd_kernel<true>, p, smem, st, "mimo_layer_bwd_kernel")
                   : launch_layer(mimo_layer_bwd_kernel<false>, p, smem, st, "mimo_layer_bwd_kernel");
    }
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
  add(a->dC, H * Fh * Nh * 2);
  if (a->envelope) add(a->denv, H * Fh * Nh);
  if (R > 0) add(a->dc_out, H * R * Fh);
  add(a->dD, H * Fh);
  add(a->dA_log, H * Nh);
  add(a->domega, H * Nh);
  add(a->detune ? a->ddetune : nullptr, H * Nh);
  add(a->dt_bias ? a->d_dt_bias : nullptr, 2 * H);
  seg.n = n;
  return semx::colsum(ws, a->S, p.K, ws + (size_t)a->S * p.K, seg, st);
}

}  // extern "C"
