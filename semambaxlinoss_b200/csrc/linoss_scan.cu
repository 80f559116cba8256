// LinOSS oscillatory scan, forward and backward, for sm_100a.
//
// Reference behaviour (paths relative to the reference project):
//   recurrence      models/linoss/linoss.py:155-180  (_linoss_recurrence)
//   discretisations models/linoss/linoss.py:183-232  (IM, IMEX, damped IMEX)
//   constraints     models/linoss/linoss.py:81-116   (sigmoid steps, relu / clamp bands)
//   generic op      models/linoss/triton.py:195-294  (M11..M22, F1, F2 -> Y2)
//
// Layout. One thread owns one (sequence s, oscillator p) chain; the flat thread index is
// s * P + p, so a warp reads 32 consecutive oscillators of the same time step (256 B of
// interleaved complex64). The state (y1, y2) is 2 complex numbers in registers. The loop
// over time is sequential; loads are issued one 8-step batch ahead of the arithmetic so
// every thread keeps 8 loads in flight.
//
// Forward (training) additionally stores the state entering every `chunk`-step block
// and the final state (16 B per chunk and chain). The backward runs the adjoint
//   a_t = (0, dY2_t) + M^T a_{t+1},  dF_t = a_t,  dM_ij += Re(a_i,t conj(s_j,t-1))
// backwards in time and needs the forward states s_{t-1}; no per-step state goes to HBM.
// linoss_bwd_kernel takes one of two paths per thread block:
//   * IMEX (rev_block): M has determinant 1 (the scheme is symplectic), so the state is
//     run backwards with the adjoint, s_{t-1} = M^-1 (s_t - F_t), from each chunk's end
//     state and reset to the exact checkpoint at every chunk start. With both eigenvalues
//     on the unit circle (trace > -2) this is as accurate as re-running the recurrence; a
//     block holding an oscillator outside that range (step^2 A near or above 4, where the
//     reversal amplifies rounding) takes the other path.
//   * otherwise (bwd_block): for each chunk, re-run the recurrence once from the
//     checkpoint, dropping the state every kSub steps into shared memory; then for each
//     kSub-step sub-block (last first) recompute the kSub states into registers and run
//     the adjoint through them.
// Both paths need the same 48 KB of shared memory at the default chunk of 64 steps, and 4
// blocks of 128 threads fit an SM either way.
// Per-oscillator parameter gradients are summed per chain in registers, written once per
// chain, and reduced over sequences by linoss_finalize_kernel in a fixed order (bitwise
// deterministic), which also applies the chain rule from (M, f) back to the raw
// parameters.
#include <algorithm>
#include <mutex>

#include "semx_common.cuh"

namespace {

constexpr int kBlock = 128;  // threads per CTA (scan kernels)
constexpr int kSub = 8;      // steps per register-resident sub-block
constexpr int kMaxChunk = 256;
constexpr int kPartials = 6;  // dM11, dM12, dM21, dM22, df1, df2
constexpr int kLook = 8;      // steps per staged batch of the reversal backward
constexpr int kStages = 3;    // staged batches in flight (reversal backward)
static_assert(kSub % kLook == 0, "chunk (a multiple of kSub) must be a multiple of kLook");
// Reversal backward only for transitions with trace above this (IMEX: step^2 A < 3.99).
constexpr float kRevTraceMin = -1.99f;

struct Coef {
  float m11, m12, m21, m22;  // transition
  float f1, f2;              // F1 = f1 * Bu, F2 = f2 * Bu (fused variants)
};

struct Params {
  int variant, a_from_g, chunk, nchunks;
  int64_t S, L, P;
  const float* M11;
  const float* M12;
  const float* M21;
  const float* M22;
  const float2* F1;
  const float2* F2;
  const float* steps;
  const float* A_diag;
  const float* G_diag;
  const float2* Bu;
  float2* Y2;
  float4* ckpt;
  const float2* dY2;
  float2* dF1;
  float2* dF2;
  float2* dBu;
  float* dM;
  float* dparams;
  float* part;  // (S, kPartials, P)
  int rev;      // 1: step t of a chain is row L - 1 - t of its sequence (kernels take it as REV)
  // Checkpoint slot j of chain (s, o) at ckpt[(s * (nchunks + 1) + j) * P + o]: the state
  // entering chunk j; slot nchunks is the final state.
};

__host__ __device__ inline int64_t ckpt_index(const Params& p, int64_t s, int j, int o) {
  return (s * (p.nchunks + 1) + j) * p.P + o;
}

__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float relu_f(float x) { return x > 0.0f ? x : 0.0f; }

// Per-oscillator constraint chain and discretisation, evaluated in the same order as the
// reference's tensor expressions (models/linoss/linoss.py:82-116, 183-232).
__device__ __forceinline__ Coef make_coef(int variant, int a_from_g, float sraw, float araw,
                                          float graw) {
  Coef k;
  const float step = sigmoid_f(sraw);
  const float st2 = step * step;
  if (variant == SEMX_LINOSS_IM) {
    const float A = relu_f(araw);
    const float schur = 1.0f / (1.0f + st2 * A);
    k.m11 = 1.0f - st2 * A * schur;
    k.m12 = -step * A * schur;
    k.m21 = step * schur;
    k.m22 = schur;
    k.f1 = k.m11 * step;
    k.f2 = k.m21 * step;
  } else if (variant == SEMX_LINOSS_IMEX) {
    const float A = relu_f(araw);
    k.m11 = 1.0f;
    k.m12 = -step * A;
    k.m21 = step;
    k.m22 = 1.0f - st2 * A;
    k.f1 = step;
    k.f2 = st2;
  } else {  // DAMPED_IMEX
    float A, G;
    if (a_from_g) {
      G = relu_f(graw);
      const float sq = sqrtf(1.0f + step * G);
      const float A_low = (2.0f + step * G - 2.0f * sq) / st2;
      const float A_high = (2.0f + step * G + 2.0f * sq) / st2;
      A = A_low + relu_f(araw - A_low) - relu_f(araw - A_high);
    } else {
      A = relu_f(araw);
      const float sA = sqrtf(A);
      const float G_low = relu_f(step * A - 2.0f * sA);
      const float G_high = step * A + 2.0f * sA;
      G = fminf(fmaxf(graw, G_low), G_high);
    }
    const float inv = 1.0f / (1.0f + step * G);
    k.m11 = inv;
    k.m12 = -step * inv * A;
    k.m21 = step * inv;
    k.m22 = 1.0f - st2 * inv * A;
    k.f1 = step * inv;
    k.f2 = st2 * inv;
  }
  return k;
}

__device__ __forceinline__ Coef load_coef(const Params& p, int o) {
  if (p.variant == SEMX_LINOSS_GENERIC) {
    Coef k;
    k.m11 = p.M11[o];
    k.m12 = p.M12[o];
    k.m21 = p.M21[o];
    k.m22 = p.M22[o];
    k.f1 = 1.0f;
    k.f2 = 1.0f;
    return k;
  }
  const float graw = (p.variant == SEMX_LINOSS_DAMPED_IMEX) ? p.G_diag[o] : 0.0f;
  return make_coef(p.variant, p.a_from_g, p.steps[o], p.A_diag[o], graw);
}

// One recurrence step. s = (y1.re, y1.im, y2.re, y2.im); forcing F1 = u1, F2 = u2.
__device__ __forceinline__ float4 lin_step(const Coef& k, float4 s, float2 u1, float2 u2) {
  float4 n;
  n.x = k.m11 * s.x + k.m12 * s.z + u1.x;
  n.y = k.m11 * s.y + k.m12 * s.w + u1.y;
  n.z = k.m21 * s.x + k.m22 * s.z + u2.x;
  n.w = k.m21 * s.y + k.m22 * s.w + u2.y;
  return n;
}

template <bool GENERIC>
__device__ __forceinline__ void forcing(const Coef& k, float2 in1, float2 in2, float2& u1,
                                        float2& u2) {
  if (GENERIC) {
    u1 = in1;
    u2 = in2;
  } else {
    u1 = make_float2(k.f1 * in1.x, k.f1 * in1.y);
    u2 = make_float2(k.f2 * in1.x, k.f2 * in1.y);
  }
}

// Per-thread views of the (S, L, P) complex tensors: element (s, t, p) of a chain lives at
// chain_base + t * P, with 32-bit step offsets (L * P < 2^31 is validated on the host).
template <bool GENERIC>
__device__ __forceinline__ void load_batch(const float2* __restrict__ src1,
                                           const float2* __restrict__ src2, int P, int t0,
                                           int tend, float2 (&a)[kSub], float2 (&b)[kSub]) {
#pragma unroll
  for (int i = 0; i < kSub; ++i) {
    if (t0 + i < tend) {
      a[i] = __ldg(src1 + (t0 + i) * P);
      if (GENERIC) b[i] = __ldg(src2 + (t0 + i) * P);
    }
  }
}

__device__ __forceinline__ void cp_async8(void* smem, const void* gmem) {
  const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

template <bool GENERIC, bool REV>
__global__ void __launch_bounds__(kBlock) linoss_fwd_kernel(const Params p) {
  const int64_t gid = (int64_t)blockIdx.x * kBlock + threadIdx.x;
  if (gid >= p.S * p.P) return;
  const int64_t s = gid / p.P;
  const int o = (int)(gid - s * p.P);
  const Coef k = load_coef(p, o);
  const int L = (int)p.L;
  const int P = REV ? -(int)p.P : (int)p.P;  // step stride; negative when scanning backwards
  const int64_t base = s * p.L * p.P + o + (REV ? (p.L - 1) * p.P : 0);
  const float2* src1 = (GENERIC ? p.F1 : p.Bu) + base;
  const float2* src2 = GENERIC ? p.F2 + base : nullptr;
  float2* y2 = p.Y2 + base;

  float4 st = make_float4(0.f, 0.f, 0.f, 0.f);
  float2 c1[kSub], c2[kSub];
  load_batch<GENERIC>(src1, src2, P, 0, L, c1, c2);
  for (int t0 = 0; t0 < L; t0 += kSub) {
    float2 n1[kSub], n2[kSub];
    load_batch<GENERIC>(src1, src2, P, t0 + kSub, L, n1, n2);
    if (p.ckpt != nullptr && (t0 % p.chunk) == 0) p.ckpt[ckpt_index(p, s, t0 / p.chunk, o)] = st;
#pragma unroll
    for (int i = 0; i < kSub; ++i) {
      if (t0 + i < L) {
        float2 u1, u2;
        forcing<GENERIC>(k, c1[i], c2[i], u1, u2);
        st = lin_step(k, st, u1, u2);
        y2[(t0 + i) * P] = make_float2(st.z, st.w);
      }
    }
#pragma unroll
    for (int i = 0; i < kSub; ++i) {
      c1[i] = n1[i];
      c2[i] = n2[i];
    }
  }
  if (p.ckpt != nullptr) p.ckpt[ckpt_index(p, s, p.nchunks, o)] = st;
}

// Shared memory of the backward kernel, per thread (kBlock threads, slot = threadIdx.x):
//   sub_ckpt[chunk / kSub]    float4  states at the start of each sub-block
//   in[2][GENERIC ? 2 : 1][kSub] float2  double-buffered forcing / Bu of a sub-block
//   dy[2][kSub]               float2  double-buffered dY2 of a sub-block
// Every thread only touches its own slots, so no block barrier is needed; cp.async
// copies are made visible to the issuing thread by cp.async.wait_group.
template <bool GENERIC>
__device__ __forceinline__ void prefetch_sub(float2* in_buf, float2* dy_buf,
                                             const float2* src1, const float2* src2,
                                             const float2* dys, int P, int ta, int t1) {
#pragma unroll
  for (int i = 0; i < kSub; ++i) {
    if (ta + i < t1) {
      cp_async8(in_buf + i * kBlock, src1 + (ta + i) * P);
      if (GENERIC) cp_async8(in_buf + (kSub + i) * kBlock, src2 + (ta + i) * P);
      cp_async8(dy_buf + i * kBlock, dys + (ta + i) * P);
    }
  }
}

// The chains of thread block `blk` (kBlock consecutive chains).
template <bool GENERIC, bool REV>
__device__ __forceinline__ void bwd_block(const Params& p, int blk, float4* smem4) {
  constexpr int kIn = GENERIC ? 2 : 1;
  const int nsub_max = p.chunk / kSub;
  float4* sub_ckpt = smem4;                                            // [nsub_max][kBlock]
  float2* in_base = reinterpret_cast<float2*>(smem4 + nsub_max * kBlock);  // [2][kIn*kSub][kBlock]
  float2* dy_base = in_base + 2 * kIn * kSub * kBlock;                     // [2][kSub][kBlock]
  const int tid = threadIdx.x;

  const int64_t gid = (int64_t)blk * kBlock + tid;
  if (gid >= p.S * p.P) return;
  const int64_t s = gid / p.P;
  const int o = (int)(gid - s * p.P);
  const Coef k = load_coef(p, o);
  const int L = (int)p.L;
  const int P = REV ? -(int)p.P : (int)p.P;  // step stride; negative when scanning backwards
  const int64_t base = s * p.L * p.P + o + (REV ? (p.L - 1) * p.P : 0);
  const float2* src1 = (GENERIC ? p.F1 : p.Bu) + base;
  const float2* src2 = GENERIC ? p.F2 + base : nullptr;
  const float2* dys = p.dY2 + base;
  float2* out1 = (GENERIC ? p.dF1 : p.dBu) + base;
  float2* out2 = GENERIC ? p.dF2 + base : nullptr;

  float a1r = 0.f, a1i = 0.f, a2r = 0.f, a2i = 0.f;  // adjoint a_{t+1}
  float g11 = 0.f, g12 = 0.f, g21 = 0.f, g22 = 0.f, gf1 = 0.f, gf2 = 0.f;

  for (int c = p.nchunks - 1; c >= 0; --c) {
    const int t0 = c * p.chunk;
    const int t1 = min(t0 + p.chunk, L);
    const int nsub = (t1 - t0 + kSub - 1) / kSub;
    // Start fetching the last sub-block of this chunk while pass 1 runs.
    prefetch_sub<GENERIC>(in_base + tid, dy_base + tid, src1, src2, dys, P,
                          t0 + (nsub - 1) * kSub, t1);
    cp_async_commit();

    // Pass 1: recurrence over the chunk, keeping the state every kSub steps on chip.
    {
      float4 st = p.ckpt[ckpt_index(p, s, c, o)];
      float2 c1[kSub], c2[kSub];
      load_batch<GENERIC>(src1, src2, P, t0, t1, c1, c2);
      for (int tb = t0; tb < t1; tb += kSub) {
        float2 n1[kSub], n2[kSub];
        load_batch<GENERIC>(src1, src2, P, tb + kSub, t1, n1, n2);
        sub_ckpt[((tb - t0) / kSub) * kBlock + tid] = st;
#pragma unroll
        for (int i = 0; i < kSub; ++i) {
          if (tb + i < t1) {
            float2 u1, u2;
            forcing<GENERIC>(k, c1[i], c2[i], u1, u2);
            st = lin_step(k, st, u1, u2);
          }
        }
#pragma unroll
        for (int i = 0; i < kSub; ++i) {
          c1[i] = n1[i];
          c2[i] = n2[i];
        }
      }
    }

    // Pass 2: sub-blocks last to first; recompute kSub states into registers from the
    // sub-block checkpoint, then run the adjoint backwards through them.
    for (int r = nsub - 1; r >= 0; --r) {
      const int buf = (nsub - 1 - r) & 1;
      const int ta = t0 + r * kSub;
      if (r > 0) {
        prefetch_sub<GENERIC>(in_base + (buf ^ 1) * kIn * kSub * kBlock + tid,
                              dy_base + (buf ^ 1) * kSub * kBlock + tid, src1, src2, dys, P,
                              ta - kSub, t1);
        cp_async_commit();
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      const float2* inb = in_base + buf * kIn * kSub * kBlock + tid;
      const float2* dyb = dy_base + buf * kSub * kBlock + tid;
      const float4 s0 = sub_ckpt[r * kBlock + tid];
      float4 hs[kSub];
      float4 st = s0;
#pragma unroll
      for (int i = 0; i < kSub; ++i) {
        if (ta + i < t1) {
          float2 u1, u2;
          forcing<GENERIC>(k, inb[i * kBlock], GENERIC ? inb[(kSub + i) * kBlock] : inb[0], u1, u2);
          st = lin_step(k, st, u1, u2);
          hs[i] = st;
        }
      }
#pragma unroll
      for (int i = kSub - 1; i >= 0; --i) {
        if (ta + i < t1) {
          const float2 dy = dyb[i * kBlock];
          const float n1r = k.m11 * a1r + k.m21 * a2r;
          const float n1i = k.m11 * a1i + k.m21 * a2i;
          const float n2r = dy.x + k.m12 * a1r + k.m22 * a2r;
          const float n2i = dy.y + k.m12 * a1i + k.m22 * a2i;
          a1r = n1r;
          a1i = n1i;
          a2r = n2r;
          a2i = n2i;
          const int off = (ta + i) * P;
          if (GENERIC) {
            out1[off] = make_float2(a1r, a1i);
            out2[off] = make_float2(a2r, a2i);
          } else {
            out1[off] = make_float2(k.f1 * a1r + k.f2 * a2r, k.f1 * a1i + k.f2 * a2i);
            const float2 bu = inb[i * kBlock];
            gf1 += a1r * bu.x + a1i * bu.y;
            gf2 += a2r * bu.x + a2i * bu.y;
          }
          const float4 sp = (i > 0) ? hs[i > 0 ? i - 1 : 0] : s0;
          g11 += a1r * sp.x + a1i * sp.y;
          g12 += a1r * sp.z + a1i * sp.w;
          g21 += a2r * sp.x + a2i * sp.y;
          g22 += a2r * sp.z + a2i * sp.w;
        }
      }
    }
  }

  float* part = p.part + s * kPartials * p.P + o;
  part[0 * p.P] = g11;
  part[1 * p.P] = g12;
  part[2 * p.P] = g21;
  part[3 * p.P] = g22;
  part[4 * p.P] = gf1;
  part[5 * p.P] = gf2;
}

__host__ __device__ inline size_t bwd_smem_bytes(int chunk, bool generic) {
  return (size_t)(chunk / kSub) * kBlock * sizeof(float4) +
         (size_t)2 * ((generic ? 2 : 1) + 1) * kSub * kBlock * sizeof(float2);
}

// Stages the Bu and dY2 values of steps [tb, te) of this thread's chain into its slots of
// one stage buffer (slot i of a buffer at i * kBlock).
__device__ __forceinline__ void stage_batch(float2* in_buf, float2* dy_buf, const float2* bu,
                                            const float2* dys, int P, int tb, int te) {
#pragma unroll
  for (int i = 0; i < kLook; ++i) {
    if (tb + i < te) {
      cp_async8(in_buf + i * kBlock, bu + (tb + i) * P);
      cp_async8(dy_buf + i * kBlock, dys + (tb + i) * P);
    }
  }
}

__host__ __device__ inline size_t rev_smem_bytes() { return (size_t)2 * kStages * kLook * kBlock * sizeof(float2); }

// IMEX backward of this thread block with the state run backwards in time (see the file
// comment); returns false, having done nothing, when one of the block's oscillators does
// not allow it. Batches of kLook steps, last first; Bu and dY2 of batch b - (kStages - 1)
// are staged by cp.async while batch b runs, so every load is issued two batches (16
// steps) before its use. That lookahead, not the warp count, is what keeps HBM busy:
// measured against 2 stages at 6 blocks/SM and register prefetch variants, 3 stages at 4
// blocks/SM is fastest. chunk is a multiple of kLook, so every chunk starts a batch.
// Shared memory: in[kStages][kLook][kBlock], dy[kStages][kLook][kBlock] float2, per-thread
// slots (no block barrier after the stability vote; a stage is refilled only by the
// thread that consumed it in the previous batch).
template <bool REV>
__device__ __forceinline__ bool rev_block(const Params& p, float4* smem4) {
  float2* in_base = reinterpret_cast<float2*>(smem4);
  float2* dy_base = in_base + kStages * kLook * kBlock;
  const int tid = threadIdx.x;
  const int64_t gid = (int64_t)blockIdx.x * kBlock + tid;
  const bool active = gid < p.S * p.P;
  const int64_t s = active ? gid / p.P : 0;
  const int o = active ? (int)(gid - s * p.P) : 0;
  const Coef k = load_coef(p, o);
  // Every thread votes (NaN parameters vote unstable): one unstable chain sends the whole
  // block to the recompute path.
  const bool stable = !active || (k.m11 + k.m22 > kRevTraceMin);
  if (!__syncthreads_and(stable)) return false;
  if (!active) return true;
  const int L = (int)p.L;
  const int P = REV ? -(int)p.P : (int)p.P;  // step stride; negative when scanning backwards
  const int64_t base = s * p.L * p.P + o + (REV ? (p.L - 1) * p.P : 0);
  const float2* bu = p.Bu + base;
  const float2* dys = p.dY2 + base;
  float2* out = p.dBu + base;
  const float rdet = 1.0f / (k.m11 * k.m22 - k.m12 * k.m21);
  const float i11 = k.m22 * rdet, i12 = -k.m12 * rdet, i21 = -k.m21 * rdet, i22 = k.m11 * rdet;

  float a1r = 0.f, a1i = 0.f, a2r = 0.f, a2i = 0.f;  // adjoint a_{t+1}
  float g11 = 0.f, g12 = 0.f, g21 = 0.f, g22 = 0.f, gf1 = 0.f, gf2 = 0.f;
  const int nb = (L + kLook - 1) / kLook;
  // Batch b lives in stage (nb - 1 - b) % kStages. One commit group per batch (empty
  // groups past the first batch keep the count uniform).
  auto stage_of = [&](int b) { return (nb - 1 - b) % kStages; };
#pragma unroll
  for (int q = 0; q < kStages - 1; ++q) {
    const int b = nb - 1 - q;
    if (b >= 0) {
      const int sg = stage_of(b);
      stage_batch(in_base + sg * kLook * kBlock + tid, dy_base + sg * kLook * kBlock + tid, bu, dys, P, b * kLook,
                  min(b * kLook + kLook, L));
    }
    cp_async_commit();
  }
  float4 st = p.ckpt[ckpt_index(p, s, p.nchunks, o)];  // state after the last step
  for (int b = nb - 1; b >= 0; --b) {
    const int bn = b - (kStages - 1);
    if (bn >= 0) {  // refills the stage consumed by batch b + 1 (full batch: bn < b)
      const int sg = stage_of(bn);
      stage_batch(in_base + sg * kLook * kBlock + tid, dy_base + sg * kLook * kBlock + tid, bu, dys, P, bn * kLook,
                  bn * kLook + kLook);
    }
    cp_async_commit();
    cp_async_wait<kStages - 1>();
    const int tb = b * kLook, te = min(tb + kLook, L);
    const bool chunk_start = (tb % p.chunk) == 0;
    float4 s_begin = make_float4(0.f, 0.f, 0.f, 0.f);
    if (chunk_start) s_begin = p.ckpt[ckpt_index(p, s, tb / p.chunk, o)];  // state before step tb
    const int sg = stage_of(b);
    const float2* inb = in_base + sg * kLook * kBlock + tid;
    const float2* dyb = dy_base + sg * kLook * kBlock + tid;
#pragma unroll
    for (int i = kLook - 1; i >= 0; --i) {
      if (tb + i < te) {
        const float2 dy = dyb[i * kBlock];
        const float2 u = inb[i * kBlock];
        const float n1r = k.m11 * a1r + k.m21 * a2r;
        const float n1i = k.m11 * a1i + k.m21 * a2i;
        const float n2r = dy.x + k.m12 * a1r + k.m22 * a2r;
        const float n2i = dy.y + k.m12 * a1i + k.m22 * a2i;
        a1r = n1r;
        a1i = n1i;
        a2r = n2r;
        a2i = n2i;
        __stcs(out + (tb + i) * P, make_float2(k.f1 * a1r + k.f2 * a2r, k.f1 * a1i + k.f2 * a2i));
        gf1 += a1r * u.x + a1i * u.y;
        gf2 += a2r * u.x + a2i * u.y;
        float4 sp;
        if (i == 0 && chunk_start) {
          sp = s_begin;
        } else {  // s_{t-1} = M^-1 (s_t - F_t)
          const float v1r = st.x - k.f1 * u.x, v1i = st.y - k.f1 * u.y;
          const float v2r = st.z - k.f2 * u.x, v2i = st.w - k.f2 * u.y;
          sp = make_float4(i11 * v1r + i12 * v2r, i11 * v1i + i12 * v2i, i21 * v1r + i22 * v2r,
                           i21 * v1i + i22 * v2i);
        }
        g11 += a1r * sp.x + a1i * sp.y;
        g12 += a1r * sp.z + a1i * sp.w;
        g21 += a2r * sp.x + a2i * sp.y;
        g22 += a2r * sp.z + a2i * sp.w;
        st = sp;
      }
    }
  }
  cp_async_wait<0>();

  float* part = p.part + s * kPartials * p.P + o;
  part[0 * p.P] = g11;
  part[1 * p.P] = g12;
  part[2 * p.P] = g21;
  part[3 * p.P] = g22;
  part[4 * p.P] = gf1;
  part[5 * p.P] = gf2;
  return true;
}

// One backward kernel for every variant (see the file comment).
template <bool GENERIC, bool REV>
__global__ void __launch_bounds__(kBlock, 4) linoss_bwd_kernel(const Params p) {
  extern __shared__ float4 smem4[];
  if (!GENERIC && p.variant == SEMX_LINOSS_IMEX && rev_block<REV>(p, smem4)) return;
  bwd_block<GENERIC, REV>(p, (int)blockIdx.x, smem4);
}

// d(loss)/d(raw parameters) from the summed gradients of (M11, M12, M21, M22, f1, f2),
// following the reference's expression graph (models/linoss/linoss.py:82-116, 183-232)
// term by term, including the sub-gradient conventions of relu (zero at 0) and of clamp
// with tensor bounds.
__device__ void linoss_chain(int variant, int a_from_g, float sraw, float araw, float graw,
                             const float g[kPartials], float& d_s, float& d_a, float& d_g) {
  const float step = sigmoid_f(sraw);
  const float st2 = step * step;
  const float gM11 = g[0], gM12 = g[1], gM21 = g[2], gM22 = g[3], gf1 = g[4], gf2 = g[5];
  float gs = 0.f, gA = 0.f, gG = 0.f;
  d_g = 0.f;
  if (variant == SEMX_LINOSS_IMEX) {
    const float A = relu_f(araw);
    gs = -A * gM12 + gM21 - 2.0f * step * A * gM22 + gf1 + 2.0f * step * gf2;
    gA = -step * gM12 - st2 * gM22;
    d_a = araw > 0.0f ? gA : 0.0f;
  } else if (variant == SEMX_LINOSS_IM) {
    const float A = relu_f(araw);
    const float q = st2 * A;
    const float schur = 1.0f / (1.0f + q);
    const float m11 = 1.0f - q * schur;
    const float m21 = step * schur;
    const float dsc_ds = -schur * schur * 2.0f * step * A;
    const float dsc_dA = -schur * schur * st2;
    const float dm11_ds = -(2.0f * step * A * schur + q * dsc_ds);
    const float dm11_dA = -(st2 * schur + q * dsc_dA);
    const float dm12_ds = -(A * schur + step * A * dsc_ds);
    const float dm12_dA = -(step * schur + step * A * dsc_dA);
    const float dm21_ds = schur + step * dsc_ds;
    const float dm21_dA = step * dsc_dA;
    gs = gM11 * dm11_ds + gM12 * dm12_ds + gM21 * dm21_ds + gM22 * dsc_ds +
         gf1 * (dm11_ds * step + m11) + gf2 * (dm21_ds * step + m21);
    gA = gM11 * dm11_dA + gM12 * dm12_dA + gM21 * dm21_dA + gM22 * dsc_dA + gf1 * dm11_dA * step +
         gf2 * dm21_dA * step;
    d_a = araw > 0.0f ? gA : 0.0f;
  } else {  // DAMPED_IMEX
    // Recompute the constrained (A, G) exactly as make_coef does.
    float A, G;
    float sq = 0.f, A_low = 0.f, A_high = 0.f, sA = 0.f, G_low = 0.f, G_high = 0.f, v = 0.f;
    if (a_from_g) {
      G = relu_f(graw);
      sq = sqrtf(1.0f + step * G);
      A_low = (2.0f + step * G - 2.0f * sq) / st2;
      A_high = (2.0f + step * G + 2.0f * sq) / st2;
      A = A_low + relu_f(araw - A_low) - relu_f(araw - A_high);
    } else {
      A = relu_f(araw);
      sA = sqrtf(A);
      v = step * A - 2.0f * sA;
      G_low = relu_f(v);
      G_high = step * A + 2.0f * sA;
      G = fminf(fmaxf(graw, G_low), G_high);
    }
    const float inv = 1.0f / (1.0f + step * G);
    const float dinv_ds = -inv * inv * G;
    const float dinv_dG = -inv * inv * step;
    // M11 = inv
    gs += gM11 * dinv_ds;
    gG += gM11 * dinv_dG;
    // M12 = -step * inv * A
    gs += gM12 * (-(inv + step * dinv_ds) * A);
    gA += gM12 * (-step * inv);
    gG += gM12 * (-step * A * dinv_dG);
    // M21 = f1 = step * inv
    gs += (gM21 + gf1) * (inv + step * dinv_ds);
    gG += (gM21 + gf1) * (step * dinv_dG);
    // M22 = 1 - step^2 * inv * A
    gs += gM22 * (-(2.0f * step * inv + st2 * dinv_ds) * A);
    gA += gM22 * (-st2 * inv);
    gG += gM22 * (-st2 * A * dinv_dG);
    // f2 = step^2 * inv
    gs += gf2 * (2.0f * step * inv + st2 * dinv_ds);
    gG += gf2 * (st2 * dinv_dG);
    if (a_from_g) {
      const bool il = (araw - A_low) > 0.0f;
      const bool ih = (araw - A_high) > 0.0f;
      d_a = gA * ((il ? 1.0f : 0.0f) - (ih ? 1.0f : 0.0f));
      const float gAl = il ? 0.0f : gA;
      const float gAh = ih ? gA : 0.0f;
      const float u = step * G;
      (void)u;
      const float gu = gAl * (1.0f - 1.0f / sq) / st2 + gAh * (1.0f + 1.0f / sq) / st2;
      gs += gAl * (-2.0f * A_low / step) + gAh * (-2.0f * A_high / step) + gu * G;
      gG += gu * step;
      d_g = graw > 0.0f ? gG : 0.0f;
    } else {
      const float g_in = (graw >= G_low && graw <= G_high) ? gG : 0.0f;
      const float g_min = (graw < G_low && G_low < G_high) ? gG : 0.0f;
      const float g_max = (graw > G_high || G_high < G_low) ? gG : 0.0f;
      d_g = g_in;
      if (araw > 0.0f) {
        const float gv = v > 0.0f ? g_min : 0.0f;
        gs += gv * A + g_max * A;
        gA += gv * step + g_max * step;
        const float gsA = -2.0f * gv + 2.0f * g_max;
        gA += gsA * (0.5f / sA);
        d_a = gA;
      } else {
        gs += (v > 0.0f ? g_min : 0.0f) * A + g_max * A;
        d_a = 0.0f;
      }
    }
  }
  d_s = gs * (step * (1.0f - step));
}

// Parameter-gradient reduction over sequences, in two fixed-order stages (bitwise
// deterministic). Stage 1: CTA (x, g) of 32x8 threads sums the rows of sequence group g
// (kRowsPerGroup consecutive sequences) for oscillators 32x .. 32x+31; lane y takes rows
// y, y+8, ... and the 8 lanes are combined by a fixed tree. Stage 2 sums the groups in
// order and applies the chain rule to the raw parameters.
constexpr int kRowsPerGroup = 32;

__device__ __forceinline__ void tree8(float (&red)[kPartials][8][33], float (&g)[kPartials]) {
#pragma unroll
  for (int j = 0; j < kPartials; ++j) {
    const float a = (red[j][0][threadIdx.x] + red[j][1][threadIdx.x]) +
                    (red[j][2][threadIdx.x] + red[j][3][threadIdx.x]);
    const float b = (red[j][4][threadIdx.x] + red[j][5][threadIdx.x]) +
                    (red[j][6][threadIdx.x] + red[j][7][threadIdx.x]);
    g[j] = a + b;
  }
}

__global__ void __launch_bounds__(256) linoss_reduce_kernel(const Params p, float* group_sums) {
  __shared__ float red[kPartials][8][33];
  const int o = blockIdx.x * 32 + threadIdx.x;
  const int ty = threadIdx.y;
  const int64_t r0 = (int64_t)blockIdx.y * kRowsPerGroup;
  const int64_t r1 = min(r0 + kRowsPerGroup, p.S);
  float acc[kPartials];
#pragma unroll
  for (int j = 0; j < kPartials; ++j) acc[j] = 0.f;
  if (o < p.P) {
    for (int64_t s = r0 + ty; s < r1; s += 8) {
      const float* src = p.part + s * kPartials * p.P + o;
#pragma unroll
      for (int j = 0; j < kPartials; ++j) acc[j] += src[j * p.P];
    }
  }
#pragma unroll
  for (int j = 0; j < kPartials; ++j) red[j][ty][threadIdx.x] = acc[j];
  __syncthreads();
  if (ty != 0 || o >= p.P) return;
  float g[kPartials];
  tree8(red, g);
#pragma unroll
  for (int j = 0; j < kPartials; ++j)
    group_sums[((int64_t)blockIdx.y * kPartials + j) * p.P + o] = g[j];
}

__global__ void __launch_bounds__(256) linoss_finalize_kernel(const Params p,
                                                              const float* group_sums,
                                                              int ngroups) {
  __shared__ float red[kPartials][8][33];
  const int o = blockIdx.x * 32 + threadIdx.x;
  const int ty = threadIdx.y;
  float acc[kPartials];
#pragma unroll
  for (int j = 0; j < kPartials; ++j) acc[j] = 0.f;
  if (o < p.P) {
    for (int gi = ty; gi < ngroups; gi += 8) {
      const float* src = group_sums + (int64_t)gi * kPartials * p.P + o;
#pragma unroll
      for (int j = 0; j < kPartials; ++j) acc[j] += src[j * p.P];
    }
  }
#pragma unroll
  for (int j = 0; j < kPartials; ++j) red[j][ty][threadIdx.x] = acc[j];
  __syncthreads();
  if (ty != 0 || o >= p.P) return;
  float g[kPartials];
  tree8(red, g);
  if (p.variant == SEMX_LINOSS_GENERIC) {
    for (int j = 0; j < 4; ++j) p.dM[j * p.P + o] = g[j];
    return;
  }
  const float graw = (p.variant == SEMX_LINOSS_DAMPED_IMEX) ? p.G_diag[o] : 0.0f;
  float ds, da, dg;
  linoss_chain(p.variant, p.a_from_g, p.steps[o], p.A_diag[o], graw, g, ds, da, dg);
  p.dparams[0 * p.P + o] = ds;
  p.dparams[1 * p.P + o] = da;
  if (p.variant == SEMX_LINOSS_DAMPED_IMEX) p.dparams[2 * p.P + o] = dg;
}

int validate(const SemxLinossArgs* a, bool bwd) {
  SEMX_REQUIRE(a->S >= 0 && a->L >= 0 && a->P >= 0, SEMX_ERR_SHAPE,
               "linoss: negative size S=%lld L=%lld P=%lld", (long long)a->S, (long long)a->L,
               (long long)a->P);
  SEMX_REQUIRE(a->L * a->P < ((int64_t)1 << 31), SEMX_ERR_SHAPE,
               "linoss: L*P=%lld must be below 2^31", (long long)(a->L * a->P));
  SEMX_REQUIRE(a->variant >= SEMX_LINOSS_GENERIC && a->variant <= SEMX_LINOSS_DAMPED_IMEX,
               SEMX_ERR_UNSUPPORTED, "linoss: unknown variant %d", a->variant);
  SEMX_REQUIRE(a->chunk >= kSub && a->chunk <= kMaxChunk && a->chunk % kSub == 0,
               SEMX_ERR_UNSUPPORTED, "linoss: chunk=%d must be a multiple of %d in [%d, %d]",
               a->chunk, kSub, kSub, kMaxChunk);
  const bool generic = a->variant == SEMX_LINOSS_GENERIC;
  // Per-oscillator parameters are read whenever there are oscillators; per-step tensors
  // only when there is at least one (sequence, step, oscillator) element.
  const bool has_osc = a->P > 0 && (a->S > 0 || bwd);
  const bool has_elems = a->S * a->L * a->P > 0;
  if (has_osc) {
    if (generic) {
      SEMX_REQUIRE(a->M11 && a->M12 && a->M21 && a->M22, SEMX_ERR_NULL, "linoss: M is NULL");
    } else {
      SEMX_REQUIRE(a->steps && a->A_diag, SEMX_ERR_NULL, "linoss: steps/A_diag is NULL");
      SEMX_REQUIRE(a->variant != SEMX_LINOSS_DAMPED_IMEX || a->G_diag, SEMX_ERR_NULL,
                   "linoss: G_diag is NULL for the damped variant");
    }
  }
  if (has_elems) {
    if (generic) {
      SEMX_REQUIRE(a->F1 && a->F2, SEMX_ERR_NULL, "linoss: F1/F2 is NULL");
      SEMX_REQUIRE(semx::aligned(a->F1, 8) && semx::aligned(a->F2, 8), SEMX_ERR_ALIGN,
                   "linoss: F1/F2 must be 8-byte aligned");
    } else {
      SEMX_REQUIRE(a->Bu != nullptr, SEMX_ERR_NULL, "linoss: Bu is NULL");
      SEMX_REQUIRE(semx::aligned(a->Bu, 8), SEMX_ERR_ALIGN, "linoss: Bu must be 8-byte aligned");
    }
    if (!bwd) {
      SEMX_REQUIRE(a->Y2 != nullptr, SEMX_ERR_NULL, "linoss: Y2 is NULL");
      SEMX_REQUIRE(semx::aligned(a->Y2, 8), SEMX_ERR_ALIGN, "linoss: Y2 must be 8-byte aligned");
    } else {
      SEMX_REQUIRE(a->ckpt && a->dY2, SEMX_ERR_NULL, "linoss bwd: ckpt/dY2 is NULL");
      SEMX_REQUIRE(semx::aligned(a->dY2, 8), SEMX_ERR_ALIGN, "linoss bwd: dY2 misaligned");
      if (generic) {
        SEMX_REQUIRE(a->dF1 && a->dF2, SEMX_ERR_NULL, "linoss bwd: dF1/dF2 is NULL");
        SEMX_REQUIRE(semx::aligned(a->dF1, 8) && semx::aligned(a->dF2, 8), SEMX_ERR_ALIGN,
                     "linoss bwd: dF1/dF2 misaligned");
      } else {
        SEMX_REQUIRE(a->dBu != nullptr, SEMX_ERR_NULL, "linoss bwd: dBu is NULL");
        SEMX_REQUIRE(semx::aligned(a->dBu, 8), SEMX_ERR_ALIGN, "linoss bwd: dBu misaligned");
      }
    }
  }
  if (bwd && a->P > 0) {
    SEMX_REQUIRE(generic ? a->dM != nullptr : a->dparams != nullptr, SEMX_ERR_NULL,
                 "linoss bwd: %s is NULL", generic ? "dM" : "dparams");
    SEMX_REQUIRE(a->workspace != nullptr || a->S == 0, SEMX_ERR_WORKSPACE,
                 "linoss bwd: workspace is NULL");
  }
  if (a->ckpt) SEMX_REQUIRE(semx::aligned(a->ckpt, 16), SEMX_ERR_ALIGN,
                            "linoss: ckpt must be 16-byte aligned");
  return SEMX_OK;
}

Params to_params(const SemxLinossArgs* a) {
  Params p;
  p.variant = a->variant;
  p.a_from_g = a->a_from_g;
  p.chunk = a->chunk;
  p.rev = a->reverse != 0;
  p.nchunks = (int)semx::cdiv(a->L, a->chunk);
  p.S = a->S;
  p.L = a->L;
  p.P = a->P;
  p.M11 = a->M11;
  p.M12 = a->M12;
  p.M21 = a->M21;
  p.M22 = a->M22;
  p.F1 = reinterpret_cast<const float2*>(a->F1);
  p.F2 = reinterpret_cast<const float2*>(a->F2);
  p.steps = a->steps;
  p.A_diag = a->A_diag;
  p.G_diag = a->G_diag;
  p.Bu = reinterpret_cast<const float2*>(a->Bu);
  p.Y2 = reinterpret_cast<float2*>(a->Y2);
  p.ckpt = reinterpret_cast<float4*>(a->ckpt);
  p.dY2 = reinterpret_cast<const float2*>(a->dY2);
  p.dF1 = reinterpret_cast<float2*>(a->dF1);
  p.dF2 = reinterpret_cast<float2*>(a->dF2);
  p.dBu = reinterpret_cast<float2*>(a->dBu);
  p.dM = a->dM;
  p.dparams = a->dparams;
  p.part = reinterpret_cast<float*>(a->workspace);
  return p;
}

}  // namespace

extern "C" {

size_t semx_linoss_args_size(void) { return sizeof(SemxLinossArgs); }

size_t semx_linoss_ckpt_bytes(int64_t S, int64_t L, int64_t P, int32_t chunk) {
  if (chunk <= 0 || S < 0 || L < 0 || P < 0) return 0;
  return (size_t)S * (size_t)(semx::cdiv(L, chunk) + 1) * (size_t)P * 4 * sizeof(float);
}

size_t semx_linoss_workspace_bytes(const SemxLinossArgs* a) {
  if (a == nullptr || a->S < 0 || a->P < 0) return 0;
  const size_t groups = (size_t)semx::cdiv(a->S, kRowsPerGroup);
  return ((size_t)a->S + groups) * kPartials * (size_t)a->P * sizeof(float);
}

int semx_linoss_fwd(const SemxLinossArgs* a, semx_stream_t stream) {
  SEMX_CHECK_ARGS(a, SemxLinossArgs);
  int rc = validate(a, false);
  if (rc != SEMX_OK) return rc;
  if (a->S * a->P == 0 || a->L == 0) return SEMX_OK;
  rc = semx::bind_device({a->Y2, a->Bu, a->F1});
  if (rc != SEMX_OK) return rc;
  const Params p = to_params(a);
  const int64_t n = a->S * a->P;
  const dim3 grid((unsigned)semx::cdiv(n, kBlock));
  cudaStream_t st = semx::as_stream(stream);
  const bool generic = a->variant == SEMX_LINOSS_GENERIC;
  if (generic && p.rev)
    linoss_fwd_kernel<true, true><<<grid, kBlock, 0, st>>>(p);
  else if (generic)
    linoss_fwd_kernel<true, false><<<grid, kBlock, 0, st>>>(p);
  else if (p.rev)
    linoss_fwd_kernel<false, true><<<grid, kBlock, 0, st>>>(p);
  else
    linoss_fwd_kernel<false, false><<<grid, kBlock, 0, st>>>(p);
  return semx::check_launch("linoss_fwd_kernel");
}

int semx_linoss_bwd(const SemxLinossArgs* a, semx_stream_t stream) {
  SEMX_CHECK_ARGS(a, SemxLinossArgs);
  int rc = validate(a, true);
  if (rc != SEMX_OK) return rc;
  rc = semx::bind_device({a->dBu, a->dF1, a->dparams, a->dM});
  if (rc != SEMX_OK) return rc;
  const Params p = to_params(a);
  cudaStream_t st = semx::as_stream(stream);
  const int64_t n = a->S * a->P;
  if (n > 0 && a->L > 0) {
    const bool generic = a->variant == SEMX_LINOSS_GENERIC;
    const size_t smem = std::max(bwd_smem_bytes(a->chunk, generic),
                                 a->variant == SEMX_LINOSS_IMEX ? rev_smem_bytes() : (size_t)0);
    const dim3 grid((unsigned)semx::cdiv(n, kBlock));
    auto kernel = generic ? (p.rev ? linoss_bwd_kernel<true, true> : linoss_bwd_kernel<true, false>)
                          : (p.rev ? linoss_bwd_kernel<false, true> : linoss_bwd_kernel<false, false>);
    if (!semx::allow_smem(kernel, smem)) return SEMX_ERR_LAUNCH;
    kernel<<<grid, kBlock, smem, st>>>(p);
    rc = semx::check_launch("linoss_bwd_kernel");
    if (rc != SEMX_OK) return rc;
  } else if (n > 0) {
    // L == 0: no steps, every partial is zero.
    cudaMemsetAsync(a->workspace, 0, (size_t)n * kPartials * sizeof(float), st);
  }
  if (a->P > 0) {
    const int ngroups = (int)semx::cdiv(a->S, kRowsPerGroup);
    float* group_sums = p.part + a->S * kPartials * a->P;
    if (ngroups > 0) {
      linoss_reduce_kernel<<<dim3((unsigned)semx::cdiv(a->P, 32), (unsigned)ngroups),
                             dim3(32, 8), 0, st>>>(p, group_sums);
      rc = semx::check_launch("linoss_reduce_kernel");
      if (rc != SEMX_OK) return rc;
    }
    linoss_finalize_kernel<<<(unsigned)semx::cdiv(a->P, 32), dim3(32, 8), 0, st>>>(
        p, group_sums, ngroups);
    return semx::check_launch("linoss_finalize_kernel");
  }
  return SEMX_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------------------
// Backward without caller-provided scratch: the reductions' partial rows live in a fixed
// pool compiled into the library. In host code the pool's name denotes a host-side shadow
// variable, not device memory, so its device address is looked up once per device with
// cudaGetSymbolAddress while that device is current, and that address is what the kernels
// get.
namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[SEMX_LINOSS_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxDevices] = {};

// Device address of the pool on the current device (looked up on first use).
int noalloc_scratch(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return semx::fail(SEMX_ERR_LAUNCH, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return semx::fail(SEMX_ERR_UNSUPPORTED, "linoss noalloc: device %d outside the %d-device table", dev,
                      kMaxDevices);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess)
      return semx::fail(SEMX_ERR_LAUNCH, "cudaGetSymbolAddress(scratch pool): %s", cudaGetErrorString(e));
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return SEMX_OK;
}

}  // namespace

extern "C" int semx_linoss_bwd_noalloc(const SemxLinossArgs* a, semx_stream_t stream) {
  SEMX_CHECK_ARGS(a, SemxLinossArgs);
  // Bound S and P before the size query multiplies them, so that a huge S*P cannot wrap
  // the byte count into something that fits the pool.
  constexpr int64_t kPoolFloats = (int64_t)(SEMX_LINOSS_NOALLOC_SCRATCH_BYTES / sizeof(float));
  SEMX_REQUIRE(a->S >= 0 && a->P >= 0 && (a->P == 0 || a->S <= kPoolFloats / (kPartials * a->P)),
               SEMX_ERR_SHAPE,
               "linoss noalloc: S=%lld, P=%lld need more scratch than the built-in pool holds (%zu B; "
               "use semx_linoss_bwd with a workspace instead)",
               (long long)a->S, (long long)a->P, (size_t)SEMX_LINOSS_NOALLOC_SCRATCH_BYTES);
  const size_t need = semx_linoss_workspace_bytes(a);
  SEMX_REQUIRE(need <= SEMX_LINOSS_NOALLOC_SCRATCH_BYTES, SEMX_ERR_SHAPE,
               "linoss noalloc: S=%lld, P=%lld need %zu B of scratch; the built-in pool holds %zu B "
               "(use semx_linoss_bwd with a workspace instead)",
               (long long)a->S, (long long)a->P, need, (size_t)SEMX_LINOSS_NOALLOC_SCRATCH_BYTES);
  // The pool is looked up on the GPU that owns the outputs; semx_linoss_bwd then
  // validates the call with the pool in place of the workspace.
  int rc = semx::bind_device({a->dBu, a->dF1, a->dparams, a->dM});
  if (rc != SEMX_OK) return rc;
  SemxLinossArgs b = *a;
  rc = noalloc_scratch(&b.workspace);
  if (rc != SEMX_OK) return rc;
  return semx_linoss_bwd(&b, stream);
}

