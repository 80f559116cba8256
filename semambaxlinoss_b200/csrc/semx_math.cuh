// Transcendentals on the special-function unit for the scan kernels.
#pragma once

namespace semx {

// Per-element transcendentals on the special-function unit (PTX ex2 / sin / cos / rsqrt /
// rcp .approx: one MUFU instruction each instead of a libm call). sin and cos take their
// argument reduced to [-pi, pi] first: r = x - k * 2pi with k = rint(x / 2pi) and 2pi
// split Cody-Waite style into hi = 6.28125 (exact: k * hi has no rounding for |k| < 2^16)
// plus lo = 2pi - hi, so r carries no reduction error worth speaking of. All forms flush
// subnormal inputs and outputs (.ftz): the scans' rsqrt arguments are clamped to >= 1e-6
// and a subnormal reduced angle changes sin by less than 1.2e-38, while the non-ftz forms
// cost extra instructions per call (complex scan forward and backward 3 % slower).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rsqrt_approx(float x) {
  float y;
  asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float reduce_2pi(float x) {
  constexpr float kInv2Pi = 0.15915494f;
  constexpr float k2PiHi = 6.28125f;
  constexpr float k2PiLo = 0.0019353072f;
  // k = rint(x / 2pi) by the 1.5 * 2^23 rounding constant on the FMA pipe (exact for
  // |x / 2pi| < 2^22, far beyond the 2^16 the Cody-Waite split allows): with rintf the
  // rounding instruction apparently shared the special-function pipe with ex2 / sin / cos /
  // rsqrt (complex selective-LRU forward 404 x 321 0.827 -> 0.779 ms without it).
  const float k = fmaf(x, kInv2Pi, 12582912.f) - 12582912.f;
  return fmaf(-k, k2PiLo, fmaf(-k, k2PiHi, x));
}
__device__ __forceinline__ void sincos_reduced(float x, float* s, float* c) {
  const float r = reduce_2pi(x);
  asm("sin.approx.ftz.f32 %0, %1;" : "=f"(*s) : "f"(r));
  asm("cos.approx.ftz.f32 %0, %1;" : "=f"(*c) : "f"(r));
}
__device__ __forceinline__ float sin_reduced(float x) {
  const float r = reduce_2pi(x);
  float s;
  asm("sin.approx.ftz.f32 %0, %1;" : "=f"(s) : "f"(r));
  return s;
}

// torch.nn.functional.softplus (beta 1, threshold 20) and its derivative.
__device__ __forceinline__ float softplus(float x) { return x > 20.f ? x : log1pf(expf(x)); }
__device__ __forceinline__ float softplus_grad(float x) { return x > 20.f ? 1.f : 1.f / (1.f + expf(-x)); }

}  // namespace semx
