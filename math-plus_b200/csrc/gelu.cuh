// Exact (erf) GELU in f32 for the device: GELU(x) = x·Φ(x), the function the reference evaluates
// in f64 (packages/special/src/index.ts:186-193, geluErf = x·normalCdf(x)).
//
// Φ(x) = ½·erfc(z) with z = -x/√2. Branch-free evaluation with t = |z|:
//   erfc(t) = exp(-t²)·erfcx(t),  erfcx(t) ≈ u·P(u),  u = 1/(1 + 0.38·t)
// — the substitution of Hastings' approximations (Abramowitz & Stegun 7.1.26) with a degree-8 P
// whose coefficients were fitted for this library by iteratively re-weighted least squares on the
// relative error of erfcx over t in [0, 12] (2e-8 in exact arithmetic, 4e-7 evaluated in f32).
// The ½ is folded into P's coefficients (an exact scaling). t² is split into hi + lo (fma) so its
// rounding stays out of the exponent. Then
//   Φ(x) = ½·erfc(t) for x <= 0,  1 - ½·erfc(t) for x > 0.
// 1/(1 + 0.38·t) and 2^y use the hardware approximations (rcp.approx, ex2.approx; both within a
// few ulp). gelu_erf_f32x2 evaluates two arguments with the paired f32 instructions of sm_100
// (fma / mul .f32x2) and gives the same bits as two calls of gelu_erf_f32.
// The tests hold it to the reference's f64 GELU on a dense grid.
#pragma once

namespace mpc {
namespace gelu_detail {

// P's coefficients, highest degree first, already multiplied by ½: the leading one, then the rest
// (Horner's scheme starts from the leading coefficient, so no multiply-add is spent on a zero).
#define MPC_GELU_P_LEAD 0.029522638767957687f
#define MPC_GELU_P_REST(X)                                                                           \
  X(-0.13134364783763885f) X(0.18237833678722382f) X(-0.081276483833789825f) X(0.11541666835546494f) \
  X(0.06914050877094269f) X(0.10200400650501251f) X(0.10695201903581619f) X(0.10720596462488174f)
constexpr float kInvSqrt2 = 0.70710678118654752f;
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ float ex2_approx(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ unsigned long long pk(float a, float b) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float2 unpk(unsigned long long v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ unsigned long long fma2(unsigned long long a, unsigned long long b, unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ unsigned long long mul2(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ unsigned long long add2(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

}  // namespace gelu_detail

__device__ __forceinline__ float gelu_erf_f32(float x) {
  using namespace gelu_detail;
  const float t = fabsf(x) * kInvSqrt2;
  const float u = rcp_approx(fmaf(0.38f, t, 1.0f));
  float p = MPC_GELU_P_LEAD;
#define MPC_HORNER(c) p = fmaf(p, u, c);
  MPC_GELU_P_REST(MPC_HORNER)
#undef MPC_HORNER
  const float hi = t * t;
  const float lo = fmaf(t, t, -hi);
  const float e = ex2_approx(hi * -kLog2e);
  const float half_erfc = fmaf(-lo, e, e) * (p * u);
  return x * (x > 0.0f ? 1.0f - half_erfc : half_erfc);
}

// GELU of (x0, x1), bit-identical to two gelu_erf_f32 calls.
__device__ __forceinline__ void gelu_erf_f32x2(float &x0, float &x1) {
  using namespace gelu_detail;
  const unsigned long long t = mul2(pk(fabsf(x0), fabsf(x1)), pk(kInvSqrt2, kInvSqrt2));
  const float2 d = unpk(fma2(pk(0.38f, 0.38f), t, pk(1.0f, 1.0f)));
  const unsigned long long u = pk(rcp_approx(d.x), rcp_approx(d.y));
  unsigned long long p = pk(MPC_GELU_P_LEAD, MPC_GELU_P_LEAD);
#define MPC_HORNER2(c) p = fma2(p, u, pk(c, c));
  MPC_GELU_P_REST(MPC_HORNER2)
#undef MPC_HORNER2
  const unsigned long long hi = mul2(t, t);
  const float2 hf = unpk(hi);
  const unsigned long long lo = fma2(t, t, pk(-hf.x, -hf.y));
  const float2 a = unpk(mul2(hi, pk(-kLog2e, -kLog2e)));
  const unsigned long long e = pk(ex2_approx(a.x), ex2_approx(a.y));
  const float2 lf = unpk(lo);
  const float2 h = unpk(mul2(fma2(pk(-lf.x, -lf.y), e, e), mul2(p, u)));
  x0 *= x0 > 0.0f ? 1.0f - h.x : h.x;
  x1 *= x1 > 0.0f ? 1.0f - h.y : h.y;
}

}  // namespace mpc
