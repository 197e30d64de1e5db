// Exact (erf) GELU in f32 for the device: GELU(x) = x·Φ(x), the function the reference evaluates
// in f64 (packages/special/src/index.ts:186-193, geluErf = x·normalCdf(x)).
//
// Φ(x) = ½·erfc(z) with z = -x/√2. Branch-free evaluation with t = |z|:
//   erfc(t) = exp(-t²)·erfcx(t),  erfcx(t) ≈ u·P(u),  u = 1/(1 + 0.38·t)
// — the substitution of Hastings' approximations (Abramowitz & Stegun 7.1.26) with a degree-8 P
// whose coefficients were fitted for this library by iteratively re-weighted least squares on the
// relative error of erfcx over t in [0, 12] (2e-8 in exact arithmetic, 4e-7 evaluated in f32).
// t² is split into hi + lo (fma) so its rounding stays out of the exponent. Then
//   Φ(x) = ½·erfc(t) for x <= 0,  1 - ½·erfc(t) for x > 0.
// The tests hold it to the reference's f64 GELU on a dense grid.
#pragma once

namespace mpc {

__device__ __forceinline__ float gelu_erf_f32(float x) {
  const float t = fabsf(x) * 0.70710678118654752f;
  const float u = __frcp_rn(fmaf(0.38f, t, 1.0f));
  float p = 0.059045277535915375f;
  p = fmaf(p, u, -0.2626872956752777f);
  p = fmaf(p, u, 0.36475667357444763f);
  p = fmaf(p, u, -0.16255296766757965f);
  p = fmaf(p, u, 0.23083333671092987f);
  p = fmaf(p, u, 0.13828101754188538f);
  p = fmaf(p, u, 0.20400801301002502f);
  p = fmaf(p, u, 0.21390403807163239f);
  p = fmaf(p, u, 0.2144119292497635f);
  const float hi = t * t;
  const float lo = fmaf(t, t, -hi);
  const float half_erfc = 0.5f * (__expf(-hi) * (1.0f - lo)) * (p * u);
  return x * (x > 0.0f ? 1.0f - half_erfc : half_erfc);
}

}  // namespace mpc
