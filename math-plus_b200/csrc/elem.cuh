// Element access in f64 for the element-wise kernels: every stored type (f32, f16, bf16, i32,
// bool) widens to f64 exactly, so an op evaluated in f64 and rounded once on store follows the
// reference's f64 evaluation.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "../../include/mathplus_cuda.h"

namespace mpc {

__device__ __forceinline__ double ld_d(const void *p, int dt, int64_t i) {
  switch (dt) {
    case MPC_F32:
      return (double)static_cast<const float *>(p)[i];
    case MPC_BF16:
      return (double)__bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
    case MPC_F16:
      return (double)__half2float(static_cast<const __half *>(p)[i]);
    case MPC_I32:
      return (double)static_cast<const int32_t *>(p)[i];
    default:
      return static_cast<const uint8_t *>(p)[i] ? 1.0 : 0.0;
  }
}

__device__ __forceinline__ void st_d(void *p, int dt, int64_t i, double v) {
  switch (dt) {
    case MPC_F32:
      static_cast<float *>(p)[i] = (float)v;
      break;
    case MPC_BF16:
      static_cast<__nv_bfloat16 *>(p)[i] = __double2bfloat16(v);
      break;
    case MPC_F16:
      static_cast<__half *>(p)[i] = __double2half(v);
      break;
    case MPC_I32:
      static_cast<int32_t *>(p)[i] = (int32_t)(long long)v;
      break;
    default:
      static_cast<uint8_t *>(p)[i] = v != 0.0 ? 1 : 0;
  }
}

}  // namespace mpc
