// The row / element-wise ops the GEMM and attention path touches (HBM-bound kernels):
// softmax (kernels.ts:219-247), exact GELU (special/src/index.ts:191-193), broadcast add,
// LayerNorm (nn-kernels.ts:108-129), embedding row gather (nn-kernels.ts:277-286) and casts.
// All accumulate in f32, read their input in any of f32 / f16 / bf16 and round once on store.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cfloat>

#include "gelu.cuh"
#include "mpc_internal.h"

namespace mpc {
namespace {

__device__ __forceinline__ float load_as_f32(const void *p, int dt, int64_t i) {
  if (dt == MPC_F32) return static_cast<const float *>(p)[i];
  if (dt == MPC_BF16) return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
  return __half2float(static_cast<const __half *>(p)[i]);
}

__device__ __forceinline__ void store_from_f32(void *p, int dt, int64_t i, float v) {
  if (dt == MPC_F32)
    static_cast<float *>(p)[i] = v;
  else if (dt == MPC_BF16)
    static_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v);
  else
    static_cast<__half *>(p)[i] = __float2half_rn(v);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Softmax over the last axis: one warp per row, three passes (max, exp-sum, scale).
__global__ void softmax_rows_kernel(const void *__restrict__ x, int dt, float *__restrict__ out, int64_t rows,
                                    int64_t dim) {
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int lane = threadIdx.x & 31;
  for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    const int64_t base = r * dim;
    float mx = -FLT_MAX;
    for (int64_t j = lane; j < dim; j += 32) mx = fmaxf(mx, load_as_f32(x, dt, base + j));
    mx = warp_max(mx);
    float s = 0.0f;
    for (int64_t j = lane; j < dim; j += 32) {
      const float e = expf(load_as_f32(x, dt, base + j) - mx);
      out[base + j] = e;
      s += e;
    }
    s = warp_sum(s);
    const float inv = 1.0f / s;
    __syncwarp();
    for (int64_t j = lane; j < dim; j += 32) out[base + j] *= inv;
  }
}

// Softmax over a middle axis of [outer, dim, inner]: one thread per (outer, inner) lane, reads
// coalesced across inner.
__global__ void softmax_lanes_kernel(const void *__restrict__ x, int dt, float *__restrict__ out, int64_t outer,
                                    int64_t dim, int64_t inner) {
  const int64_t lanes = outer * inner;
  for (int64_t l = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; l < lanes; l += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = l / inner, t = l - o * inner;
    const int64_t base = o * dim * inner + t;
    float mx = -FLT_MAX;
    for (int64_t j = 0; j < dim; ++j) mx = fmaxf(mx, load_as_f32(x, dt, base + j * inner));
    float s = 0.0f;
    for (int64_t j = 0; j < dim; ++j) {
      const float e = expf(load_as_f32(x, dt, base + j * inner) - mx);
      out[base + j * inner] = e;
      s += e;
    }
    const float inv = 1.0f / s;
    for (int64_t j = 0; j < dim; ++j) out[base + j * inner] *= inv;
  }
}

__global__ void gelu_kernel(const void *__restrict__ x, int dti, void *__restrict__ out, int dto, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    store_from_f32(out, dto, i, gelu_erf_f32(load_as_f32(x, dti, i)));
}

__global__ void add_kernel(const void *__restrict__ x, const void *__restrict__ y, void *__restrict__ out, int dt,
                           int64_t n, int64_t ny) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    store_from_f32(out, dt, i, load_as_f32(x, dt, i) + load_as_f32(y, dt, i % ny));
}

// ---- 16-byte vector forms for contiguous, aligned operands -----------------------------------
// A uint4 holds 8 f16 / bf16 or 4 f32 values; conversion to f32 and back (RNE) per element.
template <typename T>
struct Vec;
template <>
struct Vec<float> {
  static constexpr int N = 4;
  __device__ static void load(const uint4 &u, float *f) {
    f[0] = __uint_as_float(u.x), f[1] = __uint_as_float(u.y), f[2] = __uint_as_float(u.z), f[3] = __uint_as_float(u.w);
  }
  __device__ static uint4 store(const float *f) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
  }
};
template <>
struct Vec<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ static void load(const uint4 &u, float *f) {
    const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 t = __bfloat1622float2(h[i]);
      f[2 * i] = t.x, f[2 * i + 1] = t.y;
    }
  }
  __device__ static uint4 store(const float *f) {
    uint4 u;
    __nv_bfloat162 *h = reinterpret_cast<__nv_bfloat162 *>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    return u;
  }
};
template <>
struct Vec<__half> {
  static constexpr int N = 8;
  __device__ static void load(const uint4 &u, float *f) {
    const __half2 *h = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 t = __half22float2(h[i]);
      f[2 * i] = t.x, f[2 * i + 1] = t.y;
    }
  }
  __device__ static uint4 store(const float *f) {
    uint4 u;
    __half2 *h = reinterpret_cast<__half2 *>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    return u;
  }
};

// out = x + y (y a repeated block of nyv vectors), 16-byte vectors.
template <typename T>
__global__ void add_vec_kernel(const uint4 *__restrict__ x, const uint4 *__restrict__ y, uint4 *__restrict__ out,
                               int64_t nv, int64_t nyv) {
  constexpr int N = Vec<T>::N;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    float a[N], b[N];
    Vec<T>::load(x[i], a);
    Vec<T>::load(y[nyv == nv ? i : i % nyv], b);
#pragma unroll
    for (int j = 0; j < N; ++j) a[j] += b[j];
    out[i] = Vec<T>::store(a);
  }
}

// LayerNorm, one warp per row held in registers (one read, one write): rows of d elements, d a
// multiple of the vector width and at most 32 * MAXV vectors. Two-pass mean / population
// variance in f32 from the registers.
template <typename T, int MAXV>
__global__ void layer_norm_warp_kernel(const uint4 *__restrict__ x, const float *__restrict__ w,
                                       const float *__restrict__ b, float eps, uint4 *__restrict__ out, int64_t rows,
                                       int d) {
  constexpr int N = Vec<T>::N;
  const int dv = d / N;
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
  // Short rows (at most 4 vectors per lane): the warp's next row is loaded while the current one
  // is normalised. Longer rows already keep enough bytes in flight per warp (and the registers a
  // second row would take cost occupancy).
  constexpr bool kAhead = MAXV <= 4;
  uint4 nxt[MAXV];
  if (kAhead && r < rows) {
#pragma unroll
    for (int k = 0; k < MAXV; ++k)
      if (lane + 32 * k < dv) nxt[k] = x[r * dv + lane + 32 * k];
  }
  for (; r < rows; r += warps) {
    float v[MAXV][N];
#pragma unroll
    for (int k = 0; k < MAXV; ++k)
      if (lane + 32 * k < dv) Vec<T>::load(kAhead ? nxt[k] : x[r * dv + lane + 32 * k], v[k]);
    if (kAhead && r + warps < rows) {
#pragma unroll
      for (int k = 0; k < MAXV; ++k)
        if (lane + 32 * k < dv) nxt[k] = x[(r + warps) * dv + lane + 32 * k];
    }
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < MAXV; ++k) {
      if (lane + 32 * k < dv) {
#pragma unroll
        for (int e = 0; e < N; ++e) s += v[k][e];
      }
    }
    const float mean = warp_sum(s) / (float)d;
    float q = 0.0f;
#pragma unroll
    for (int k = 0; k < MAXV; ++k) {
      if (lane + 32 * k < dv) {
#pragma unroll
        for (int e = 0; e < N; ++e) {
          const float c = v[k][e] - mean;
          q += c * c;
        }
      }
    }
    const float inv = 1.0f / sqrtf(warp_sum(q) / (float)d + eps);
    uint4 *orow = out + r * dv;
#pragma unroll
    for (int k = 0; k < MAXV; ++k) {
      const int j = lane + 32 * k;
      if (j < dv) {
        float y[N], wv[N], bv[N];
#pragma unroll
        for (int e = 0; e < N; e += 4) {  // weight / bias rows are f32, 16-byte aligned per vector
          const float4 a = w ? __ldg(reinterpret_cast<const float4 *>(w + j * N + e)) : make_float4(1, 1, 1, 1);
          const float4 c = b ? __ldg(reinterpret_cast<const float4 *>(b + j * N + e)) : make_float4(0, 0, 0, 0);
          wv[e] = a.x, wv[e + 1] = a.y, wv[e + 2] = a.z, wv[e + 3] = a.w;
          bv[e] = c.x, bv[e + 1] = c.y, bv[e + 2] = c.z, bv[e + 3] = c.w;
        }
#pragma unroll
        for (int e = 0; e < N; ++e) y[e] = (v[k][e] - mean) * inv * wv[e] + bv[e];
        orow[j] = Vec<T>::store(y);
      }
    }
  }
}

// Sum over a 256-thread block (8 warps); every thread gets the total.
__device__ __forceinline__ float block_sum256(float v, float *red) {
  v = warp_sum(v);
  const int wi = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[wi] = v;
  __syncthreads();
  float t = l < 8 ? red[l] : 0.0f;
  t = warp_sum(t);
  __syncthreads();  // red is written again by the next call
  return t;
}

// LayerNorm of rows too long for one warp's registers (up to 256 x PER 16-byte vectors): one
// 256-thread block per row holds the row in registers, so x is read once; block-wide sums.
template <typename T, int PER>
__global__ void __launch_bounds__(256) layer_norm_block_kernel(const uint4 *__restrict__ x, const float *__restrict__ w,
                                                               const float *__restrict__ b, float eps,
                                                               uint4 *__restrict__ out, int64_t rows, int d) {
  __shared__ float red[8];
  constexpr int N = Vec<T>::N;
  const int dv = d / N;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const uint4 *xr = x + r * dv;
    float v[PER][N];
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int j = threadIdx.x + 256 * k;
      if (j < dv) {
        Vec<T>::load(xr[j], v[k]);
#pragma unroll
        for (int e = 0; e < N; ++e) s += v[k][e];
      }
    }
    const float mean = block_sum256(s, red) / (float)d;
    float q = 0.0f;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      if (threadIdx.x + 256 * k < dv) {
#pragma unroll
        for (int e = 0; e < N; ++e) {
          const float c = v[k][e] - mean;
          q += c * c;
        }
      }
    }
    const float inv = 1.0f / sqrtf(block_sum256(q, red) / (float)d + eps);
    uint4 *orow = out + r * dv;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int j = threadIdx.x + 256 * k;
      if (j < dv) {
        float y[N], wv[N], bv[N];
#pragma unroll
        for (int e = 0; e < N; e += 4) {
          const float4 a = w ? __ldg(reinterpret_cast<const float4 *>(w + j * N + e)) : make_float4(1, 1, 1, 1);
          const float4 c = b ? __ldg(reinterpret_cast<const float4 *>(b + j * N + e)) : make_float4(0, 0, 0, 0);
          wv[e] = a.x, wv[e + 1] = a.y, wv[e + 2] = a.z, wv[e + 3] = a.w;
          bv[e] = c.x, bv[e + 1] = c.y, bv[e + 2] = c.z, bv[e + 3] = c.w;
        }
#pragma unroll
        for (int e = 0; e < N; ++e) y[e] = (v[k][e] - mean) * inv * wv[e] + bv[e];
        orow[j] = Vec<T>::store(y);
      }
    }
  }
}

// LayerNorm: one block per row, two-pass mean / population variance in f32.
__global__ void layer_norm_kernel(const void *__restrict__ x, int dti, const float *__restrict__ w,
                                  const float *__restrict__ b, float eps, void *__restrict__ out, int dto,
                                  int64_t rows, int64_t d) {
  __shared__ float red[32];
  __shared__ float stat;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const int64_t base = r * d;
    float s = 0.0f;
    for (int64_t j = threadIdx.x; j < d; j += blockDim.x) s += load_as_f32(x, dti, base + j);
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
      float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
      v = warp_sum(v);
      if (threadIdx.x == 0) stat = v / (float)d;
    }
    __syncthreads();
    const float mean = stat;
    __syncthreads();
    float q = 0.0f;
    for (int64_t j = threadIdx.x; j < d; j += blockDim.x) {
      const float c = load_as_f32(x, dti, base + j) - mean;
      q += c * c;
    }
    q = warp_sum(q);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = q;
    __syncthreads();
    if (threadIdx.x < 32) {
      float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
      v = warp_sum(v);
      if (threadIdx.x == 0) stat = rsqrtf(v / (float)d + eps);
    }
    __syncthreads();
    const float inv = stat;
    for (int64_t j = threadIdx.x; j < d; j += blockDim.x) {
      float y = (load_as_f32(x, dti, base + j) - mean) * inv;
      if (w) y *= w[j];
      if (b) y += b[j];
      store_from_f32(out, dto, base + j, y);
    }
    __syncthreads();
  }
}

// Row gather: out[i] = table[ids[i]]; an id outside [0, rows) leaves a zero row and records the
// smallest offending position in *bad.
__global__ void embedding_kernel(const void *__restrict__ table, int dt, const int32_t *__restrict__ ids,
                                 void *__restrict__ out, int64_t n_ids, int64_t rows, int64_t d,
                                 unsigned long long *bad) {
  const int64_t total = n_ids * d;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t pos = i / d, c = i - pos * d;
    const int32_t id = ids[pos];
    if (id < 0 || id >= rows) {
      if (c == 0) atomicMin(bad, (unsigned long long)pos);
      store_from_f32(out, dt, i, 0.0f);
    } else {
      store_from_f32(out, dt, i, load_as_f32(table, dt, (int64_t)id * d + c));
    }
  }
}

// The same gather when rows are whole 16-byte vectors: one vector per thread (a GPT-2 token
// embedding, [32768] ids x 768 bf16, moves 50 MB at the rate of a copy).
__global__ void embedding_vec_kernel(const uint4 *__restrict__ table, const int32_t *__restrict__ ids,
                                     uint4 *__restrict__ out, int64_t n_ids, int64_t rows, int64_t dv,
                                     unsigned long long *bad) {
  const int64_t total = n_ids * dv;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t pos = i / dv, c = i - pos * dv;
    const int32_t id = ids[pos];
    if (id < 0 || id >= rows) {
      if (c == 0) atomicMin(bad, (unsigned long long)pos);
      out[i] = make_uint4(0, 0, 0, 0);
    } else {
      out[i] = table[(int64_t)id * dv + c];
    }
  }
}

__global__ void cast_kernel(const void *__restrict__ x, int dti, void *__restrict__ out, int dto, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    store_from_f32(out, dto, i, load_as_f32(x, dti, i));
}

// out = x permuted: out[i_0..i_{r-1}] = x[... i_k at axis perm[k] ...]. Each thread gathers one
// element (or one 16-byte unit when the innermost axis is kept); writes are coalesced.
struct PermParams {
  int rank;
  long long out_shape[6];
  long long in_stride[6];  // element stride in x of output axis k (= x's stride of axis perm[k])
  long long total;
};
// Index type I: 32-bit when every offset fits (cheaper divisions), else 64-bit.
template <typename T, typename I>
__global__ void permute_kernel(const T *__restrict__ x, T *__restrict__ out, const PermParams p) {
  I shape[6], stride[6];
#pragma unroll
  for (int k = 0; k < 6; ++k) shape[k] = (I)p.out_shape[k], stride[k] = (I)p.in_stride[k];
  const I total = (I)p.total;
  for (I i = blockIdx.x * (I)blockDim.x + threadIdx.x; i < total; i += (I)gridDim.x * blockDim.x) {
    I rem = i, off = 0;
#pragma unroll
    for (int k = 5; k >= 0; --k) {
      if (k < p.rank) {
        const I q = rem / shape[k];
        off += (rem - q * shape[k]) * stride[k];
        rem = q;
      }
    }
    out[i] = x[off];
  }
}

bool float_dtype(int dt) { return dt == MPC_F32 || dt == MPC_F16 || dt == MPC_BF16; }

unsigned grid_for(mpc_device *dev, int64_t n, int threads) {
  const int64_t cap = (int64_t)dev->prop.multiProcessorCount * 8;
  int64_t g = (n + threads - 1) / threads;
  if (g > cap) g = cap;
  return (unsigned)(g < 1 ? 1 : g);
}

}  // namespace
}  // namespace mpc

using namespace mpc;

extern "C" {

int mpc_softmax(mpc_device *dev, const void *x, int32_t dtype, float *out, int64_t outer, int64_t dim, int64_t inner,
                mpc_stream s) {
  int rc = enter(dev);
  if (rc) return rc;
  if (!float_dtype(dtype)) return fail(MPC_ERR_INVALID, "mpc_softmax: dtype %d is not a float type", dtype);
  if (outer < 0 || dim < 0 || inner < 0) return fail(MPC_ERR_INVALID, "mpc_softmax: negative extent");
  if (outer == 0 || dim == 0 || inner == 0) return MPC_OK;
  if (!x || !out) return fail(MPC_ERR_INVALID, "mpc_softmax: null pointer");
  cudaStream_t st = stream_of(dev, s);
  if (inner == 1)
    softmax_rows_kernel<<<grid_for(dev, outer * 32, 256), 256, 0, st>>>(x, dtype, out, outer, dim);
  else
    softmax_lanes_kernel<<<grid_for(dev, outer * inner, 256), 256, 0, st>>>(x, dtype, out, outer, dim, inner);
  dev->launches++;
  return check_launch(dev, "softmax kernel");
}

int mpc_gelu(mpc_device *dev, const void *x, int32_t dti, void *out, int32_t dto, int64_t n, mpc_stream s) {
  int rc = enter(dev);
  if (rc) return rc;
  if (!float_dtype(dti) || !float_dtype(dto)) return fail(MPC_ERR_INVALID, "mpc_gelu: float dtypes only");
  if (n <= 0) return n < 0 ? fail(MPC_ERR_INVALID, "mpc_gelu: negative size") : MPC_OK;
  if (!x || !out) return fail(MPC_ERR_INVALID, "mpc_gelu: null pointer");
  gelu_kernel<<<grid_for(dev, n, 256), 256, 0, stream_of(dev, s)>>>(x, dti, out, dto, n);
  dev->launches++;
  return check_launch(dev, "gelu_kernel");
}

int mpc_add(mpc_device *dev, const void *x, const void *y, void *out, int32_t dt, int64_t n_x, int64_t n_y,
            mpc_stream s) {
  int rc = enter(dev);
  if (rc) return rc;
  if (!float_dtype(dt)) return fail(MPC_ERR_INVALID, "mpc_add: float dtypes only");
  if (n_x < 0 || n_y <= 0 || n_x % n_y)
    return fail(MPC_ERR_INVALID, "mpc_add: %lld elements do not repeat a block of %lld", (long long)n_x, (long long)n_y);
  if (n_x == 0) return MPC_OK;
  if (!x || !y || !out) return fail(MPC_ERR_INVALID, "mpc_add: null pointer");
  const int vw = dt == MPC_F32 ? 4 : 8;
  const bool aligned = !(((uintptr_t)x | (uintptr_t)y | (uintptr_t)out) & 15) && n_x % vw == 0 && n_y % vw == 0;
  cudaStream_t st = stream_of(dev, s);
  if (aligned) {
    const int64_t nv = n_x / vw, nyv = n_y / vw;
    const unsigned g = grid_for(dev, nv, 256);
    const uint4 *xv = static_cast<const uint4 *>(x), *yv = static_cast<const uint4 *>(y);
    uint4 *ov = static_cast<uint4 *>(out);
    if (dt == MPC_F32)
      add_vec_kernel<float><<<g, 256, 0, st>>>(xv, yv, ov, nv, nyv);
    else if (dt == MPC_BF16)
      add_vec_kernel<__nv_bfloat16><<<g, 256, 0, st>>>(xv, yv, ov, nv, nyv);
    else
      add_vec_kernel<__half><<<g, 256, 0, st>>>(xv, yv, ov, nv, nyv);
  } else {
    add_kernel<<<grid_for(dev, n_x, 256), 256, 0, st>>>(x, y, out, dt, n_x, n_y);
  }
  dev->launches++;
  return check_launch(dev, "add_kernel");
}

int mpc_layer_norm(mpc_device *dev, const void *x, int32_t dti, const float *weight, const float *bias, float eps,
                   void *out, int32_t dto, int64_t rows, int64_t d, mpc_stream s) {
  int rc = enter(dev);
  if (rc) return rc;
  if (!float_dtype(dti) || !float_dtype(dto)) return fail(MPC_ERR_INVALID, "mpc_layer_norm: float dtypes only");
  if (rows < 0 || d < 0) return fail(MPC_ERR_INVALID, "mpc_layer_norm: negative extent");
  if (rows == 0 || d == 0) return MPC_OK;
  if (!x || !out) return fail(MPC_ERR_INVALID, "mpc_layer_norm: null pointer");
  cudaStream_t st = stream_of(dev, s);
  const int vw = dti == MPC_F32 ? 4 : 8;
  const int64_t per_lane = (d / vw + 31) / 32;  // 16-byte vectors each lane holds in registers
  if (dti == dto && d % vw == 0 && per_lane <= 8 && !(((uintptr_t)x | (uintptr_t)out) & 15) &&
      !(((uintptr_t)weight | (uintptr_t)bias) & 15)) {
    const int64_t blocks_needed = (rows + 7) / 8;  // 8 warps (rows) per 256-thread block
    const uint4 *xv = static_cast<const uint4 *>(x);
    uint4 *ov = static_cast<uint4 *>(out);
    const int dd = (int)d;
    // One resident wave of blocks (the occupancy of the instantiation); each warp then walks rows,
    // loading its next row while it normalises the current one. The register footprint follows
    // the row length (fewer registers, more rows in flight).
    auto grid_of_ln = [&](const void *kern, bool ahead) -> unsigned {
      int nb = 16;  // without the next-row load: up to 16 blocks per SM queued
      if (ahead && (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, 256, 0) != cudaSuccess || nb < 1)) nb = 1;
      const int64_t cap = (int64_t)dev->prop.multiProcessorCount * nb;
      return (unsigned)(blocks_needed < cap ? blocks_needed : cap);
    };
#define MPC_LN_CASE(T, K)                                                                               \
  {                                                                                                     \
    const unsigned g = grid_of_ln(reinterpret_cast<const void *>(layer_norm_warp_kernel<T, K>), K <= 4); \
    layer_norm_warp_kernel<T, K><<<g, 256, 0, st>>>(xv, weight, bias, eps, ov, rows, dd);               \
  }
#define MPC_LN(T)                   \
  switch (per_lane) {               \
    case 1: MPC_LN_CASE(T, 1) break; \
    case 2: MPC_LN_CASE(T, 2) break; \
    case 3: MPC_LN_CASE(T, 3) break; \
    case 4: MPC_LN_CASE(T, 4) break; \
    default: MPC_LN_CASE(T, 8) break; \
  }
    if (dti == MPC_F32) {
      MPC_LN(float)
    } else if (dti == MPC_BF16) {
      MPC_LN(__nv_bfloat16)
    } else {
      MPC_LN(__half)
    }
#undef MPC_LN
#undef MPC_LN_CASE
    dev->launches++;
    return check_launch(dev, "layer_norm_warp_kernel");
  }
  const int64_t per_thread = (d / vw + 255) / 256;  // 16-byte vectors each thread of a 256-thread block holds
  if (dti == dto && d % vw == 0 && per_thread <= 8 && d <= INT32_MAX && !(((uintptr_t)x | (uintptr_t)out) & 15) &&
      !(((uintptr_t)weight | (uintptr_t)bias) & 15)) {
    const uint4 *xv = static_cast<const uint4 *>(x);
    uint4 *ov = static_cast<uint4 *>(out);
    const int dd = (int)d;
    auto grid_of_lnb = [&](const void *kern) -> unsigned {
      int nb = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, 256, 0) != cudaSuccess || nb < 1) nb = 1;
      const int64_t cap = (int64_t)dev->prop.multiProcessorCount * nb;
      return (unsigned)(rows < cap ? rows : cap);
    };
#define MPC_LNB_CASE(T, K)                                                                         \
  {                                                                                                \
    const unsigned g = grid_of_lnb(reinterpret_cast<const void *>(layer_norm_block_kernel<T, K>)); \
    layer_norm_block_kernel<T, K><<<g, 256, 0, st>>>(xv, weight, bias, eps, ov, rows, dd);         \
  }
#define MPC_LNB(T)                                                \
  if (per_thread <= 1) MPC_LNB_CASE(T, 1) else if (per_thread <= 2) MPC_LNB_CASE(T, 2) \
  else if (per_thread <= 4) MPC_LNB_CASE(T, 4) else MPC_LNB_CASE(T, 8)
    if (dti == MPC_F32) {
      MPC_LNB(float)
    } else if (dti == MPC_BF16) {
      MPC_LNB(__nv_bfloat16)
    } else {
      MPC_LNB(__half)
    }
#undef MPC_LNB
#undef MPC_LNB_CASE
    dev->launches++;
    return check_launch(dev, "layer_norm_block_kernel");
  }
  const unsigned grid = (unsigned)(rows < (int64_t)dev->prop.multiProcessorCount * 16 ? rows
                                                                                      : dev->prop.multiProcessorCount * 16);
  layer_norm_kernel<<<grid, 256, 0, st>>>(x, dti, weight, bias, eps, out, dto, rows, d);
  dev->launches++;
  return check_launch(dev, "layer_norm_kernel");
}

int mpc_embedding(mpc_device *dev, const void *table, int32_t dt, const int32_t *ids, void *out, int64_t n_ids,
                  int64_t rows, int64_t d, int64_t *bad_index, mpc_stream s) {
  int rc = enter(dev);
  if (rc) return rc;
  if (bad_index) *bad_index = -1;
  if (!float_dtype(dt)) return fail(MPC_ERR_INVALID, "mpc_embedding: float tables only");
  if (n_ids < 0 || rows < 0 || d < 0) return fail(MPC_ERR_INVALID, "mpc_embedding: negative extent");
  if (n_ids == 0 || d == 0) return MPC_OK;
  if (!table || !ids || !out) return fail(MPC_ERR_INVALID, "mpc_embedding: null pointer");
  cudaStream_t st = stream_of(dev, s);
  Scratch flag;
  if ((rc = flag.get(dev, st, sizeof(unsigned long long)))) return rc;
  MPC_CUDA(dev, cudaMemsetAsync(flag.ptr, 0xff, sizeof(unsigned long long), st));
  const int64_t row_bytes = d * (int64_t)dtype_size(dt);
  if (row_bytes % 16 == 0 && !(((uintptr_t)table | (uintptr_t)out) & 15)) {
    const int64_t dv = row_bytes / 16;
    embedding_vec_kernel<<<grid_for(dev, n_ids * dv, 256), 256, 0, st>>>(
        static_cast<const uint4 *>(table), ids, static_cast<uint4 *>(out), n_ids, rows, dv,
        static_cast<unsigned long long *>(flag.ptr));
    dev->launches++;
    if ((rc = check_launch(dev, "embedding_vec_kernel"))) return rc;
  } else {
    embedding_kernel<<<grid_for(dev, n_ids * d, 256), 256, 0, st>>>(table, dt, ids, out, n_ids, rows, d,
                                                                    static_cast<unsigned long long *>(flag.ptr));
    dev->launches++;
    if ((rc = check_launch(dev, "embedding_kernel"))) return rc;
  }
  unsigned long long bad = 0;
  MPC_CUDA(dev, cudaMemcpyAsync(&bad, flag.ptr, sizeof(bad), cudaMemcpyDeviceToHost, st));
  MPC_CUDA(dev, cudaStreamSynchronize(st));
  if (bad != ~0ull) {
    if (bad_index) *bad_index = (int64_t)bad;
    return fail(MPC_ERR_INVALID, "mpc_embedding: id at position %llu is out of range [0, %lld)", bad, (long long)rows);
  }
  return MPC_OK;
}

int mpc_cast(mpc_device *dev, const void *x, int32_t dti, void *out, int32_t dto, int64_t n, mpc_stream s) {
  int rc = enter(dev);
  if (rc) return rc;
  if (!float_dtype(dti) || !float_dtype(dto)) return fail(MPC_ERR_UNSUPPORTED, "mpc_cast: float <-> float only");
  if (n <= 0) return n < 0 ? fail(MPC_ERR_INVALID, "mpc_cast: negative size") : MPC_OK;
  if (!x || !out) return fail(MPC_ERR_INVALID, "mpc_cast: null pointer");
  cast_kernel<<<grid_for(dev, n, 256), 256, 0, stream_of(dev, s)>>>(x, dti, out, dto, n);
  dev->launches++;
  return check_launch(dev, "cast_kernel");
}

int mpc_transpose(mpc_device *dev, const void *x, void *out, int32_t elem_bytes, int32_t rank, const int64_t *shape,
                  const int32_t *perm, mpc_stream s) {
  int rc = enter(dev);
  if (rc) return rc;
  if (rank < 1 || rank > 6 || !shape || !perm) return fail(MPC_ERR_INVALID, "mpc_transpose: rank %d (1..6)", rank);
  if (elem_bytes != 1 && elem_bytes != 2 && elem_bytes != 4 && elem_bytes != 8)
    return fail(MPC_ERR_INVALID, "mpc_transpose: element size %d", elem_bytes);
  long long in_shape[6], in_stride[6], total = 1;
  bool seen[6] = {false, false, false, false, false, false};
  for (int k = 0; k < rank; ++k) {
    if (shape[k] < 0) return fail(MPC_ERR_INVALID, "mpc_transpose: negative extent");
    if (perm[k] < 0 || perm[k] >= rank || seen[perm[k]])
      return fail(MPC_ERR_INVALID, "mpc_transpose: [%d...] is not a permutation", perm[0]);
    seen[perm[k]] = true;
    in_shape[k] = shape[k];
    total *= shape[k];
  }
  if (total == 0) return MPC_OK;
  if (!x || !out) return fail(MPC_ERR_INVALID, "mpc_transpose: null pointer");
  long long acc = 1;
  for (int k = rank - 1; k >= 0; --k) {
    in_stride[k] = acc;
    acc *= in_shape[k];
  }
  PermParams p{};
  p.rank = rank;
  p.total = total;
  for (int k = 0; k < rank; ++k) {
    p.out_shape[k] = in_shape[perm[k]];
    p.in_stride[k] = in_stride[perm[k]];
  }
  // Innermost axis kept in place with 16-byte rows: move 16-byte units instead of elements.
  int eb = elem_bytes;
  if (perm[rank - 1] == rank - 1 && (in_shape[rank - 1] * elem_bytes) % 16 == 0 && !((uintptr_t)x & 15) &&
      !((uintptr_t)out & 15)) {
    const long long f = 16 / elem_bytes;
    p.out_shape[rank - 1] /= f;
    for (int k = 0; k < rank - 1; ++k) p.in_stride[k] /= f;
    p.total /= f;
    eb = 16;
  }
  cudaStream_t st = stream_of(dev, s);
  const unsigned grid = grid_for(dev, p.total, 256);
  // 32-bit indexing when the element count (and so every offset) stays below 2^31 with the grid
  // stride added.
  const bool small = p.total + (long long)grid * 256 < (1ll << 31);
  switch (eb) {
#define MPC_PERMUTE(T)                                                                  \
  if (small)                                                                            \
    permute_kernel<T, uint32_t><<<grid, 256, 0, st>>>((const T *)x, (T *)out, p);       \
  else                                                                                  \
    permute_kernel<T, long long><<<grid, 256, 0, st>>>((const T *)x, (T *)out, p);
    case 1: MPC_PERMUTE(uint8_t) break;
    case 2: MPC_PERMUTE(uint16_t) break;
    case 4: MPC_PERMUTE(uint32_t) break;
    case 8: MPC_PERMUTE(uint2) break;
    default: MPC_PERMUTE(uint4) break;
#undef MPC_PERMUTE
  }
  dev->launches++;
  return check_launch(dev, "permute_kernel");
}

}  // extern "C"
