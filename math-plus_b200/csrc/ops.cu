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
template <typename T>
__global__ void permute_kernel(const T *__restrict__ x, T *__restrict__ out, const PermParams p) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < p.total;
       i += (long long)gridDim.x * blockDim.x) {
    long long rem = i, off = 0;
#pragma unroll
    for (int k = 5; k >= 0; --k) {
      if (k < p.rank) {
        const long long c = rem % p.out_shape[k];
        rem /= p.out_shape[k];
        off += c * p.in_stride[k];
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
  add_kernel<<<grid_for(dev, n_x, 256), 256, 0, stream_of(dev, s)>>>(x, y, out, dt, n_x, n_y);
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
  const unsigned grid = (unsigned)(rows < (int64_t)dev->prop.multiProcessorCount * 16 ? rows
                                                                                      : dev->prop.multiProcessorCount * 16);
  layer_norm_kernel<<<grid, 256, 0, stream_of(dev, s)>>>(x, dti, weight, bias, eps, out, dto, rows, d);
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
  embedding_kernel<<<grid_for(dev, n_ids * d, 256), 256, 0, st>>>(table, dt, ids, out, n_ids, rows, d,
                                                                  static_cast<unsigned long long *>(flag.ptr));
  dev->launches++;
  if ((rc = check_launch(dev, "embedding_kernel"))) return rc;
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
  switch (eb) {
    case 1: permute_kernel<uint8_t><<<grid, 256, 0, st>>>((const uint8_t *)x, (uint8_t *)out, p); break;
    case 2: permute_kernel<uint16_t><<<grid, 256, 0, st>>>((const uint16_t *)x, (uint16_t *)out, p); break;
    case 4: permute_kernel<uint32_t><<<grid, 256, 0, st>>>((const uint32_t *)x, (uint32_t *)out, p); break;
    case 8: permute_kernel<uint2><<<grid, 256, 0, st>>>((const uint2 *)x, (uint2 *)out, p); break;
    default: permute_kernel<uint4><<<grid, 256, 0, st>>>((const uint4 *)x, (uint4 *)out, p); break;
  }
  dev->launches++;
  return check_launch(dev, "permute_kernel");
}

}  // extern "C"
