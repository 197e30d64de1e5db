// The last of the Backend's ops on the device (tensor-cpu's CpuBackendImpl,
// packages/tensor-cpu/src/index.ts:724-861): sort along an axis, per-batch row gather, split-half
// rotary embedding, GEGLU and masked mean pooling. HBM-bound kernels; arithmetic in f64 with one
// rounding on store, as the reference evaluates in f64 and rounds once.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "elem.cuh"
#include "mpc_internal.h"

namespace mpc {
namespace {

bool float_type(int dt) { return dt == MPC_F32 || dt == MPC_F16 || dt == MPC_BF16; }
bool any_type(int dt) { return dt >= MPC_F32 && dt <= MPC_BOOL; }

unsigned grid_cap(mpc_device *dev, long long n, int threads) {
  const long long cap = (long long)dev->prop.multiProcessorCount * 8;
  long long g = (n + threads - 1) / threads;
  if (g > cap) g = cap;
  return (unsigned)(g < 1 ? 1 : g);
}

// ---- sort -------------------------------------------------------------------------------------
// Keys: every value maps to a uint32 whose unsigned order is the typed-array sort order of the
// reference (sortAxis, packages/tensor-core/src/kernels.ts:601-617, ``TypedArray.prototype.sort``):
// numeric ascending, -0 before +0, NaN last. Floats (f16 / bf16 widen exactly to f32) flip the
// sign bit of non-negatives and all bits of negatives; i32 flips the sign bit; bool is its byte.
// Padding past the lane's end is 0xffffffff, which sorts last (it ties only with NaN or INT32_MAX,
// which decode to the same values).
constexpr int kSortCap = 4096;     // keys sorted in shared memory by one CTA (16 KB)
constexpr int kSortThreads = 512;

__device__ __forceinline__ uint32_t sort_key(const void *p, int dt, int64_t i) {
  if (dt == MPC_I32) return (uint32_t) static_cast<const int32_t *>(p)[i] ^ 0x80000000u;
  if (dt == MPC_BOOL) return static_cast<const uint8_t *>(p)[i];
  const float f = (float)ld_d(p, dt, i);
  if (f != f) return 0xffffffffu;
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ void store_key(void *p, int dt, int64_t i, uint32_t k) {
  if (dt == MPC_I32) {
    static_cast<int32_t *>(p)[i] = (int32_t)(k ^ 0x80000000u);
  } else if (dt == MPC_BOOL) {
    static_cast<uint8_t *>(p)[i] = (uint8_t)k;
  } else {
    const uint32_t b = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
    st_d(p, dt, i, (double)__uint_as_float(b));
  }
}

// Bitonic stages over kSortCap keys in shared memory. A lane is n2 keys (a power of two); key e
// of the block sits at index (li_base + e) & (n2 - 1) of its lane, which sets each comparison's
// direction. For each k in [k_lo, k_hi] the stages j = min(k / 2, j_top) .. 1 run.
__device__ void bitonic_block(uint32_t *sk, int64_t n2, int64_t k_lo, int64_t k_hi, int64_t j_top, int64_t li_base) {
  for (int64_t k = k_lo; k <= k_hi; k <<= 1) {
    for (int64_t j = (k >> 1) < j_top ? (k >> 1) : j_top; j > 0; j >>= 1) {
      for (int q = threadIdx.x; q < kSortCap / 2; q += blockDim.x) {
        const int i = ((q & ~(int)(j - 1)) << 1) | (q & (int)(j - 1));
        const int l = i + (int)j;
        const bool asc = (((li_base + i) & (n2 - 1)) & k) == 0;
        const uint32_t a = sk[i], b = sk[l];
        if ((a > b) == asc) {
          sk[i] = b;
          sk[l] = a;
        }
      }
      __syncthreads();
    }
  }
}

// Lanes of n2 <= kSortCap keys, kSortCap / n2 lanes per CTA, read from x and written to out.
__global__ void __launch_bounds__(kSortThreads) sort_small_kernel(const void *__restrict__ x, int dt,
                                                                  void *__restrict__ out, int64_t lanes, int64_t dim,
                                                                  int64_t inner, int64_t n2) {
  __shared__ uint32_t sk[kSortCap];
  const int64_t per = kSortCap / n2;
  for (int64_t l0 = (int64_t)blockIdx.x * per; l0 < lanes; l0 += (int64_t)gridDim.x * per) {
    for (int e = threadIdx.x; e < kSortCap; e += blockDim.x) {
      const int64_t l = l0 + e / n2, j = e & (n2 - 1);
      uint32_t key = 0xffffffffu;
      if (l < lanes && j < dim) {
        const int64_t o = l / inner, t = l - o * inner;
        key = sort_key(x, dt, (o * dim + j) * inner + t);
      }
      sk[e] = key;
    }
    __syncthreads();
    bitonic_block(sk, n2, 2, n2, n2, 0);
    for (int e = threadIdx.x; e < kSortCap; e += blockDim.x) {
      const int64_t l = l0 + e / n2, j = e & (n2 - 1);
      if (l < lanes && j < dim) {
        const int64_t o = l / inner, t = l - o * inner;
        store_key(out, dt, (o * dim + j) * inner + t, sk[e]);
      }
    }
    __syncthreads();
  }
}

// Longer lanes: keys in a scratch array [lanes, n2], sorted by chunk stages in shared memory and
// compare-exchange stages in global memory.
__global__ void sort_fill_kernel(const void *__restrict__ x, int dt, uint32_t *__restrict__ keys, int64_t lanes,
                                 int64_t dim, int64_t inner, int64_t n2) {
  const int64_t total = lanes * n2;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t l = e / n2, j = e - l * n2;
    uint32_t key = 0xffffffffu;
    if (j < dim) {
      const int64_t o = l / inner, t = l - o * inner;
      key = sort_key(x, dt, (o * dim + j) * inner + t);
    }
    keys[e] = key;
  }
}

__global__ void __launch_bounds__(kSortThreads) sort_chunk_kernel(uint32_t *__restrict__ keys, int64_t chunks,
                                                                  int64_t n2, int64_t k_lo, int64_t k_hi,
                                                                  int64_t j_top) {
  __shared__ uint32_t sk[kSortCap];
  for (int64_t c = blockIdx.x; c < chunks; c += gridDim.x) {
    uint32_t *g = keys + c * kSortCap;
    for (int e = threadIdx.x; e < kSortCap; e += blockDim.x) sk[e] = g[e];
    __syncthreads();
    bitonic_block(sk, n2, k_lo, k_hi, j_top, (c * kSortCap) & (n2 - 1));
    for (int e = threadIdx.x; e < kSortCap; e += blockDim.x) g[e] = sk[e];
    __syncthreads();
  }
}

__global__ void sort_global_stage_kernel(uint32_t *__restrict__ keys, int64_t lanes, int64_t n2, int64_t k,
                                         int64_t j) {
  const int64_t pairs = lanes * (n2 >> 1);
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < pairs; p += (int64_t)gridDim.x * blockDim.x) {
    const int64_t l = p / (n2 >> 1), q = p - l * (n2 >> 1);
    const int64_t i = ((q & ~(j - 1)) << 1) | (q & (j - 1));
    const bool asc = (i & k) == 0;
    uint32_t *base = keys + l * n2;
    const uint32_t a = base[i], b = base[i + j];
    if ((a > b) == asc) {
      base[i] = b;
      base[i + j] = a;
    }
  }
}

__global__ void sort_store_kernel(const uint32_t *__restrict__ keys, int dt, void *__restrict__ out, int64_t lanes,
                                  int64_t dim, int64_t inner, int64_t n2) {
  const int64_t total = lanes * dim;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t l = e / dim, j = e - l * dim;
    const int64_t o = l / inner, t = l - o * inner;
    store_key(out, dt, (o * dim + j) * inner + t, keys[l * n2 + j]);
  }
}

// ---- gatherRows -------------------------------------------------------------------------------
template <typename T>
__global__ void gather_rows_kernel(const T *__restrict__ x, const int32_t *__restrict__ idx, T *__restrict__ out,
                                   int64_t L, int64_t M, int64_t D, int64_t total, unsigned long long *bad) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t bm = e / D, c = e - bm * D;
    const int64_t b = bm / M;
    const int64_t raw = idx[bm];
    const int64_t r = raw < 0 ? raw + L : raw;
    if (r < 0 || r >= L) {
      atomicMin(bad, (unsigned long long)bm);
      continue;
    }
    out[e] = x[(b * L + r) * D + c];
  }
}

__global__ void rows_check_kernel(const int32_t *__restrict__ idx, int64_t L, int64_t n, unsigned long long *bad) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t raw = idx[e];
    const int64_t r = raw < 0 ? raw + L : raw;
    if (r < 0 || r >= L) atomicMin(bad, (unsigned long long)e);
  }
}

// ---- rope -------------------------------------------------------------------------------------
// Split-half rotary embedding (ropeHalf, packages/tensor-core/src/nn-kernels.ts:138-160) over BH
// contiguous [L, Dh] blocks. The angle follows the reference's f32 roundings: inv_freq =
// f32(2^f32(-f32(i / half) · f32(log2 base))), θ = f32(p · inv_freq); cos θ and sin θ in f64; the
// rotation in f64 (no fused multiply-add) with one rounding on store. One thread per (p, i) pair
// computes the angle once and walks the blocks.
__global__ void rope_kernel(const void *__restrict__ x, int dt, void *__restrict__ out, int64_t bh_count, int64_t L,
                            int64_t half, float lb) {
  const int64_t pairs = L * half;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < pairs; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = e / half, i = e - p * half;
    const float fi = __double2float_rn((double)i / (double)half);
    const float y = __double2float_rn(-(double)fi * (double)lb);
    const float inv_freq = __double2float_rn(exp2((double)y));
    const float th = __double2float_rn((double)p * (double)inv_freq);
    double s, c;
    sincos((double)th, &s, &c);
    for (int64_t bh = blockIdx.y; bh < bh_count; bh += gridDim.y) {
      const int64_t base = (bh * L + p) * 2 * half;
      const double x1 = ld_d(x, dt, base + i), x2 = ld_d(x, dt, base + half + i);
      st_d(out, dt, base + i, __dsub_rn(__dmul_rn(x1, c), __dmul_rn(x2, s)));
      st_d(out, dt, base + half + i, __dadd_rn(__dmul_rn(x2, c), __dmul_rn(x1, s)));
    }
  }
}

// ---- geglu ------------------------------------------------------------------------------------
// gegluRows (nn-kernels.ts:245-250): o[r, j] = GELU(x[r, j]) · x[r, D + j], GELU = v·Φ(v) in f64.
__global__ void geglu_kernel(const void *__restrict__ x, int dt, void *__restrict__ out, int64_t rows, int64_t D) {
  const int64_t total = rows * D;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = e / D, j = e - r * D;
    const double v = ld_d(x, dt, r * 2 * D + j), g = ld_d(x, dt, r * 2 * D + D + j);
    st_d(out, dt, e, __dmul_rn(__dmul_rn(v, normcdf(v)), g));
  }
}

// ---- meanPool ---------------------------------------------------------------------------------
// maskedMeanPool (nn-kernels.ts:256-271): x [B, L, D], mask [B, L] (nonzero and not NaN = keep) ->
// o [B, D]; an f64 sum over the kept positions in order, times 1 / max(count, 1). One thread per
// (b, j): the threads of a warp read consecutive j of the same row.
__global__ void mean_pool_kernel(const void *__restrict__ x, int dt, const void *__restrict__ mask, int mdt,
                                 void *__restrict__ out, int64_t B, int64_t L, int64_t D) {
  const int64_t total = B * D;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = e / D, j = e - b * D;
    double acc = 0.0;
    int64_t cnt = 0;
    for (int64_t l = 0; l < L; ++l) {
      const double m = ld_d(mask, mdt, b * L + l);
      if (m == 0.0 || m != m) continue;
      ++cnt;
      acc = __dadd_rn(acc, ld_d(x, dt, (b * L + l) * D + j));
    }
    st_d(out, dt, e, __dmul_rn(acc, 1.0 / (double)(cnt > 1 ? cnt : 1)));
  }
}

}  // namespace
}  // namespace mpc

using namespace mpc;

extern "C" {

int mpc_sort(mpc_device *dev, const void *x, int32_t dtype, void *out, int64_t outer, int64_t dim, int64_t inner,
             mpc_stream s) {
  int rc = enter(dev);
  if (rc) return rc;
  if (!any_type(dtype)) return fail(MPC_ERR_INVALID, "mpc_sort: dtype %d", dtype);
  if (outer < 0 || dim < 0 || inner < 0) return fail(MPC_ERR_INVALID, "mpc_sort: negative extent");
  if (outer == 0 || dim == 0 || inner == 0) return MPC_OK;
  if (!x || !out) return fail(MPC_ERR_INVALID, "mpc_sort: null pointer");
  if (dim > (int64_t(1) << 30)) return fail(MPC_ERR_UNSUPPORTED, "mpc_sort: lanes longer than 2^30");
  const int64_t lanes = outer * inner;
  int64_t n2 = 1;
  while (n2 < dim) n2 <<= 1;
  cudaStream_t st = stream_of(dev, s);
  if (n2 <= kSortCap) {
    const int64_t per = kSortCap / n2;
    sort_small_kernel<<<grid_cap(dev, (lanes + per - 1) / per * kSortThreads, kSortThreads), kSortThreads, 0, st>>>(
        x, dtype, out, lanes, dim, inner, n2);
    dev->launches++;
    return check_launch(dev, "sort_small_kernel");
  }
  Scratch keys;
  if ((rc = keys.get(dev, st, (size_t)(lanes * n2) * sizeof(uint32_t)))) return rc;
  uint32_t *k = static_cast<uint32_t *>(keys.ptr);
  sort_fill_kernel<<<grid_cap(dev, lanes * n2, 256), 256, 0, st>>>(x, dtype, k, lanes, dim, inner, n2);
  dev->launches++;
  const int64_t chunks = lanes * n2 / kSortCap;
  const unsigned gc = grid_cap(dev, chunks * kSortThreads, kSortThreads);
  sort_chunk_kernel<<<gc, kSortThreads, 0, st>>>(k, chunks, n2, 2, kSortCap, kSortCap);
  dev->launches++;
  for (int64_t kk = 2 * kSortCap; kk <= n2; kk <<= 1) {
    for (int64_t j = kk >> 1; j >= kSortCap; j >>= 1) {
      sort_global_stage_kernel<<<grid_cap(dev, lanes * (n2 >> 1), 256), 256, 0, st>>>(k, lanes, n2, kk, j);
      dev->launches++;
    }
    sort_chunk_kernel<<<gc, kSortThreads, 0, st>>>(k, chunks, n2, kk, kk, kSortCap / 2);
    dev->launches++;
  }
  sort_store_kernel<<<grid_cap(dev, lanes * dim, 256), 256, 0, st>>>(k, dtype, out, lanes, dim, inner, n2);
  dev->launches++;
  return check_launch(dev, "sort_store_kernel");
}

int mpc_gather_rows(mpc_device *dev, const void *x, int32_t dtype, const int32_t *idx, void *out, int64_t B, int64_t L,
                    int64_t M, int64_t D, int64_t *bad_index, mpc_stream s) {
  int rc = enter(dev);
  if (rc) return rc;
  if (bad_index) *bad_index = -1;
  if (!any_type(dtype)) return fail(MPC_ERR_INVALID, "mpc_gather_rows: dtype %d", dtype);
  if (B < 0 || L < 0 || M < 0 || D < 0) return fail(MPC_ERR_INVALID, "mpc_gather_rows: negative extent");
  if (B == 0 || M == 0) return MPC_OK;
  if (!idx || (D > 0 && (!x || !out))) return fail(MPC_ERR_INVALID, "mpc_gather_rows: null pointer");
  cudaStream_t st = stream_of(dev, s);
  Scratch flag;
  if ((rc = flag.get(dev, st, sizeof(unsigned long long)))) return rc;
  MPC_CUDA(dev, cudaMemsetAsync(flag.ptr, 0xff, sizeof(unsigned long long), st));
  unsigned long long *bad = static_cast<unsigned long long *>(flag.ptr);
  const int64_t total = B * M * D;
  const unsigned g = grid_cap(dev, D > 0 ? total : B * M, 256);
  const size_t eb = dtype_size(dtype);
  if (D == 0) {  // nothing to copy; the indices are still checked
    rows_check_kernel<<<g, 256, 0, st>>>(idx, L, B * M, bad);
  } else if (eb == 4) {
    gather_rows_kernel<uint32_t><<<g, 256, 0, st>>>(static_cast<const uint32_t *>(x), idx, static_cast<uint32_t *>(out),
                                                     L, M, D, total, bad);
  } else if (eb == 2) {
    gather_rows_kernel<uint16_t><<<g, 256, 0, st>>>(static_cast<const uint16_t *>(x), idx, static_cast<uint16_t *>(out),
                                                     L, M, D, total, bad);
  } else {
    gather_rows_kernel<uint8_t><<<g, 256, 0, st>>>(static_cast<const uint8_t *>(x), idx, static_cast<uint8_t *>(out),
                                                    L, M, D, total, bad);
  }
  dev->launches++;
  if ((rc = check_launch(dev, "gather_rows_kernel"))) return rc;
  unsigned long long b = 0;
  MPC_CUDA(dev, cudaMemcpyAsync(&b, flag.ptr, sizeof(b), cudaMemcpyDeviceToHost, st));
  MPC_CUDA(dev, cudaStreamSynchronize(st));
  if (b != ~0ull) {
    if (bad_index) *bad_index = (int64_t)b;
    return fail(MPC_ERR_INVALID, "mpc_gather_rows: index at position %llu is out of range for length %lld", b,
                (long long)L);
  }
  return MPC_OK;
}

int mpc_rope(mpc_device *dev, const void *x, int32_t dtype, void *out, int64_t bh, int64_t L, int64_t dh, double base,
             mpc_stream s) {
  int rc = enter(dev);
  if (rc) return rc;
  if (!float_type(dtype)) return fail(MPC_ERR_INVALID, "mpc_rope: float dtypes only");
  if (bh < 0 || L < 0 || dh < 0) return fail(MPC_ERR_INVALID, "mpc_rope: negative extent");
  if (dh % 2) return fail(MPC_ERR_INVALID, "mpc_rope: needs an even head dim, got %lld", (long long)dh);
  if (bh == 0 || L == 0 || dh == 0) return MPC_OK;
  if (!x || !out) return fail(MPC_ERR_INVALID, "mpc_rope: null pointer");
  const int64_t half = dh / 2, pairs = L * half;
  const float lb = (float)log2(base);
  const unsigned gx = grid_cap(dev, pairs, 256);
  const long long want = (long long)dev->prop.multiProcessorCount * 8 / gx;
  const unsigned gy = (unsigned)(bh < want ? bh : (want < 1 ? 1 : (want > 65535 ? 65535 : want)));
  rope_kernel<<<dim3(gx, gy), 256, 0, stream_of(dev, s)>>>(x, dtype, out, bh, L, half, lb);
  dev->launches++;
  return check_launch(dev, "rope_kernel");
}

int mpc_geglu(mpc_device *dev, const void *x, int32_t dtype, void *out, int64_t rows, int64_t d, mpc_stream s) {
  int rc = enter(dev);
  if (rc) return rc;
  if (!float_type(dtype)) return fail(MPC_ERR_INVALID, "mpc_geglu: float dtypes only");
  if (rows < 0 || d < 0) return fail(MPC_ERR_INVALID, "mpc_geglu: negative extent");
  if (rows == 0 || d == 0) return MPC_OK;
  if (!x || !out) return fail(MPC_ERR_INVALID, "mpc_geglu: null pointer");
  geglu_kernel<<<grid_cap(dev, rows * d, 256), 256, 0, stream_of(dev, s)>>>(x, dtype, out, rows, d);
  dev->launches++;
  return check_launch(dev, "geglu_kernel");
}

int mpc_mean_pool(mpc_device *dev, const void *x, int32_t dtype, const void *mask, int32_t mask_dtype, void *out,
                  int64_t B, int64_t L, int64_t D, mpc_stream s) {
  int rc = enter(dev);
  if (rc) return rc;
  if (!float_type(dtype)) return fail(MPC_ERR_INVALID, "mpc_mean_pool: float dtypes only");
  if (!any_type(mask_dtype)) return fail(MPC_ERR_INVALID, "mpc_mean_pool: mask dtype %d", mask_dtype);
  if (B < 0 || L < 0 || D < 0) return fail(MPC_ERR_INVALID, "mpc_mean_pool: negative extent");
  if (B == 0 || D == 0) return MPC_OK;
  if (!out || (L > 0 && (!x || !mask))) return fail(MPC_ERR_INVALID, "mpc_mean_pool: null pointer");
  mean_pool_kernel<<<grid_cap(dev, B * D, 256), 256, 0, stream_of(dev, s)>>>(x, dtype, mask, mask_dtype, out, B, L,
                                                                            D);
  dev->launches++;
  return check_launch(dev, "mean_pool_kernel");
}

}  // extern "C"
