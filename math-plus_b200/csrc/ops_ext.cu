// The rest of the Backend's element-wise, comparison, selection, reduction and copy ops on the
// device (the method set of tensor-cpu's CpuBackendImpl, packages/tensor-cpu/src/index.ts:200-861,
// beyond the GEMM / attention path): HBM-bound grid-stride kernels.
//
// Every op evaluates in f64 (each stored type widens exactly) and rounds once on store, as the
// reference evaluates in f64 and rounds once: +, -, *, /, sqrt, maximum, neg, abs, relu, comparisons,
// selections, sums and extrema give the reference's bits; the transcendental ops (exp, log, tanh,
// sigmoid, erf, rsqrt, pow) differ from them only where CUDA's f64 functions and V8's differ in the
// last f64 place, which the rounding to f32 / f16 / bf16 almost always hides.
//
// Broadcasting is general: every operand carries element strides aligned to the output shape
// (0 on broadcast axes), up to 6 axes, the same rule as tensor-core's broadcastStrides.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cfloat>

#include "elem.cuh"
#include "mpc_internal.h"

namespace mpc {
namespace {

constexpr int kMaxRank = 6;

struct Index {
  int rank;
  long long shape[kMaxRank];
  long long st[3][kMaxRank];  // element strides of up to three inputs, aligned to shape
  long long total;
};

// Offsets of up to three inputs for the flat output index i (row-major over shape).
__device__ __forceinline__ void offsets(const Index &ix, long long i, long long (&off)[3]) {
  off[0] = off[1] = off[2] = 0;
#pragma unroll
  for (int k = kMaxRank - 1; k >= 0; --k) {
    if (k < ix.rank) {
      const long long q = i / ix.shape[k];
      const long long c = i - q * ix.shape[k];
      i = q;
      off[0] += c * ix.st[0][k];
      off[1] += c * ix.st[1][k];
      off[2] += c * ix.st[2][k];
    }
  }
}

__device__ __forceinline__ double unary_op(int op, double x, double alpha) {
  switch (op) {
    case MPC_OP_NEG:
      return -x;
    case MPC_OP_ABS:
      return fabs(x);
    case MPC_OP_EXP:
      return exp(x);
    case MPC_OP_LOG:
      return log(x);
    case MPC_OP_SQRT:
      return sqrt(x);
    case MPC_OP_RSQRT:
      return 1.0 / sqrt(x);
    case MPC_OP_TANH:
      return tanh(x);
    case MPC_OP_SIGMOID: {  // the overflow-free form of nn-kernels.ts:37-41
      if (x >= 0.0) return 1.0 / (1.0 + exp(-x));
      const double e = exp(x);
      return e / (1.0 + e);
    }
    case MPC_OP_RELU:
      return x > 0.0 ? x : 0.0;  // NaN -> 0, as nn-kernels.ts:27
    case MPC_OP_ERF:
      return erf(x);
    case MPC_OP_SCALE:
      return x * alpha;
    case MPC_OP_POW_SCALAR:
      return pow(x, alpha);
    case MPC_OP_LOGICAL_NOT:
      return x == 0.0 ? 1.0 : 0.0;
    default:
      return x;
  }
}

__device__ __forceinline__ double binary_op(int op, double a, double b) {
  switch (op) {
    case MPC_OP_ADD:
      return a + b;
    case MPC_OP_SUB:
      return a - b;
    case MPC_OP_MUL:
      return a * b;
    case MPC_OP_DIV:
      return a / b;
    case MPC_OP_MAXIMUM:
      return (a != a || b != b) ? a + b : fmax(a, b);  // NaN propagates, as Math.max
    case MPC_OP_POW:
      return pow(a, b);
    case MPC_OP_EQUAL:
      return a == b ? 1.0 : 0.0;
    case MPC_OP_NOT_EQUAL:
      return a != b ? 1.0 : 0.0;
    case MPC_OP_LESS:
      return a < b ? 1.0 : 0.0;
    case MPC_OP_LESS_EQUAL:
      return a <= b ? 1.0 : 0.0;
    case MPC_OP_GREATER:
      return a > b ? 1.0 : 0.0;
    case MPC_OP_GREATER_EQUAL:
      return a >= b ? 1.0 : 0.0;
    case MPC_OP_LOGICAL_AND:
      return (a != 0.0 && b != 0.0) ? 1.0 : 0.0;
    case MPC_OP_LOGICAL_OR:
      return (a != 0.0 || b != 0.0) ? 1.0 : 0.0;
    default:
      return a;
  }
}

__global__ void unary_kernel(int op, const void *__restrict__ x, int dti, void *__restrict__ out, int dto, int64_t n,
                             float alpha) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    st_d(out, dto, i, unary_op(op, ld_d(x, dti, i), (double)alpha));
}

__global__ void binary_kernel(int op, const void *__restrict__ x, const void *__restrict__ y, int dti,
                              void *__restrict__ out, int dto, const Index ix) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < ix.total;
       i += (long long)gridDim.x * blockDim.x) {
    long long off[3];
    offsets(ix, i, off);
    st_d(out, dto, i, binary_op(op, ld_d(x, dti, off[0]), ld_d(y, dti, off[1])));
  }
}

__global__ void where_kernel(const uint8_t *__restrict__ c, const void *__restrict__ x, const void *__restrict__ y,
                             int dt, void *__restrict__ out, const Index ix) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < ix.total;
       i += (long long)gridDim.x * blockDim.x) {
    long long off[3];
    offsets(ix, i, off);
    st_d(out, dt, i, c[off[0]] ? ld_d(x, dt, off[1]) : ld_d(y, dt, off[2]));
  }
}

// Strided copy of any element size: out[o-offset] = x[x-offset] over shape (st[0] = x, st[1] = out).
template <typename T>
__global__ void copy_kernel(const T *__restrict__ x, T *__restrict__ out, const Index ix) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < ix.total;
       i += (long long)gridDim.x * blockDim.x) {
    long long off[3];
    offsets(ix, i, off);
    out[off[1]] = x[off[0]];
  }
}

// Reduction of the middle axis of [outer, dim, inner], one thread per (outer, inner) lane (reads
// coalesced over inner). The order and comparisons are the reference's (kernels.ts:125-187,
// :543-568): sums accumulate in f64 in index order; max / min / argmax / argmin start from the
// first element and replace it only on a strict > / < (so a NaN counts only in first place).
__global__ void reduce_lanes_kernel(int op, const void *__restrict__ x, int dti, void *__restrict__ out, int dto,
                                    int64_t outer, int64_t dim, int64_t inner) {
  const int64_t lanes = outer * inner;
  for (int64_t l = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; l < lanes; l += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = l / inner, t = l - o * inner;
    const int64_t base = o * dim * inner + t;
    if (op == MPC_OP_SUM || op == MPC_OP_MEAN) {
      double acc = 0.0;
      for (int64_t j = 0; j < dim; ++j) acc += ld_d(x, dti, base + j * inner);
      st_d(out, dto, l, op == MPC_OP_MEAN ? acc / (double)dim : acc);
      continue;
    }
    const bool want_max = op == MPC_OP_MAX || op == MPC_OP_ARGMAX;
    double best = ld_d(x, dti, base);
    int bi = 0;
    for (int64_t j = 1; j < dim; ++j) {
      const double v = ld_d(x, dti, base + j * inner);
      if (want_max ? v > best : v < best) best = v, bi = (int)j;
    }
    if (op == MPC_OP_ARGMAX || op == MPC_OP_ARGMIN)
      static_cast<int32_t *>(out)[l] = bi;
    else
      st_d(out, dto, l, best);
  }
}

__global__ void cumsum_kernel(const void *__restrict__ x, int dti, void *__restrict__ out, int dto, int64_t outer,
                              int64_t dim, int64_t inner) {
  const int64_t lanes = outer * inner;
  for (int64_t l = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; l < lanes; l += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = l / inner, t = l - o * inner;
    const int64_t base = o * dim * inner + t;
    double acc = 0.0;
    for (int64_t j = 0; j < dim; ++j) {
      acc += ld_d(x, dti, base + j * inner);
      st_d(out, dto, base + j * inner, acc);
    }
  }
}

unsigned grid_of(mpc_device *dev, long long n) {
  const long long cap = (long long)dev->prop.multiProcessorCount * 8;
  long long g = (n + 255) / 256;
  if (g > cap) g = cap;
  return (unsigned)(g < 1 ? 1 : g);
}

bool any_dtype(int dt) { return dt >= MPC_F32 && dt <= MPC_BOOL; }

int make_index(Index &ix, int rank, const int64_t *shape, const int64_t *const *strides, int n_in, const char *who) {
  if (rank < 0 || rank > kMaxRank) return fail(MPC_ERR_UNSUPPORTED, "%s: rank %d (at most %d)", who, rank, kMaxRank);
  if (rank > 0 && !shape) return fail(MPC_ERR_INVALID, "%s: null shape", who);
  ix = Index{};
  ix.rank = rank;
  ix.total = 1;
  for (int k = 0; k < rank; ++k) {
    if (shape[k] < 0) return fail(MPC_ERR_INVALID, "%s: negative extent", who);
    ix.shape[k] = shape[k];
    ix.total *= shape[k];
    for (int a = 0; a < n_in; ++a) {
      if (!strides[a]) return fail(MPC_ERR_INVALID, "%s: null strides", who);
      if (strides[a][k] < 0) return fail(MPC_ERR_INVALID, "%s: negative stride", who);
      ix.st[a][k] = strides[a][k];
    }
  }
  for (int k = rank; k < kMaxRank; ++k) ix.shape[k] = 1;
  return MPC_OK;
}

}  // namespace
}  // namespace mpc

using namespace mpc;

extern "C" {

int mpc_unary(mpc_device *dev, int32_t op, const void *x, int32_t dtype_in, void *out, int32_t dtype_out, int64_t n,
              float alpha, mpc_stream s) {
  int rc = enter(dev);
  if (rc) return rc;
  if (op < MPC_OP_NEG || op > MPC_OP_LOGICAL_NOT) return fail(MPC_ERR_INVALID, "mpc_unary: op %d", op);
  if (!any_dtype(dtype_in) || !any_dtype(dtype_out)) return fail(MPC_ERR_INVALID, "mpc_unary: dtype");
  if (n < 0) return fail(MPC_ERR_INVALID, "mpc_unary: negative size");
  if (n == 0) return MPC_OK;
  if (!x || !out) return fail(MPC_ERR_INVALID, "mpc_unary: null pointer");
  unary_kernel<<<grid_of(dev, n), 256, 0, stream_of(dev, s)>>>(op, x, dtype_in, out, dtype_out, n, alpha);
  dev->launches++;
  return check_launch(dev, "unary_kernel");
}

int mpc_binary(mpc_device *dev, int32_t op, const void *x, const void *y, int32_t dtype_in, void *out,
               int32_t dtype_out, int32_t rank, const int64_t *shape, const int64_t *x_strides,
               const int64_t *y_strides, mpc_stream s) {
  int rc = enter(dev);
  if (rc) return rc;
  if (op < MPC_OP_ADD || op > MPC_OP_LOGICAL_OR) return fail(MPC_ERR_INVALID, "mpc_binary: op %d", op);
  if (!any_dtype(dtype_in) || !any_dtype(dtype_out)) return fail(MPC_ERR_INVALID, "mpc_binary: dtype");
  Index ix;
  const int64_t *st[2] = {x_strides, y_strides};
  if ((rc = make_index(ix, rank, shape, st, 2, "mpc_binary"))) return rc;
  if (ix.total == 0) return MPC_OK;
  if (!x || !y || !out) return fail(MPC_ERR_INVALID, "mpc_binary: null pointer");
  binary_kernel<<<grid_of(dev, ix.total), 256, 0, stream_of(dev, s)>>>(op, x, y, dtype_in, out, dtype_out, ix);
  dev->launches++;
  return check_launch(dev, "binary_kernel");
}

int mpc_where(mpc_device *dev, const uint8_t *cond, const void *x, const void *y, int32_t dtype, void *out,
              int32_t rank, const int64_t *shape, const int64_t *c_strides, const int64_t *x_strides,
              const int64_t *y_strides, mpc_stream s) {
  int rc = enter(dev);
  if (rc) return rc;
  if (!any_dtype(dtype)) return fail(MPC_ERR_INVALID, "mpc_where: dtype");
  Index ix;
  const int64_t *st[3] = {c_strides, x_strides, y_strides};
  if ((rc = make_index(ix, rank, shape, st, 3, "mpc_where"))) return rc;
  if (ix.total == 0) return MPC_OK;
  if (!cond || !x || !y || !out) return fail(MPC_ERR_INVALID, "mpc_where: null pointer");
  where_kernel<<<grid_of(dev, ix.total), 256, 0, stream_of(dev, s)>>>(cond, x, y, dtype, out, ix);
  dev->launches++;
  return check_launch(dev, "where_kernel");
}

int mpc_strided_copy(mpc_device *dev, const void *x, const int64_t *x_strides, void *out, const int64_t *out_strides,
                     int32_t elem_bytes, int32_t rank, const int64_t *shape, mpc_stream s) {
  int rc = enter(dev);
  if (rc) return rc;
  Index ix;
  const int64_t *st[2] = {x_strides, out_strides};
  if ((rc = make_index(ix, rank, shape, st, 2, "mpc_strided_copy"))) return rc;
  if (ix.total == 0) return MPC_OK;
  if (!x || !out) return fail(MPC_ERR_INVALID, "mpc_strided_copy: null pointer");
  const unsigned g = grid_of(dev, ix.total);
  cudaStream_t st_ = stream_of(dev, s);
  switch (elem_bytes) {
    case 1:
      copy_kernel<uint8_t><<<g, 256, 0, st_>>>((const uint8_t *)x, (uint8_t *)out, ix);
      break;
    case 2:
      copy_kernel<uint16_t><<<g, 256, 0, st_>>>((const uint16_t *)x, (uint16_t *)out, ix);
      break;
    case 4:
      copy_kernel<uint32_t><<<g, 256, 0, st_>>>((const uint32_t *)x, (uint32_t *)out, ix);
      break;
    case 8:
      copy_kernel<uint2><<<g, 256, 0, st_>>>((const uint2 *)x, (uint2 *)out, ix);
      break;
    default:
      return fail(MPC_ERR_INVALID, "mpc_strided_copy: element size %d", elem_bytes);
  }
  dev->launches++;
  return check_launch(dev, "copy_kernel");
}

int mpc_reduce(mpc_device *dev, int32_t op, const void *x, int32_t dtype_in, void *out, int32_t dtype_out,
               int64_t outer, int64_t dim, int64_t inner, mpc_stream s) {
  int rc = enter(dev);
  if (rc) return rc;
  if (op < MPC_OP_SUM || op > MPC_OP_ARGMIN) return fail(MPC_ERR_INVALID, "mpc_reduce: op %d", op);
  if (!any_dtype(dtype_in) || !any_dtype(dtype_out)) return fail(MPC_ERR_INVALID, "mpc_reduce: dtype");
  if ((op == MPC_OP_ARGMAX || op == MPC_OP_ARGMIN) && dtype_out != MPC_I32)
    return fail(MPC_ERR_INVALID, "mpc_reduce: argmax / argmin write i32");
  if (outer < 0 || dim < 0 || inner < 0) return fail(MPC_ERR_INVALID, "mpc_reduce: negative extent");
  if (dim == 0 && op != MPC_OP_SUM && op != MPC_OP_MEAN)
    return fail(MPC_ERR_INVALID, "mpc_reduce: max / min / argmax / argmin over an empty axis");
  if (outer == 0 || inner == 0) return MPC_OK;
  if (!out || (dim > 0 && !x)) return fail(MPC_ERR_INVALID, "mpc_reduce: null pointer");
  reduce_lanes_kernel<<<grid_of(dev, outer * inner), 256, 0, stream_of(dev, s)>>>(op, x, dtype_in, out, dtype_out,
                                                                                 outer, dim, inner);
  dev->launches++;
  return check_launch(dev, "reduce_lanes_kernel");
}

int mpc_cumsum(mpc_device *dev, const void *x, int32_t dtype_in, void *out, int32_t dtype_out, int64_t outer,
               int64_t dim, int64_t inner, mpc_stream s) {
  int rc = enter(dev);
  if (rc) return rc;
  if (!any_dtype(dtype_in) || !any_dtype(dtype_out)) return fail(MPC_ERR_INVALID, "mpc_cumsum: dtype");
  if (outer < 0 || dim < 0 || inner < 0) return fail(MPC_ERR_INVALID, "mpc_cumsum: negative extent");
  if (outer == 0 || dim == 0 || inner == 0) return MPC_OK;
  if (!x || !out) return fail(MPC_ERR_INVALID, "mpc_cumsum: null pointer");
  cumsum_kernel<<<grid_of(dev, outer * inner), 256, 0, stream_of(dev, s)>>>(x, dtype_in, out, dtype_out, outer, dim,
                                                                           inner);
  dev->launches++;
  return check_launch(dev, "cumsum_kernel");
}

}  // extern "C"
