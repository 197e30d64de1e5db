/*
 * libmathplus_cuda.so — the C ABI of the math-plus CUDA device backend (B200, sm_100a).
 *
 * This is the boundary a math-plus device facade binds (Node-API, Deno.dlopen, bun:ffi or
 * Python ctypes): plain pointers, sizes in bytes or elements, C linkage, an int status on
 * every call and no C++ or torch types. It replaces, for the GEMM / attention path, what the
 * WebGPU runtime does under packages/tensor-webgpu (the external @johnhenry/backend-webgpu
 * kernels) and what tensor-cpu's Backend does on the host:
 *
 *   mpc_gemm   <- Backend.matmul / Backend.linear   (packages/tensor-cpu/src/index.ts:755-774)
 *   mpc_sdpa   <- Backend.sdpa                      (packages/tensor-cpu/src/index.ts:821-840)
 *   mpc_softmax, mpc_gelu, mpc_add, mpc_layer_norm, mpc_embedding, mpc_cast
 *              <- Backend.softmax/gelu/add/layerNorm/embedding/cast (index.ts:598, 716-722, 776-791, 406-425)
 *   mpc_memcpy_h2d_async / mpc_memcpy_d2h_async
 *              <- Backend.fromHost / Backend.read   (packages/tensor-cpu/src/index.ts:216-260)
 *
 * Conventions (kept from the reference's native FFI, crates/tensor-wasm-kernels/src/lib.rs:17-38
 * and packages/tensor-wasm/src/native.ts:96-104): every call returns an mpc_status and never
 * aborts; a failed call leaves a message for mpc_last_error(); strides and offsets are in
 * ELEMENTS; a NULL stream means the device's own stream.
 */
#ifndef MATHPLUS_CUDA_H
#define MATHPLUS_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default) /* the library builds with hidden visibility; export only this API */
#endif

#define MPC_ABI_VERSION 1

typedef enum {
  MPC_OK = 0,
  MPC_ERR_INVALID = 1,     /* bad argument: shape, stride, dtype, null pointer */
  MPC_ERR_UNSUPPORTED = 2, /* valid request this build does not implement */
  MPC_ERR_OOM = 3,         /* device allocation failed (or the allocator cap was reached) */
  MPC_ERR_CUDA = 4,        /* a CUDA runtime / driver call failed */
  MPC_ERR_TIMEOUT = 5,     /* a kernel's bounded wait ran out; the kernel returned early */
  MPC_ERR_POISONED = 6,    /* an earlier fault poisoned this device handle: destroy it */
  MPC_ERR_NO_DEVICE = 7,   /* no CUDA device / not an sm_100 device */
  MPC_ERR_COMM = 8,        /* NCCL unavailable or a collective failed */
  MPC_ERR_COMPILE = 9      /* NVRTC unavailable or it could not compile a fused expression */
} mpc_status;

typedef enum { MPC_F32 = 0, MPC_F16 = 1, MPC_BF16 = 2, MPC_I32 = 3, MPC_BOOL = 4 } mpc_dtype;

typedef struct mpc_device mpc_device; /* one per CUDA device ordinal and process */
typedef void *mpc_stream;             /* a cudaStream_t; NULL = the device's own stream */
typedef void *mpc_event;              /* a cudaEvent_t */
typedef struct mpc_comm mpc_comm;     /* an NCCL communicator (one rank of a group) */
typedef struct mpc_fused mpc_fused;   /* a compiled fused element-wise expression */

typedef struct {
  char name[128];
  int ordinal;
  int cc_major, cc_minor;
  int sm_count;
  size_t total_bytes;
  size_t smem_per_block_optin;
  int runtime_version, driver_version;
} mpc_device_info_t;

/* ---- device and errors (no reference counterpart beyond createWebGpuDevice,
 *      packages/tensor-webgpu/src/facade.ts:52-64, and detectWebGPU, src/device.ts:87-121) */
int mpc_version(void);
int mpc_device_count(int *count);
int mpc_device_create(int ordinal, unsigned flags, mpc_device **dev);
int mpc_device_destroy(mpc_device *dev);
int mpc_device_info(mpc_device *dev, mpc_device_info_t *info);
/* Thread-local message of the last failed call on this thread (dev may be NULL). */
const char *mpc_last_error(mpc_device *dev);
/* Status of the device handle: MPC_OK, or the sticky MPC_ERR_POISONED / MPC_ERR_TIMEOUT. */
int mpc_device_status(mpc_device *dev);
/* Limit for every in-kernel bounded wait (nanoseconds; 0 restores the default). */
int mpc_set_wait_timeout_ns(mpc_device *dev, uint64_t ns);
/* Clears a recorded MPC_ERR_TIMEOUT once the caller has handled it (not a poisoned handle). */
int mpc_device_clear_error(mpc_device *dev);
/* Failure-path self test: launches one wait on an mbarrier nothing releases, with the given
 * limit; returns MPC_ERR_TIMEOUT once the kernel has given up and returned (the context stays
 * usable; clear it with mpc_device_clear_error). No fault, trap or hang is involved. */
int mpc_selftest_wait_timeout(mpc_device *dev, uint64_t timeout_ns);

/* ---- memory: a caching allocator per device (Backend.fromHost's one copy, index.ts:225) ----
 * Stream-ordered like the library's kernels: mpc_free returns a block at the current point of the
 * device stream, and mpc_alloc may hand it out again at once, for work queued on the device stream
 * after that point. Work that uses a block on another stream must first wait for the device
 * stream (an event recorded there). */
int mpc_alloc(mpc_device *dev, size_t bytes, void **ptr);
int mpc_free(mpc_device *dev, void *ptr);
/* Cap on bytes handed out by mpc_alloc (0 = no cap): lets tests inject allocation failure. */
int mpc_set_alloc_limit(mpc_device *dev, size_t bytes);
int mpc_alloc_stats(mpc_device *dev, size_t *in_use, size_t *cached);
int mpc_trim(mpc_device *dev);
int mpc_host_alloc(mpc_device *dev, size_t bytes, void **ptr); /* pinned host memory */
int mpc_host_free(mpc_device *dev, void *ptr);
int mpc_memcpy_h2d_async(mpc_device *dev, void *dst, const void *src, size_t bytes, mpc_stream s);
int mpc_memcpy_d2h_async(mpc_device *dev, void *dst, const void *src, size_t bytes, mpc_stream s);
int mpc_memcpy_d2d_async(mpc_device *dev, void *dst, const void *src, size_t bytes, mpc_stream s);
int mpc_memset_async(mpc_device *dev, void *dst, int value, size_t bytes, mpc_stream s);

/* ---- streams and events (the GPU profiler of backend-webgpu, packages/tensor-webgpu/README.md:111-115) */
int mpc_stream_create(mpc_device *dev, mpc_stream *s);
int mpc_stream_destroy(mpc_device *dev, mpc_stream s);
int mpc_stream_sync(mpc_device *dev, mpc_stream s);
int mpc_device_stream(mpc_device *dev, mpc_stream *s);
int mpc_event_create(mpc_device *dev, mpc_event *e);
int mpc_event_destroy(mpc_device *dev, mpc_event e);
int mpc_event_record(mpc_device *dev, mpc_event e, mpc_stream s);
/* Work queued on s after this call waits for e's last recording (cross-stream ordering). */
int mpc_stream_wait_event(mpc_device *dev, mpc_stream s, mpc_event e);
int mpc_event_elapsed_ms(mpc_device *dev, mpc_event start, mpc_event stop, float *ms);
/* Waits for all work of the device, then reports any kernel-side error word. */
int mpc_sync(mpc_device *dev);
/* Number of this library's kernels launched on the device so far. */
int mpc_launch_count(mpc_device *dev, uint64_t *count);

/* ---- GEMM: C = epilogue(alpha * A·B) ------------------------------------------------------
 * Replaces Backend.matmul (B is [K,N]; packages/tensor-cpu/src/index.ts:755-762 ->
 * Tensor.matmul, packages/tensor-core/src/index.ts:1584-1730) and Backend.linear (B is a
 * PyTorch [N,K] weight plus bias; index.ts:764-774 -> linearNT, nn-kernels.ts:74-101), and the
 * DeviceArray chain matmul -> add(bias) -> gelu fused into one kernel.
 * f16 / bf16 inputs run on tcgen05 (f32 accumulation); f32 inputs run 3xTF32 on tcgen05.
 * A is [batch.., M, K] and C is [batch, M, N], both row-major; bias is f32 [N]. */
enum { MPC_EPI_BIAS = 1, MPC_EPI_GELU = 2, MPC_EPI_RESIDUAL = 4 };
enum { MPC_B_KN = 0, MPC_B_NK = 1 };
typedef struct {
  int64_t m, n, k;
  int32_t dtype_in;   /* MPC_F32, MPC_F16 or MPC_BF16 (A and B alike) */
  int32_t dtype_out;  /* MPC_F32, MPC_F16 or MPC_BF16 */
  int32_t b_layout;   /* MPC_B_KN (matmul) or MPC_B_NK (linear) */
  int32_t epilogue;   /* MPC_EPI_* flags */
  float alpha;        /* scale applied to A·B before the bias */
  int32_t batch_rank; /* 0..4 batch axes, output batch shape below (C-contiguous) */
  int64_t batch_shape[4];
  int64_t a_batch_stride[4]; /* element strides of A / B per batch axis; 0 = broadcast */
  int64_t b_batch_stride[4];
} mpc_gemm_desc;
int mpc_gemm(mpc_device *dev, const mpc_gemm_desc *desc, const void *A, const void *B, void *C,
             const float *bias, mpc_stream s);
/* mpc_gemm with MPC_EPI_RESIDUAL: C = act(alpha * A·B + bias) + R, R [batch, M, N] contiguous in
 * C's dtype (the residual add of a transformer block, DeviceArray.add after linear, fused into
 * the GEMM's epilogue). R may be C itself (in-place accumulate). */
int mpc_gemm_residual(mpc_device *dev, const mpc_gemm_desc *desc, const void *A, const void *B, void *C,
                      const float *bias, const void *R, mpc_stream s);

/* What the GEMM and attention kernels use on a device (gemmCapabilities,
 * packages/tensor-webgpu/src/gemm-caps.ts:60-86: the record of optional features a device's GEMM
 * may use). Advisory: every call still runs on the device whatever the record says. */
typedef struct {
  int32_t f16;                    /* f16 operands, f32 accumulation (tcgen05.mma kind::f16) */
  int32_t bf16;                   /* bf16 operands, f32 accumulation */
  int32_t f32_3xtf32;             /* f32 operands as 3xTF32 (kind::tf32 on hi / lo parts) */
  int32_t cta_pairs;              /* 256 x 256 output tiles on the two SMs of a TPC (cta_group::2) */
  int32_t sm_count;
  int32_t pair_min_tiles;         /* f16 / bf16 problems with at least this many 256 x 256 tiles run on pairs */
  int32_t tf32_narrow_below;      /* f32 problems with fewer 128 x 128 tiles than this run 128 x 64 tiles */
  int32_t attention_tc_head_dims; /* bit mask of head dims on the tensor-core attention path: 1 = 64, 2 = 128 */
  int32_t attention_max_head_dim; /* largest head dim of the CUDA-core attention path */
  int32_t reserved;
  int64_t max_dim;                /* largest M, N, K (and attention L) */
} mpc_gemm_caps;
int mpc_gemm_capabilities(mpc_device *dev, mpc_gemm_caps *caps);

/* Allocation-free variant of the f32 (3xTF32) path of mpc_gemm. It has no counterpart in the
 * reference: it exists for callers that cannot allocate device memory (a host runtime that owns
 * every device byte, or hands this library a fixed budget it may not grow). Its scratch (the tf32
 * hi/lo planes, and a padded copy of C when C's rows are not 16-byte aligned) lives in one static
 * device array of 32 MiB that every GPU loading the library holds until exit; requests needing more
 * return MPC_ERR_INVALID. It uses the calling thread's current device and the given stream (NULL =
 * the legacy default stream) and needs no mpc_device. The first call on a device resolves the
 * array's address (cudaGetSymbolAddress): make it before any stream capture; that set-up is not
 * redone after cudaDeviceReset. All calls share the array: calls that overlap on the GPU race.
 * desc must say f32 in and out; everything else is as for mpc_gemm. A kernel wait that runs out is
 * not reported by the call itself (it returns before the kernels run): see
 * mpc_gemm_f32_noalloc_status. */
int mpc_gemm_f32_noalloc(const mpc_gemm_desc *desc, const float *A, const float *B, float *C,
                         const float *bias, mpc_stream s);
/* Waits for stream s, then reports whether a bounded wait inside any mpc_gemm_f32_noalloc kernel on
 * the current device ran out since the last query (MPC_ERR_TIMEOUT: that call's C is incomplete) and
 * clears the record. Allocates nothing. */
int mpc_gemm_f32_noalloc_status(mpc_stream s);
/* Failure-path self test of that record: one wait on an mbarrier nothing releases, limited to
 * timeout_ns, recorded where mpc_gemm_f32_noalloc's kernels record theirs (no fault, trap or hang). */
int mpc_gemm_f32_noalloc_selftest(uint64_t timeout_ns, mpc_stream s);

/* ---- fused scaled-dot-product attention ----------------------------------------------------
 * softmax(scale * Q·Kᵀ + mask) · V over Q [B,H,Lq,D], K [B,Hk,Lk,D], V [B,Hk,Lk,Dv] into
 * O [B,H,Lq,Dv] (all contiguous), H a multiple of Hk (grouped-query heads share K/V).
 * Replaces Backend.sdpa (packages/tensor-cpu/src/index.ts:821-840 -> attention,
 * packages/tensor-core/src/nn-kernels.ts:179-239). causal = 1 hides key j from query i when
 * j > i (the [Lq,Lk] lower-triangular bool mask of the reference tests). A query row with no
 * visible key yields zeros (nn-kernels.ts:222-225). LSE (optional, f32 [B,H,Lq]) receives the
 * natural-log softmax normaliser of each row (-inf for a fully masked row). */
enum { MPC_MASK_NONE = 0, MPC_MASK_BOOL = 1, MPC_MASK_ADD = 2 };
typedef struct {
  int64_t b, h, hk, lq, lk, d, dv;
  int32_t dtype;     /* MPC_F16 / MPC_BF16 (tcgen05 path) or MPC_F32 (CUDA-core path); O has this dtype */
  int32_t causal;
  float scale;
  int32_t mask_kind; /* MPC_MASK_* ; mask is u8 (bool) or f32 (additive) */
  int64_t mask_strides[4]; /* element strides aligned to [B,H,Lq,Lk]; 0 = broadcast */
} mpc_sdpa_desc;
int mpc_sdpa(mpc_device *dev, const mpc_sdpa_desc *desc, const void *Q, const void *K, const void *V,
             const void *mask, void *O, float *LSE, mpc_stream s);
/* mpc_sdpa over strided Q / K / V / O: element strides of the (batch, head, row) axes, the head-dim
 * axis contiguous. It reads a packed projection [B, L, 3, H, D] in place (Q = base, K = base + H*D,
 * V = base + 2*H*D, each with strides (3*L*H*D, D, 3*H*D)) and writes O as [B, L, H, D]
 * (strides (L*H*D, D, H*D)), the layout of MultiheadAttention before out_proj
 * (packages/tensor-autograd/src/transformer.ts:223-241), with no head split / merge copies.
 * The tensor-core path needs every stride times 2 bytes to be a multiple of 16. */
typedef struct {
  int64_t q[3], k[3], v[3], o[3];
} mpc_sdpa_layout;
int mpc_sdpa_strided(mpc_device *dev, const mpc_sdpa_desc *desc, const void *Q, const void *K, const void *V,
                     const void *mask, void *O, float *LSE, const mpc_sdpa_layout *layout, mpc_stream s);

/* ---- the element-wise / row ops the GEMM and attention path touches ------------------------ */
/* softmax along the middle axis of a contiguous [outer, dim, inner] block, f32 out
 * (Backend.softmax -> softmaxAxis, packages/tensor-core/src/kernels.ts:219-247). */
int mpc_softmax(mpc_device *dev, const void *x, int32_t dtype, float *out, int64_t outer, int64_t dim,
                int64_t inner, mpc_stream s);
/* exact-erf GELU (Backend.gelu -> geluErf, packages/special/src/index.ts:191-193). */
int mpc_gelu(mpc_device *dev, const void *x, int32_t dtype_in, void *out, int32_t dtype_out, int64_t n,
             mpc_stream s);
/* out = x + y with y broadcast as a [rows_y, n] block repeated (rows_y = 1 for a bias row)
 * (Backend.add, packages/tensor-cpu/src/device-array.ts:289-291). */
int mpc_add(mpc_device *dev, const void *x, const void *y, void *out, int32_t dtype, int64_t n_x,
            int64_t n_y, mpc_stream s);
/* LayerNorm over the last axis (Backend.layerNorm -> layerNormRows, nn-kernels.ts:108-129). */
int mpc_layer_norm(mpc_device *dev, const void *x, int32_t dtype_in, const float *weight, const float *bias,
                   float eps, void *out, int32_t dtype_out, int64_t rows, int64_t d, mpc_stream s);
/* Row gather (Backend.embedding -> takeRows, nn-kernels.ts:277-286). An out-of-range id
 * returns MPC_ERR_INVALID after the call (the offending position goes to *bad_index). */
int mpc_embedding(mpc_device *dev, const void *table, int32_t dtype, const int32_t *ids, void *out,
                  int64_t n_ids, int64_t rows, int64_t d, int64_t *bad_index, mpc_stream s);
/* Element type conversion f32 <-> f16 / bf16, RNE (Backend.cast, index.ts:406-425). */
int mpc_cast(mpc_device *dev, const void *x, int32_t dtype_in, void *out, int32_t dtype_out, int64_t n,
             mpc_stream s);

/* Axis permutation of a contiguous tensor of up to 6 axes: out has shape shape[perm[k]]
 * (Backend.transpose, packages/tensor-cpu/src/device-array.ts:459-471; also the head split /
 * merge of attention and the reassembly of a column-split GEMM). */
int mpc_transpose(mpc_device *dev, const void *x, void *out, int32_t elem_bytes, int32_t rank, const int64_t *shape,
                  const int32_t *perm, mpc_stream s);

/* ---- the rest of the Backend op set (CpuBackendImpl, packages/tensor-cpu/src/index.ts:560-735) --
 * Arithmetic in f64 (every stored type widens exactly), one rounding on store. Operand
 * strides are element strides aligned to the output shape, 0 on broadcast axes (at most 6 axes).
 * Comparison and logical results are bool (u8 0 / 1); argmax / argmin write i32. */
enum {
  MPC_OP_NEG = 1, MPC_OP_ABS, MPC_OP_EXP, MPC_OP_LOG, MPC_OP_SQRT, MPC_OP_RSQRT, MPC_OP_TANH, MPC_OP_SIGMOID,
  MPC_OP_RELU, MPC_OP_ERF, MPC_OP_SCALE, MPC_OP_POW_SCALAR, MPC_OP_LOGICAL_NOT,           /* unary */
  MPC_OP_ADD = 32, MPC_OP_SUB, MPC_OP_MUL, MPC_OP_DIV, MPC_OP_MAXIMUM, MPC_OP_POW, MPC_OP_EQUAL,
  MPC_OP_NOT_EQUAL, MPC_OP_LESS, MPC_OP_LESS_EQUAL, MPC_OP_GREATER, MPC_OP_GREATER_EQUAL,
  MPC_OP_LOGICAL_AND, MPC_OP_LOGICAL_OR,                                                  /* binary */
  MPC_OP_SUM = 64, MPC_OP_MEAN, MPC_OP_MAX, MPC_OP_MIN, MPC_OP_ARGMAX, MPC_OP_ARGMIN     /* reductions */
};
/* out[i] = op(x[i]) (alpha: the factor of SCALE, the exponent of POW_SCALAR). */
int mpc_unary(mpc_device *dev, int32_t op, const void *x, int32_t dtype_in, void *out, int32_t dtype_out, int64_t n,
              float alpha, mpc_stream s);
/* out = op(x, y) over shape[rank] with broadcast strides. */
int mpc_binary(mpc_device *dev, int32_t op, const void *x, const void *y, int32_t dtype_in, void *out,
               int32_t dtype_out, int32_t rank, const int64_t *shape, const int64_t *x_strides,
               const int64_t *y_strides, mpc_stream s);
/* out = cond ? x : y (Backend.where), cond bool. */
int mpc_where(mpc_device *dev, const uint8_t *cond, const void *x, const void *y, int32_t dtype, void *out,
              int32_t rank, const int64_t *shape, const int64_t *c_strides, const int64_t *x_strides,
              const int64_t *y_strides, mpc_stream s);
/* Reduction of the middle axis of a contiguous [outer, dim, inner] (Backend.sum / mean / max / min /
 * argmax / argmin, kernels.ts:125-187, :543-568), out [outer, inner]. */
int mpc_reduce(mpc_device *dev, int32_t op, const void *x, int32_t dtype_in, void *out, int32_t dtype_out,
               int64_t outer, int64_t dim, int64_t inner, mpc_stream s);
/* Inclusive prefix sum along the middle axis (Backend.cumsum, kernels.ts:577-592). */
int mpc_cumsum(mpc_device *dev, const void *x, int32_t dtype_in, void *out, int32_t dtype_out, int64_t outer,
               int64_t dim, int64_t inner, mpc_stream s);
/* out[Σ i_k·out_strides_k] = x[Σ i_k·x_strides_k] over shape[rank]: slice, concat, broadcast copies. */
int mpc_strided_copy(mpc_device *dev, const void *x, const int64_t *x_strides, void *out, const int64_t *out_strides,
                     int32_t elem_bytes, int32_t rank, const int64_t *shape, mpc_stream s);
/* Ascending sort of every lane along the middle axis of a contiguous [outer, dim, inner]
 * (Backend.sort -> sortAxis, tensor-cpu/src/index.ts:724-734, kernels.ts:601-617): numeric order,
 * -0 before +0, NaN last; any dtype. */
int mpc_sort(mpc_device *dev, const void *x, int32_t dtype, void *out, int64_t outer, int64_t dim, int64_t inner,
             mpc_stream s);
/* Per-batch row gather (Backend.gatherRows, tensor-cpu/src/index.ts:793-810): x [B, L, D], idx i32
 * [B, M] (a negative index counts from the end) -> out [B, M, D] in x's dtype. An index outside
 * [-L, L) fails with MPC_ERR_INVALID and its flat position in *bad_index (synchronises). */
int mpc_gather_rows(mpc_device *dev, const void *x, int32_t dtype, const int32_t *idx, void *out, int64_t B, int64_t L,
                    int64_t M, int64_t D, int64_t *bad_index, mpc_stream s);
/* Split-half rotary embedding over bh contiguous [L, dh] blocks, positions 0..L-1 (Backend.rope ->
 * ropeHalf, tensor-cpu/src/index.ts:812-819, nn-kernels.ts:138-160); dh even. */
int mpc_rope(mpc_device *dev, const void *x, int32_t dtype, void *out, int64_t bh, int64_t L, int64_t dh, double base,
             mpc_stream s);
/* GEGLU over rows of 2d: out[r, j] = GELU(x[r, j]) * x[r, d + j] (Backend.geglu -> gegluRows,
 * tensor-cpu/src/index.ts:842-850, nn-kernels.ts:245-250). */
int mpc_geglu(mpc_device *dev, const void *x, int32_t dtype, void *out, int64_t rows, int64_t d, mpc_stream s);
/* Masked mean over axis 1: x [B, L, D], mask [B, L] (nonzero = keep; any dtype) -> out [B, D]; a
 * row with nothing kept gives 0 (Backend.meanPool -> maskedMeanPool, tensor-cpu/src/index.ts:852-860,
 * nn-kernels.ts:256-271). */
int mpc_mean_pool(mpc_device *dev, const void *x, int32_t dtype, const void *mask, int32_t mask_dtype, void *out,
                  int64_t B, int64_t L, int64_t D, mpc_stream s);

/* ---- element-wise fusion (WebGpuDevice.fuse / compile, packages/tensor-webgpu/src/facade.ts:137-164,
 * lowering as fusion-wgsl.ts:303-431) ------------------------------------------------------------
 * A traced expression of the tensor-compile IR (packages/tensor-compile/src/ir.ts:66-72) as a DAG
 * of instructions {op, a, b, c}, int32 each: MPC_IR_INPUT (a = input index), MPC_IR_CONST (a =
 * index into consts), a unary op (a = operand), a binary or comparison op (a, b), MPC_IR_SELECT
 * (a = condition, b = then, c = else); operands are indices of EARLIER instructions and the last
 * instruction is the result. Every node evaluates in f64 with the reference's formulas and the
 * result is rounded once to f32. The expression is compiled at run time (NVRTC, sm_100a) into one
 * kernel. */
enum {
  MPC_IR_INPUT = 1, MPC_IR_CONST = 2, MPC_IR_SELECT = 3,
  MPC_IR_NEG = 16, MPC_IR_RELU, MPC_IR_SIGMOID, MPC_IR_GELU, MPC_IR_GELU_TANH, MPC_IR_EXP, MPC_IR_LOG, MPC_IR_SQRT,
  MPC_IR_SIN, MPC_IR_COS, MPC_IR_TAN, MPC_IR_ASIN, MPC_IR_ACOS, MPC_IR_ATAN, MPC_IR_SINH, MPC_IR_COSH, MPC_IR_TANH,
  MPC_IR_COT, MPC_IR_SEC, MPC_IR_CSC, MPC_IR_ASINH, MPC_IR_ACOSH, MPC_IR_ATANH, MPC_IR_COTH, MPC_IR_SECH,
  MPC_IR_CSCH, MPC_IR_ACOT, MPC_IR_ASEC, MPC_IR_ACSC, MPC_IR_ACOTH, MPC_IR_ASECH, MPC_IR_ACSCH, MPC_IR_ABS,
  MPC_IR_LOG10, MPC_IR_LOG2, MPC_IR_CBRT, MPC_IR_FLOOR, MPC_IR_CEIL, MPC_IR_ROUND, MPC_IR_SIGN, MPC_IR_TRUNC,
  MPC_IR_EXPM1, MPC_IR_LOG1P, MPC_IR_ERF,                                                    /* UnaryOp */
  MPC_IR_ADD = 64, MPC_IR_SUB, MPC_IR_MUL, MPC_IR_DIV, MPC_IR_POW, MPC_IR_ATAN2, MPC_IR_HYPOT, MPC_IR_MIN,
  MPC_IR_MAX,                                                                                 /* BinaryOp */
  MPC_IR_LT = 80, MPC_IR_LE, MPC_IR_GT, MPC_IR_GE, MPC_IR_EQ, MPC_IR_NE                      /* CmpOp */
};
/* Compiles `code` (n_instr instructions) over n_inputs inputs of the given dtypes (f32, f16, bf16;
 * at most 16) into *out. The expression is evaluated in f64 (the reference's JavaScript numbers)
 * and rounded once to the f32 output. */
int mpc_fused_create(mpc_device *dev, const int32_t *code, int32_t n_instr, const double *consts, int32_t n_consts,
                     int32_t n_inputs, const int32_t *dtypes, mpc_fused **out);
/* Evaluate in f32 (the WebGPU backend's WGSL arithmetic) instead of f64: every intermediate value
 * is rounded to f32, the math functions are their single-precision versions. */
#define MPC_FUSED_F32 1u
/* mpc_fused_create with MPC_FUSED_* flags. */
int mpc_fused_create_ex(mpc_device *dev, const int32_t *code, int32_t n_instr, const double *consts,
                        int32_t n_consts, int32_t n_inputs, const int32_t *dtypes, uint32_t flags, mpc_fused **out);
/* out (f32, contiguous, `shape`) = the expression over the inputs, each read through element
 * strides aligned to `shape` (0 on broadcast axes): strides[j * rank + k] for input j, axis k. */
int mpc_fused_run(mpc_fused *f, const void *const *inputs, int32_t rank, const int64_t *shape,
                  const int64_t *strides, float *out, mpc_stream s);
int mpc_fused_destroy(mpc_fused *f);
/* The CUDA source a program lowers to under MPC_FUSED_* flags (validation included; no device
 * needed), written to buf (NUL-terminated, truncated to cap) with its full length in *len;
 * check_compile != 0 also compiles it with NVRTC. */
int mpc_fused_lower(const int32_t *code, int32_t n_instr, const double *consts, int32_t n_consts, int32_t n_inputs,
                    const int32_t *dtypes, uint32_t flags, int32_t check_compile, char *buf, size_t cap,
                    size_t *len);

/* ---- multi-GPU: NCCL over NVLink, one rank per process (no reference counterpart) ----------
 * Communicators are created non-blocking and every NCCL call on one is waited for with a deadline,
 * so a rank that never joins (or never reaches a collective) cannot hold the others forever: the
 * call returns MPC_ERR_TIMEOUT instead (the graceful, never-hang contract the reference's native
 * loader keeps, packages/tensor-wasm/src/native.ts:128-139). */
int mpc_comm_unique_id(void *id128);
/* mpc_comm_init_timeout with a 10-minute limit. */
int mpc_comm_init(mpc_device *dev, int nranks, int rank, const void *id128, mpc_comm **comm);
/* Joins rank `rank` of `nranks` to the communicator named by id128. When the group is not complete
 * within timeout_ms (a rank that never calls init), the half-built communicator is aborted and the
 * call returns MPC_ERR_TIMEOUT; later NCCL calls on the communicator use the same limit. */
int mpc_comm_init_timeout(mpc_device *dev, int nranks, int rank, const void *id128, int64_t timeout_ms,
                          mpc_comm **comm);
int mpc_comm_destroy(mpc_comm *comm);
int mpc_comm_abort(mpc_comm *comm);
/* Gathers `bytes` from every rank into recv (rank r's block at offset r*bytes). */
int mpc_allgather(mpc_comm *comm, const void *send, void *recv, size_t bytes, mpc_stream s);

/* ---- peer memory and the GEMM fused with its all-gather (no reference counterpart) ----------
 * A peer buffer is one device allocation per rank of a communicator, every rank's allocation
 * mapped into every process (CUDA IPC over NVLink). Creating and destroying one are collective:
 * every rank calls them, in the same order. mpc_peer_barrier queues a device-side barrier over
 * the group on stream s; a rank that does not arrive within the device's wait timeout makes the
 * next synchronisation return MPC_ERR_TIMEOUT. */
typedef struct mpc_peer_buffer mpc_peer_buffer;
int mpc_peer_buffer_create(mpc_comm *comm, size_t bytes, mpc_peer_buffer **buf);
int mpc_peer_buffer_ptr(mpc_peer_buffer *buf, int rank, void **ptr);
int mpc_peer_barrier(mpc_peer_buffer *buf, mpc_stream s);
int mpc_peer_buffer_destroy(mpc_peer_buffer *buf);
/* The product of desc (f16 / bf16 operands) stored into ndst (1..8) row-major matrices with row
 * pitch ldc elements, at columns col_offset .. col_offset + n - 1 of each. ldc and col_offset in
 * bytes and every destination address must be multiples of 16. */
int mpc_gemm_multi_store(mpc_device *dev, const mpc_gemm_desc *desc, const void *A, const void *B,
                         const float *bias, void *const *dsts, int32_t ndst, int64_t ldc, int64_t col_offset,
                         mpc_stream s);
/* Column-split GEMM with its all-gather in one kernel: rank r of p computes A [m, k] times its
 * column block B_r (desc->n = n columns, one matrix) and the epilogue writes each output block
 * into every rank's C buffer, so that on return (in stream order) every rank's buffer holds the
 * whole C as the shard-major blocked view [p, m, n] (rank r's block contiguous at index r). When
 * rows_out is not null, a permute also writes the row-major C [m, p*n] there (local memory,
 * m*p*n elements of desc->dtype_out). A peer barrier precedes the GEMM (no rank still reads the
 * previous C) and follows it (all blocks have landed). */
int mpc_gemm_allgather(mpc_device *dev, const mpc_gemm_desc *desc, const void *A, const void *B,
                       const float *bias, mpc_peer_buffer *C, void *rows_out, mpc_stream s);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif
#endif
