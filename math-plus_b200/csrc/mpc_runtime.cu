// Device lifecycle, errors, the caching allocator, copies, streams and events of
// libmathplus_cuda.so. Every exported call returns an mpc_status and never aborts (the
// "defined failure, not panic" rule of crates/tensor-wasm-kernels/src/lib.rs:17-38); a CUDA
// error that corrupts the context poisons the handle for good, like tensor-wasm's trap
// poisoning (packages/tensor-wasm/src/index.ts:291-340).
#include <cstdio>
#include <cstring>

#include "mpc_internal.h"
#include "sm100.cuh"

namespace mpc {

static thread_local char g_last_error[1024] = "";

void set_error(const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int fail(int status, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

static bool is_sticky(cudaError_t e) {
  switch (e) {
    case cudaErrorIllegalAddress:
    case cudaErrorLaunchFailure:
    case cudaErrorIllegalInstruction:
    case cudaErrorMisalignedAddress:
    case cudaErrorInvalidAddressSpace:
    case cudaErrorInvalidPc:
    case cudaErrorHardwareStackError:
    case cudaErrorAssert:
    case cudaErrorLaunchTimeout:
    case cudaErrorECCUncorrectable:
      return true;
    default:
      return false;
  }
}

int cuda_fail(mpc_device *dev, cudaError_t e, const char *what) {
  if (e == cudaErrorMemoryAllocation) {
    cudaGetLastError();
    return fail(MPC_ERR_OOM, "%s: %s", what, cudaGetErrorString(e));
  }
  if (dev && is_sticky(e)) dev->sticky = MPC_ERR_POISONED;
  return fail(MPC_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

int enter(mpc_device *dev) {
  if (!dev) return fail(MPC_ERR_INVALID, "null device handle");
  if (dev->sticky == MPC_ERR_POISONED)
    return fail(MPC_ERR_POISONED, "device %d is poisoned by an earlier fault; destroy it", dev->ordinal);
  cudaError_t e = cudaSetDevice(dev->ordinal);
  if (e != cudaSuccess) return cuda_fail(dev, e, "cudaSetDevice");
  return MPC_OK;
}

cudaStream_t stream_of(mpc_device *dev, mpc_stream s) { return s ? static_cast<cudaStream_t>(s) : dev->stream; }

int check_launch(mpc_device *dev, const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(dev, e, what);
  return MPC_OK;
}

int free_on(mpc_device *dev, void *ptr, cudaStream_t st) {
  if (!ptr) return MPC_OK;
  mpc_allocator &a = dev->alloc;
  std::lock_guard<std::mutex> lk(a.mu);
  auto it = a.live.find(ptr);
  if (it == a.live.end()) return fail(MPC_ERR_INVALID, "mpc_free: %p was not allocated by this device", ptr);
  const size_t bytes = it->second;
  a.live.erase(it);
  a.in_use -= bytes;
  cudaEvent_t ev = nullptr;
  cudaStream_t on = st ? st : dev->stream;
  if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) == cudaSuccess) cudaEventRecord(ev, on);
  a.free_blocks.emplace(bytes, mpc_free_block{ptr, ev, on});
  a.cached += bytes;
  return MPC_OK;
}

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int make_map_3d(CUtensorMap *map, CUtensorMapDataType dt, const void *base, uint64_t d0, uint64_t d1, uint64_t d2,
                uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0, uint32_t box1, CUtensorMapSwizzle swz) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return fail(MPC_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if (d2 == 1) stride2_bytes = d1 * stride1_bytes;  // any valid stride: the third coordinate is always 0
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {box0, box1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, dt, 3, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(MPC_ERR_INVALID,
                "cuTensorMapEncodeTiled failed (%d): base %p dims {%llu,%llu,%llu} strides {%llu,%llu} box {%u,%u}",
                (int)r, base, (unsigned long long)d0, (unsigned long long)d1, (unsigned long long)d2,
                (unsigned long long)stride1_bytes, (unsigned long long)stride2_bytes, box0, box1);
  return MPC_OK;
}

int make_map_4d(CUtensorMap *map, CUtensorMapDataType dt, const void *base, const uint64_t dims[4],
                const uint64_t strides_bytes[3], const uint32_t box_dims[4], CUtensorMapSwizzle swz) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return fail(MPC_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t d[4] = {dims[0], dims[1], dims[2], dims[3]};
  cuuint64_t st[3] = {strides_bytes[0], strides_bytes[1], strides_bytes[2]};
  cuuint32_t box[4] = {box_dims[0], box_dims[1], box_dims[2], box_dims[3]};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, dt, 4, const_cast<void *>(base), d, st, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(MPC_ERR_INVALID,
                "cuTensorMapEncodeTiled failed (%d): base %p dims {%llu,%llu,%llu,%llu} strides {%llu,%llu,%llu}",
                (int)r, base, (unsigned long long)d[0], (unsigned long long)d[1], (unsigned long long)d[2],
                (unsigned long long)d[3], (unsigned long long)st[0], (unsigned long long)st[1],
                (unsigned long long)st[2]);
  return MPC_OK;
}

// A single thread waits on an mbarrier that nothing ever arrives on. Its bounded wait runs out,
// records kErrWaitProbe in the device error word and returns: the failure path every pipeline
// wait of the GEMM and attention kernels takes, exercised without any fault.
__global__ void wait_probe_kernel(int *err, unsigned long long timeout_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(&bar, 0, &abort_flag, err, kErrWaitProbe, timeout_ns);
}

int wait_probe_run(mpc_device *dev, uint64_t timeout_ns, cudaStream_t st) {
  wait_probe_kernel<<<1, 32, 0, st>>>(dev->d_err, timeout_ns);
  dev->launches++;
  return check_launch(dev, "wait_probe_kernel");
}

// Size classes: 512-byte steps up to 1 MiB, then 2 MiB steps.
static size_t round_alloc(size_t bytes) {
  if (bytes <= 512) return 512;
  if (bytes <= (1u << 20)) return (bytes + 511) & ~size_t(511);
  return (bytes + (2u << 20) - 1) & ~size_t((2u << 20) - 1);
}

int alloc_on(mpc_device *dev, size_t bytes, cudaStream_t st, void **ptr) {
  *ptr = nullptr;
  const size_t sz = round_alloc(bytes);
  mpc_allocator &a = dev->alloc;
  std::lock_guard<std::mutex> lk(a.mu);
  if (a.limit && a.in_use + sz > a.limit)
    return fail(MPC_ERR_OOM, "mpc_alloc: %zu bytes would exceed the allocator cap (%zu in use of %zu)", sz, a.in_use,
                a.limit);
  auto range = a.free_blocks.equal_range(sz);
  for (auto it = range.first; it != range.second; ++it) {
    const mpc_free_block fb = it->second;
    if (fb.stream != st && fb.ev && cudaEventQuery(fb.ev) != cudaSuccess) continue;  // another stream may still use it
    cudaGetLastError();
    if (fb.ev) cudaEventDestroy(fb.ev);
    a.free_blocks.erase(it);
    a.cached -= sz;
    a.live[fb.ptr] = sz;
    a.in_use += sz;
    *ptr = fb.ptr;
    return MPC_OK;
  }
  void *p = nullptr;
  cudaError_t e = cudaMalloc(&p, sz);
  if (e == cudaErrorMemoryAllocation && !a.free_blocks.empty()) {
    // Release the cache (after the device drains) and retry once.
    cudaGetLastError();
    cudaDeviceSynchronize();
    for (auto &kv : a.free_blocks) {
      if (kv.second.ev) cudaEventDestroy(kv.second.ev);
      cudaFree(kv.second.ptr);
    }
    a.free_blocks.clear();
    a.cached = 0;
    e = cudaMalloc(&p, sz);
  }
  if (e != cudaSuccess) return cuda_fail(dev, e, "cudaMalloc");
  a.live[p] = sz;
  a.in_use += sz;
  *ptr = p;
  return MPC_OK;
}

}  // namespace mpc

using namespace mpc;

extern "C" {

int mpc_version(void) { return MPC_ABI_VERSION; }

const char *mpc_last_error(mpc_device *) { return g_last_error; }

int mpc_device_count(int *count) {
  if (!count) return fail(MPC_ERR_INVALID, "mpc_device_count: null out pointer");
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) {
    cudaGetLastError();
    *count = 0;
    return MPC_OK;
  }
  if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaGetDeviceCount");
  *count = n;
  return MPC_OK;
}

int mpc_device_create(int ordinal, unsigned flags, mpc_device **out) {
  (void)flags;
  if (!out) return fail(MPC_ERR_INVALID, "mpc_device_create: null out pointer");
  *out = nullptr;
  int n = 0;
  int rc = mpc_device_count(&n);
  if (rc) return rc;
  if (n == 0) return fail(MPC_ERR_NO_DEVICE, "no CUDA device is visible");
  if (ordinal < 0 || ordinal >= n) return fail(MPC_ERR_INVALID, "device ordinal %d out of range [0, %d)", ordinal, n);
  mpc_device *dev = new mpc_device();
  dev->ordinal = ordinal;
  cudaError_t e;
  if ((e = cudaSetDevice(ordinal)) != cudaSuccess || (e = cudaGetDeviceProperties(&dev->prop, ordinal)) != cudaSuccess) {
    rc = cuda_fail(nullptr, e, "mpc_device_create");
    delete dev;
    return rc;
  }
  if (dev->prop.major != 10) {
    rc = fail(MPC_ERR_NO_DEVICE, "device %d is compute capability %d.%d; this library is built for sm_100a (B200)",
              ordinal, dev->prop.major, dev->prop.minor);
    delete dev;
    return rc;
  }
  if ((e = cudaStreamCreateWithFlags(&dev->stream, cudaStreamNonBlocking)) != cudaSuccess ||
      (e = cudaMalloc(&dev->d_err, 256)) != cudaSuccess || (e = cudaMemset(dev->d_err, 0, 256)) != cudaSuccess) {
    rc = cuda_fail(nullptr, e, "mpc_device_create");
    if (dev->stream) cudaStreamDestroy(dev->stream);
    delete dev;
    return rc;
  }
  *out = dev;
  return MPC_OK;
}

int mpc_device_destroy(mpc_device *dev) {
  if (!dev) return MPC_OK;
  cudaSetDevice(dev->ordinal);
  if (dev->sticky != MPC_ERR_POISONED) cudaStreamSynchronize(dev->stream);
  {
    std::lock_guard<std::mutex> lk(dev->alloc.mu);
    for (auto &kv : dev->alloc.free_blocks) {
      if (kv.second.ev) cudaEventDestroy(kv.second.ev);
      cudaFree(kv.second.ptr);
    }
    for (auto &kv : dev->alloc.live) cudaFree(kv.first);
  }
  if (dev->d_err) cudaFree(dev->d_err);
  if (dev->stream) cudaStreamDestroy(dev->stream);
  delete dev;
  return MPC_OK;
}

int mpc_device_info(mpc_device *dev, mpc_device_info_t *info) {
  if (!dev || !info) return fail(MPC_ERR_INVALID, "mpc_device_info: null argument");
  memset(info, 0, sizeof(*info));
  snprintf(info->name, sizeof(info->name), "%s", dev->prop.name);
  info->ordinal = dev->ordinal;
  info->cc_major = dev->prop.major;
  info->cc_minor = dev->prop.minor;
  info->sm_count = dev->prop.multiProcessorCount;
  info->total_bytes = dev->prop.totalGlobalMem;
  info->smem_per_block_optin = dev->prop.sharedMemPerBlockOptin;
  cudaRuntimeGetVersion(&info->runtime_version);
  cudaDriverGetVersion(&info->driver_version);
  return MPC_OK;
}

int mpc_gemm_capabilities(mpc_device *dev, mpc_gemm_caps *caps) {
  if (!dev || !caps) return fail(MPC_ERR_INVALID, "mpc_gemm_capabilities: null argument");
  return gemm_capabilities(dev, caps);
}

int mpc_device_status(mpc_device *dev) {
  if (!dev) return fail(MPC_ERR_INVALID, "null device handle");
  return dev->sticky;
}

int mpc_set_wait_timeout_ns(mpc_device *dev, uint64_t ns) {
  if (!dev) return fail(MPC_ERR_INVALID, "null device handle");
  dev->timeout_ns = ns ? ns : 2000000000ull;
  return MPC_OK;
}

// ---- allocator ------------------------------------------------------------------------------
int mpc_alloc(mpc_device *dev, size_t bytes, void **ptr) {
  int rc = enter(dev);
  if (rc) return rc;
  if (!ptr) return fail(MPC_ERR_INVALID, "mpc_alloc: null out pointer");
  *ptr = nullptr;
  return alloc_on(dev, bytes, dev->stream, ptr);
}

int mpc_free(mpc_device *dev, void *ptr) {
  if (!dev) return fail(MPC_ERR_INVALID, "null device handle");
  if (!ptr) return MPC_OK;
  cudaSetDevice(dev->ordinal);
  return free_on(dev, ptr, dev->stream);
}

int mpc_set_alloc_limit(mpc_device *dev, size_t bytes) {
  if (!dev) return fail(MPC_ERR_INVALID, "null device handle");
  std::lock_guard<std::mutex> lk(dev->alloc.mu);
  dev->alloc.limit = bytes;
  return MPC_OK;
}

int mpc_alloc_stats(mpc_device *dev, size_t *in_use, size_t *cached) {
  if (!dev) return fail(MPC_ERR_INVALID, "null device handle");
  std::lock_guard<std::mutex> lk(dev->alloc.mu);
  if (in_use) *in_use = dev->alloc.in_use;
  if (cached) *cached = dev->alloc.cached;
  return MPC_OK;
}

int mpc_trim(mpc_device *dev) {
  int rc = enter(dev);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(dev->alloc.mu);
  for (auto it = dev->alloc.free_blocks.begin(); it != dev->alloc.free_blocks.end();) {
    cudaEvent_t ev = it->second.ev;
    if (ev) cudaEventSynchronize(ev);
    if (ev) cudaEventDestroy(ev);
    cudaFree(it->second.ptr);
    dev->alloc.cached -= it->first;
    it = dev->alloc.free_blocks.erase(it);
  }
  return MPC_OK;
}

int mpc_host_alloc(mpc_device *dev, size_t bytes, void **ptr) {
  int rc = enter(dev);
  if (rc) return rc;
  if (!ptr) return fail(MPC_ERR_INVALID, "mpc_host_alloc: null out pointer");
  MPC_CUDA(dev, cudaHostAlloc(ptr, bytes ? bytes : 1, cudaHostAllocPortable));
  return MPC_OK;
}

int mpc_host_free(mpc_device *dev, void *ptr) {
  if (!ptr) return MPC_OK;
  int rc = enter(dev);
  if (rc) return rc;
  MPC_CUDA(dev, cudaFreeHost(ptr));
  return MPC_OK;
}

// ---- copies ---------------------------------------------------------------------------------
static int copy_async(mpc_device *dev, void *dst, const void *src, size_t bytes, mpc_stream s, cudaMemcpyKind kind,
                      const char *what) {
  int rc = enter(dev);
  if (rc) return rc;
  if (!bytes) return MPC_OK;
  if (!dst || !src) return fail(MPC_ERR_INVALID, "%s: null pointer", what);
  MPC_CUDA(dev, cudaMemcpyAsync(dst, src, bytes, kind, stream_of(dev, s)));
  return MPC_OK;
}

int mpc_memcpy_h2d_async(mpc_device *dev, void *dst, const void *src, size_t bytes, mpc_stream s) {
  return copy_async(dev, dst, src, bytes, s, cudaMemcpyHostToDevice, "mpc_memcpy_h2d_async");
}
int mpc_memcpy_d2h_async(mpc_device *dev, void *dst, const void *src, size_t bytes, mpc_stream s) {
  return copy_async(dev, dst, src, bytes, s, cudaMemcpyDeviceToHost, "mpc_memcpy_d2h_async");
}
int mpc_memcpy_d2d_async(mpc_device *dev, void *dst, const void *src, size_t bytes, mpc_stream s) {
  return copy_async(dev, dst, src, bytes, s, cudaMemcpyDeviceToDevice, "mpc_memcpy_d2d_async");
}
int mpc_memset_async(mpc_device *dev, void *dst, int value, size_t bytes, mpc_stream s) {
  int rc = enter(dev);
  if (rc) return rc;
  if (!bytes) return MPC_OK;
  if (!dst) return fail(MPC_ERR_INVALID, "mpc_memset_async: null pointer");
  MPC_CUDA(dev, cudaMemsetAsync(dst, value, bytes, stream_of(dev, s)));
  return MPC_OK;
}

// ---- streams, events, sync ------------------------------------------------------------------
int mpc_stream_create(mpc_device *dev, mpc_stream *s) {
  int rc = enter(dev);
  if (rc) return rc;
  if (!s) return fail(MPC_ERR_INVALID, "mpc_stream_create: null out pointer");
  cudaStream_t st;
  MPC_CUDA(dev, cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  *s = st;
  return MPC_OK;
}
int mpc_stream_destroy(mpc_device *dev, mpc_stream s) {
  int rc = enter(dev);
  if (rc) return rc;
  if (s) MPC_CUDA(dev, cudaStreamDestroy(static_cast<cudaStream_t>(s)));
  return MPC_OK;
}
int mpc_device_stream(mpc_device *dev, mpc_stream *s) {
  if (!dev || !s) return fail(MPC_ERR_INVALID, "mpc_device_stream: null argument");
  *s = dev->stream;
  return MPC_OK;
}

static int read_error_word(mpc_device *dev) {
  int word = 0;
  cudaError_t e = cudaMemcpy(&word, dev->d_err, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(dev, e, "reading the kernel error word");
  if (word) {
    dev->sticky = MPC_ERR_TIMEOUT;
    return fail(MPC_ERR_TIMEOUT, "a kernel's bounded wait ran out (site 0x%x); its results are invalid", word);
  }
  return MPC_OK;
}

int mpc_stream_sync(mpc_device *dev, mpc_stream s) {
  int rc = enter(dev);
  if (rc) return rc;
  MPC_CUDA(dev, cudaStreamSynchronize(stream_of(dev, s)));
  return read_error_word(dev);
}

int mpc_sync(mpc_device *dev) {
  int rc = enter(dev);
  if (rc) return rc;
  MPC_CUDA(dev, cudaDeviceSynchronize());
  return read_error_word(dev);
}

int mpc_event_create(mpc_device *dev, mpc_event *e) {
  int rc = enter(dev);
  if (rc) return rc;
  if (!e) return fail(MPC_ERR_INVALID, "mpc_event_create: null out pointer");
  cudaEvent_t ev;
  MPC_CUDA(dev, cudaEventCreate(&ev));
  *e = ev;
  return MPC_OK;
}
int mpc_event_destroy(mpc_device *dev, mpc_event e) {
  int rc = enter(dev);
  if (rc) return rc;
  if (e) MPC_CUDA(dev, cudaEventDestroy(static_cast<cudaEvent_t>(e)));
  return MPC_OK;
}
int mpc_event_record(mpc_device *dev, mpc_event e, mpc_stream s) {
  int rc = enter(dev);
  if (rc) return rc;
  MPC_CUDA(dev, cudaEventRecord(static_cast<cudaEvent_t>(e), stream_of(dev, s)));
  return MPC_OK;
}
int mpc_stream_wait_event(mpc_device *dev, mpc_stream s, mpc_event e) {
  int rc = enter(dev);
  if (rc) return rc;
  if (!e) return fail(MPC_ERR_INVALID, "mpc_stream_wait_event: null event");
  MPC_CUDA(dev, cudaStreamWaitEvent(stream_of(dev, s), static_cast<cudaEvent_t>(e), 0));
  return MPC_OK;
}
int mpc_event_elapsed_ms(mpc_device *dev, mpc_event a, mpc_event b, float *ms) {
  int rc = enter(dev);
  if (rc) return rc;
  if (!ms) return fail(MPC_ERR_INVALID, "mpc_event_elapsed_ms: null out pointer");
  MPC_CUDA(dev, cudaEventSynchronize(static_cast<cudaEvent_t>(b)));
  MPC_CUDA(dev, cudaEventElapsedTime(ms, static_cast<cudaEvent_t>(a), static_cast<cudaEvent_t>(b)));
  return MPC_OK;
}

int mpc_launch_count(mpc_device *dev, uint64_t *count) {
  if (!dev || !count) return fail(MPC_ERR_INVALID, "mpc_launch_count: null argument");
  *count = dev->launches.load();
  return MPC_OK;
}

// Clears a recorded kernel timeout (after the caller has handled it) so the handle can be reused.
int mpc_device_clear_error(mpc_device *dev) {
  if (!dev) return fail(MPC_ERR_INVALID, "null device handle");
  if (dev->sticky == MPC_ERR_POISONED) return fail(MPC_ERR_POISONED, "a poisoned device cannot be cleared");
  int rc = enter(dev);
  if (rc) return rc;
  MPC_CUDA(dev, cudaDeviceSynchronize());
  MPC_CUDA(dev, cudaMemset(dev->d_err, 0, 256));
  dev->sticky = MPC_OK;
  return MPC_OK;
}

int mpc_selftest_wait_timeout(mpc_device *dev, uint64_t timeout_ns) {
  int rc = enter(dev);
  if (rc) return rc;
  if (timeout_ns == 0 || timeout_ns > 10000000000ull)
    return fail(MPC_ERR_INVALID, "mpc_selftest_wait_timeout: timeout must be in (0, 10 s]");
  if ((rc = wait_probe_run(dev, timeout_ns, dev->stream))) return rc;
  return mpc_stream_sync(dev, nullptr);
}

// ---- the hot-path entry points --------------------------------------------------------------
int mpc_gemm(mpc_device *dev, const mpc_gemm_desc *desc, const void *A, const void *B, void *C, const float *bias,
             mpc_stream s) {
  int rc = enter(dev);
  if (rc) return rc;
  if (!desc) return fail(MPC_ERR_INVALID, "mpc_gemm: null descriptor");
  if (desc->epilogue & MPC_EPI_RESIDUAL)
    return fail(MPC_ERR_INVALID, "mpc_gemm: the RESIDUAL epilogue needs mpc_gemm_residual");
  return gemm_run(dev, desc, A, B, C, bias, nullptr, stream_of(dev, s));
}

int mpc_gemm_residual(mpc_device *dev, const mpc_gemm_desc *desc, const void *A, const void *B, void *C,
                      const float *bias, const void *R, mpc_stream s) {
  int rc = enter(dev);
  if (rc) return rc;
  if (!desc) return fail(MPC_ERR_INVALID, "mpc_gemm_residual: null descriptor");
  return gemm_run(dev, desc, A, B, C, bias, R, stream_of(dev, s));
}

int mpc_sdpa(mpc_device *dev, const mpc_sdpa_desc *desc, const void *Q, const void *K, const void *V,
             const void *mask, void *O, float *LSE, mpc_stream s) {
  int rc = enter(dev);
  if (rc) return rc;
  if (!desc) return fail(MPC_ERR_INVALID, "mpc_sdpa: null descriptor");
  return sdpa_run(dev, desc, Q, K, V, mask, O, LSE, nullptr, stream_of(dev, s));
}

int mpc_sdpa_strided(mpc_device *dev, const mpc_sdpa_desc *desc, const void *Q, const void *K, const void *V,
                     const void *mask, void *O, float *LSE, const mpc_sdpa_layout *layout, mpc_stream s) {
  int rc = enter(dev);
  if (rc) return rc;
  if (!desc || !layout) return fail(MPC_ERR_INVALID, "mpc_sdpa_strided: null descriptor or layout");
  return sdpa_run(dev, desc, Q, K, V, mask, O, LSE, layout, stream_of(dev, s));
}

}  // extern "C"
