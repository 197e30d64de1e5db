// Internal declarations shared by the library's translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdint>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/mathplus_cuda.h"

struct mpc_block {
  void *ptr;
  size_t bytes;
};

// A cached block: freed on `stream`, where `ev` was recorded at the time of the free.
struct mpc_free_block {
  void *ptr;
  cudaEvent_t ev;
  cudaStream_t stream;
};

// Caching device allocator: freed blocks are kept per rounded size and handed out again,
// stream-ordered: a block freed on stream S is handed at once to a request for use on S (work
// queued on S after the free runs after every earlier use), and to a request for another stream
// only once the event recorded at the free has completed.
struct mpc_allocator {
  std::mutex mu;
  std::unordered_multimap<size_t, mpc_free_block> free_blocks;
  std::unordered_map<void *, size_t> live;
  size_t in_use = 0, cached = 0, limit = 0;
};

struct mpc_device {
  int ordinal = -1;
  cudaStream_t stream = nullptr;
  int *d_err = nullptr;  // kernel error word (device memory)
  std::atomic<int> sticky{0};
  uint64_t timeout_ns = 2000000000ull;
  std::atomic<uint64_t> launches{0};
  cudaDeviceProp prop{};
  mpc_allocator alloc;
};

// One rank of an NCCL communicator (comm.cu).
struct mpc_comm {
  mpc_device *dev;
  void *comm;  // ncclComm_t (non-blocking)
  int nranks, rank;
  int64_t timeout_ms;  // limit for each NCCL call on it to settle
};

namespace mpc {

// Thread-local last-error text and the helpers that fill it.
void set_error(const char *fmt, ...);
int fail(int status, const char *fmt, ...);
int cuda_fail(mpc_device *dev, cudaError_t e, const char *what);

#define MPC_CUDA(dev, call)                                   \
  do {                                                        \
    cudaError_t e_ = (call);                                  \
    if (e_ != cudaSuccess) return mpc::cuda_fail(dev, e_, #call); \
  } while (0)

// Validates a device handle and makes its ordinal current.
int enter(mpc_device *dev);
cudaStream_t stream_of(mpc_device *dev, mpc_stream s);
int check_launch(mpc_device *dev, const char *what);

// Returns a block to the device cache once the work queued on `st` so far has finished.
int free_on(mpc_device *dev, void *ptr, cudaStream_t st);
// A block for work queued on `st` (stream-ordered reuse, see mpc_allocator).
int alloc_on(mpc_device *dev, size_t bytes, cudaStream_t st, void **ptr);

// Scratch memory from the device allocator for the kernels queued on one stream; the block is
// handed back on scope exit, ordered after that stream's pending work.
struct Scratch {
  mpc_device *dev = nullptr;
  cudaStream_t st = nullptr;
  void *ptr = nullptr;
  Scratch() = default;
  Scratch(const Scratch &) = delete;
  Scratch &operator=(const Scratch &) = delete;
  ~Scratch() {
    if (ptr) free_on(dev, ptr, st);
  }
  int get(mpc_device *d, cudaStream_t s, size_t bytes) {
    dev = d;
    st = s;
    return alloc_on(d, bytes ? bytes : 256, s, &ptr);
  }
};

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled();
// Builds a 3-D tiled map over a row-major [d2][d1][d0] tensor (d0 contiguous). Strides in bytes.
int make_map_3d(CUtensorMap *map, CUtensorMapDataType dt, const void *base, uint64_t d0, uint64_t d1, uint64_t d2,
                uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0, uint32_t box1, CUtensorMapSwizzle swz);
// A 4-D tiled map over [d3][d2][d1][d0] (d0 contiguous) with byte strides of axes 1..3.
int make_map_4d(CUtensorMap *map, CUtensorMapDataType dt, const void *base, const uint64_t dims[4],
                const uint64_t strides_bytes[3], const uint32_t box[4], CUtensorMapSwizzle swz);

inline size_t dtype_size(int dt) {
  switch (dt) {
    case MPC_F32:
    case MPC_I32:
      return 4;
    case MPC_F16:
    case MPC_BF16:
      return 2;
    case MPC_BOOL:
      return 1;
    default:
      return 0;
  }
}

// Kernel entry points implemented in other translation units.
int gemm_run(mpc_device *dev, const mpc_gemm_desc *d, const void *A, const void *B, void *C, const float *bias,
             const void *resid, cudaStream_t st);
int sdpa_run(mpc_device *dev, const mpc_sdpa_desc *d, const void *Q, const void *K, const void *V, const void *mask,
             void *O, float *LSE, const mpc_sdpa_layout *layout, cudaStream_t st);
int wait_probe_run(mpc_device *dev, uint64_t timeout_ns, cudaStream_t st);
int gemm_capabilities(mpc_device *dev, mpc_gemm_caps *caps);
// The product stored into `ndst` row-major matrices (pitch ldc, columns col_offset..+N-1).
int gemm_run_multi(mpc_device *dev, const mpc_gemm_desc *d, const void *A, const void *B, const float *bias,
                   void *const *dsts, int ndst, int64_t ldc, int64_t col_offset, cudaStream_t st);

}  // namespace mpc
