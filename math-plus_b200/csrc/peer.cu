// Peer memory over NVLink / NVSwitch and the GEMM fused with its all-gather.
//
// A column-split GEMM (rank r of p computes C[:, r*n : (r+1)*n] = A · B_r) needs every rank to end
// up with the whole C. Instead of computing into a local shard and then running an all-gather,
// each rank's GEMM epilogue stores every finished output block straight into every rank's copy of
// C (the shard-major [p, m, n] view) through CUDA IPC mappings of the peers' buffers, so the
// NVLink transfer overlaps the tensor-core work tile by tile. A local permute then gives the
// row-major [m, p*n] where the caller asks for it.
//
// mpc_peer_buffer: one device allocation per rank (the data area plus a small signal area), its
// IPC handle exchanged over the communicator, every peer's allocation opened in this process.
// mpc_peer_barrier: a one-warp kernel. Lane t writes the barrier's epoch into rank t's signal slot
// for this rank (a system-scope release store over NVLink) and then waits, bounded by the device's
// timeout, until rank t's epoch has arrived in this rank's own slot t. A wait that runs out records
// kErrWaitPeer in the device's error word (MPC_ERR_TIMEOUT at the next synchronisation) and
// returns, so a rank that never arrives ends the call with an error instead of a hang.
#include <cuda_runtime.h>

#include <cstring>

#include "mpc_internal.h"
#include "sm100.cuh"

namespace mpc {
namespace {

constexpr int kMaxRanks = 8;
constexpr size_t kSignalBytes = 256;  // kMaxRanks u32 slots, padded

struct BarrierArgs {
  uint32_t *peer_sig[kMaxRanks];  // rank t's signal area as mapped in this process
  uint32_t *my_sig;
  int rank, world;
  uint32_t epoch;
  int *err;
  unsigned long long timeout_ns;
};

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void peer_barrier_kernel(BarrierArgs a) {
  const int t = threadIdx.x;
  if (t >= a.world) return;
  __threadfence_system();  // everything this GPU wrote before the barrier is visible before the signal
  st_release_sys(a.peer_sig[t] + a.rank, a.epoch);
  const uint64_t t0 = globaltimer_ns();
  while (static_cast<int>(ld_acquire_sys(a.my_sig + t) - a.epoch) < 0) {
    if (globaltimer_ns() - t0 > a.timeout_ns) {
      atomicCAS(a.err, 0, kErrWaitPeer);
      return;
    }
    __nanosleep(64);
  }
}

}  // namespace
}  // namespace mpc

struct mpc_peer_buffer {
  mpc_comm *comm;
  mpc_device *dev;
  int rank, world;
  size_t bytes;              // data bytes (the signal area follows at round_up(bytes, 256))
  uint8_t *base[mpc::kMaxRanks];  // each rank's allocation as mapped here (base[rank] is ours)
  uint32_t epoch;
};

using namespace mpc;

static size_t data_span(size_t bytes) { return (bytes + 255) / 256 * 256; }

static int peer_barrier_launch(mpc_peer_buffer *b, cudaStream_t st) {
  BarrierArgs a{};
  for (int r = 0; r < b->world; ++r) a.peer_sig[r] = reinterpret_cast<uint32_t *>(b->base[r] + data_span(b->bytes));
  a.my_sig = a.peer_sig[b->rank];
  a.rank = b->rank;
  a.world = b->world;
  a.epoch = ++b->epoch;
  a.err = b->dev->d_err;
  a.timeout_ns = b->dev->timeout_ns;
  peer_barrier_kernel<<<1, 32, 0, st>>>(a);
  b->dev->launches++;
  return check_launch(b->dev, "peer_barrier_kernel");
}

extern "C" {

int mpc_peer_buffer_create(mpc_comm *comm, size_t bytes, mpc_peer_buffer **out) {
  if (!comm || !out) return fail(MPC_ERR_INVALID, "mpc_peer_buffer_create: null argument");
  *out = nullptr;
  mpc_device *dev = comm->dev;
  int rc = enter(dev);
  if (rc) return rc;
  if (comm->nranks > kMaxRanks)
    return fail(MPC_ERR_UNSUPPORTED, "mpc_peer_buffer_create: %d ranks (at most %d)", comm->nranks, kMaxRanks);
  auto *b = new mpc_peer_buffer{};
  b->comm = comm;
  b->dev = dev;
  b->rank = comm->rank;
  b->world = comm->nranks;
  b->bytes = bytes;
  const size_t total = data_span(bytes) + kSignalBytes;
  void *mine = nullptr;
  cudaError_t e = cudaMalloc(&mine, total);
  if (e != cudaSuccess) {
    delete b;
    return cuda_fail(dev, e, "mpc_peer_buffer_create: cudaMalloc");
  }
  b->base[b->rank] = static_cast<uint8_t *>(mine);
  void *xchg = nullptr;
  auto undo = [&](int status) {
    for (int r = 0; r < b->world; ++r)
      if (r != b->rank && b->base[r]) cudaIpcCloseMemHandle(b->base[r]);
    if (xchg) cudaFree(xchg);
    cudaFree(mine);
    delete b;
    return status;
  };
  cudaIpcMemHandle_t h;
  if ((e = cudaMemset(static_cast<uint8_t *>(mine) + data_span(bytes), 0, kSignalBytes)) != cudaSuccess ||
      (e = cudaIpcGetMemHandle(&h, mine)) != cudaSuccess ||
      (e = cudaMalloc(&xchg, sizeof(h) * (b->world + 1))) != cudaSuccess ||
      (e = cudaMemcpy(xchg, &h, sizeof(h), cudaMemcpyHostToDevice)) != cudaSuccess)
    return undo(cuda_fail(dev, e, "mpc_peer_buffer_create: IPC handle"));
  uint8_t *gathered = static_cast<uint8_t *>(xchg) + sizeof(h);
  if ((rc = mpc_allgather(comm, xchg, gathered, sizeof(h), dev->stream))) return undo(rc);
  cudaIpcMemHandle_t all[kMaxRanks];
  if ((e = cudaStreamSynchronize(dev->stream)) != cudaSuccess ||
      (e = cudaMemcpy(all, gathered, sizeof(h) * b->world, cudaMemcpyDeviceToHost)) != cudaSuccess)
    return undo(cuda_fail(dev, e, "mpc_peer_buffer_create: handle exchange"));
  for (int r = 0; r < b->world; ++r) {
    if (r == b->rank) continue;
    void *p = nullptr;
    if ((e = cudaIpcOpenMemHandle(&p, all[r], cudaIpcMemLazyEnablePeerAccess)) != cudaSuccess)
      return undo(cuda_fail(dev, e, "mpc_peer_buffer_create: cudaIpcOpenMemHandle"));
    b->base[r] = static_cast<uint8_t *>(p);
  }
  cudaFree(xchg);
  *out = b;
  return MPC_OK;
}

int mpc_peer_buffer_ptr(mpc_peer_buffer *b, int rank, void **ptr) {
  if (!b || !ptr) return fail(MPC_ERR_INVALID, "mpc_peer_buffer_ptr: null argument");
  if (rank < 0 || rank >= b->world) return fail(MPC_ERR_INVALID, "mpc_peer_buffer_ptr: rank %d of %d", rank, b->world);
  *ptr = b->base[rank];
  return MPC_OK;
}

int mpc_peer_barrier(mpc_peer_buffer *b, mpc_stream s) {
  if (!b) return fail(MPC_ERR_INVALID, "mpc_peer_barrier: null buffer");
  int rc = enter(b->dev);
  if (rc) return rc;
  return peer_barrier_launch(b, stream_of(b->dev, s));
}

int mpc_peer_buffer_destroy(mpc_peer_buffer *b) {
  if (!b) return MPC_OK;
  int rc = enter(b->dev);
  if (rc) return rc;
  // No rank may still write into an allocation that its owner frees, and no rank frees its
  // allocation while another still maps it: a device barrier (all peer stores have landed), unmap
  // the peers, then a barrier that touches only local memory (an NCCL all-gather of one byte per
  // rank inside this rank's own signal area; the peer mappings are gone by then), then free.
  cudaStream_t st = b->dev->stream;
  int status = peer_barrier_launch(b, st);
  cudaError_t e = cudaStreamSynchronize(st);
  for (int r = 0; r < b->world; ++r)
    if (r != b->rank && b->base[r]) cudaIpcCloseMemHandle(b->base[r]);
  uint8_t *sig = b->base[b->rank] + data_span(b->bytes);
  const int ag = mpc_allgather(b->comm, sig + 64, sig + 128, 1, st);
  if (!status) status = ag;
  const cudaError_t e2 = cudaStreamSynchronize(st);
  if (e == cudaSuccess) e = e2;
  cudaFree(b->base[b->rank]);
  delete b;
  if (status) return status;
  return e == cudaSuccess ? MPC_OK : cuda_fail(nullptr, e, "mpc_peer_buffer_destroy");
}

int mpc_gemm_multi_store(mpc_device *dev, const mpc_gemm_desc *desc, const void *A, const void *B, const float *bias,
                         void *const *dsts, int32_t ndst, int64_t ldc, int64_t col_offset, mpc_stream s) {
  int rc = enter(dev);
  if (rc) return rc;
  if (!desc) return fail(MPC_ERR_INVALID, "mpc_gemm_multi_store: null descriptor");
  return gemm_run_multi(dev, desc, A, B, bias, dsts, ndst, ldc, col_offset, stream_of(dev, s));
}

int mpc_gemm_allgather(mpc_device *dev, const mpc_gemm_desc *desc, const void *A, const void *B, const float *bias,
                       mpc_peer_buffer *C, void *rows_out, mpc_stream s) {
  int rc = enter(dev);
  if (rc) return rc;
  if (!desc || !C) return fail(MPC_ERR_INVALID, "mpc_gemm_allgather: null argument");
  if (C->dev != dev) return fail(MPC_ERR_INVALID, "mpc_gemm_allgather: the buffer belongs to another device");
  if (desc->batch_rank != 0) return fail(MPC_ERR_INVALID, "mpc_gemm_allgather: one matrix (batch_rank 0)");
  const size_t eo = dtype_size(desc->dtype_out);
  const size_t block = (size_t)(desc->m * desc->n) * eo;
  if (block * C->world > C->bytes)
    return fail(MPC_ERR_INVALID, "mpc_gemm_allgather: C needs %zu bytes, the buffer has %zu", block * C->world,
                C->bytes);
  cudaStream_t st = stream_of(dev, s);
  // Every rank's buffer is the shard-major [p, m, n]: this rank's block is the contiguous [m, n]
  // at index rank in each of them. (Storing straight into a row-major [m, p*n] instead spreads
  // every 128-row tile over 128 rows of p*n columns in p buffers at once; with 8 ranks that
  // many distinct pages per tile made the peer stores an order of magnitude slower.)
  void *dsts[kMaxRanks];
  for (int i = 0; i < C->world; ++i) dsts[i] = C->base[(C->rank + 1 + i) % C->world] + block * C->rank;  // own last
  if ((rc = peer_barrier_launch(C, st))) return rc;  // every rank is done with the previous contents
  if ((rc = gemm_run_multi(dev, desc, A, B, bias, dsts, C->world, desc->n, 0, st))) return rc;
  if ((rc = peer_barrier_launch(C, st))) return rc;  // every rank's blocks have landed everywhere
  if (!rows_out) return MPC_OK;
  const int64_t shape[3] = {C->world, desc->m, desc->n};
  const int32_t perm[3] = {1, 0, 2};  // [p, m, n] -> [m, p, n] = row-major [m, p*n]
  return mpc_transpose(dev, C->base[C->rank], rows_out, (int32_t)eo, 3, shape, perm, s);
}

}  // extern "C"
