// NCCL over NVLink / NVSwitch, one rank per process: the one exchange step of the path (the
// all-gather that reassembles a GEMM split over N across GPUs). NCCL is resolved at run time
// with dlopen("libnccl.so.2"), so a process that already loaded NCCL (torch.distributed) shares
// that copy instead of loading a second one.
#include <dlfcn.h>

#include <chrono>
#include <climits>
#include <cstring>
#include <thread>

#include "mpc_internal.h"

namespace mpc {
namespace {

typedef int ncclResult_t;
typedef void *ncclComm_t;
struct ncclUniqueId {
  char internal[128];
};
enum { ncclInt8 = 0, ncclInProgress = 7 };

// NCCL's ncclConfig_t as its 2.18 header lays it out (later versions append fields; the library
// reads `size` and `version` to know which fields the caller's struct has, and gives the rest their
// defaults). Only `blocking` is set here; every other field keeps NCCL's "undefined" marker, so NCCL
// chooses it as it does for ncclCommInitRank.
struct NcclConfig {
  size_t size = sizeof(NcclConfig);
  unsigned int magic = 0xcafebeefu;
  unsigned int version = 21800;  // NCCL_VERSION(2, 18, 0): the layout below
  int blocking = 0;
  int cgaClusterSize = INT_MIN;
  int minCTAs = INT_MIN;
  int maxCTAs = INT_MIN;
  const char *netName = nullptr;
  int splitShare = INT_MIN;
};

struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int, NcclConfig *) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
  ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*AllGather)(const void *, void *, size_t, int, ncclComm_t, cudaStream_t) = nullptr;
  const char *(*GetErrorString)(ncclResult_t) = nullptr;
  bool ok = false;
  char why[256] = "";
};

NcclApi &nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      snprintf(api.why, sizeof(api.why), "dlopen(libnccl.so.2): %s", dlerror());
      return;
    }
    api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
    api.CommInitRankConfig = reinterpret_cast<decltype(api.CommInitRankConfig)>(dlsym(h, "ncclCommInitRankConfig"));
    api.CommGetAsyncError = reinterpret_cast<decltype(api.CommGetAsyncError)>(dlsym(h, "ncclCommGetAsyncError"));
    api.CommFinalize = reinterpret_cast<decltype(api.CommFinalize)>(dlsym(h, "ncclCommFinalize"));
    api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
    api.CommAbort = reinterpret_cast<decltype(api.CommAbort)>(dlsym(h, "ncclCommAbort"));
    api.AllGather = reinterpret_cast<decltype(api.AllGather)>(dlsym(h, "ncclAllGather"));
    api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
    api.ok = api.GetUniqueId && api.CommInitRankConfig && api.CommGetAsyncError && api.CommFinalize &&
             api.CommDestroy && api.CommAbort && api.AllGather && api.GetErrorString;
    if (!api.ok) snprintf(api.why, sizeof(api.why), "libnccl.so.2 lacks an expected symbol");
  });
  return api;
}

int nccl_fail(ncclResult_t r, const char *what) {
  return fail(MPC_ERR_COMM, "%s: %s", what, nccl().GetErrorString ? nccl().GetErrorString(r) : "NCCL error");
}

// Communicators are created non-blocking, so that a rank that never joins cannot hold the caller
// forever: every NCCL call on one may return ncclInProgress, after which the communicator's state
// (ncclCommGetAsyncError) is polled here until it leaves that state. Returns the final state, or
// ncclInProgress when `timeout_ms` passed first.
ncclResult_t settle(ncclComm_t c, int64_t timeout_ms) {
  const auto t0 = std::chrono::steady_clock::now();
  for (int spin = 0;; ++spin) {
    ncclResult_t st = ncclInProgress;
    const ncclResult_t r = nccl().CommGetAsyncError(c, &st);
    if (r != 0) return r;
    if (st != ncclInProgress) return st;
    const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0);
    if (ms.count() >= timeout_ms) return ncclInProgress;
    if (spin < 1000)
      std::this_thread::yield();
    else
      std::this_thread::sleep_for(std::chrono::milliseconds(1));
  }
}

// The status of an NCCL call on communicator `comm` once it has settled.
int finish(mpc_comm *comm, ncclResult_t r, const char *what) {
  if (r == ncclInProgress) r = settle(comm->comm, comm->timeout_ms);
  if (r == ncclInProgress)
    return fail(MPC_ERR_TIMEOUT, "%s: rank %d of %d: NCCL did not finish within %lld ms (abort the communicator)",
                what, comm->rank, comm->nranks, (long long)comm->timeout_ms);
  return r ? nccl_fail(r, what) : MPC_OK;
}

constexpr int64_t kDefaultCommTimeoutMs = 600000;  // 10 minutes: far above any healthy init

}  // namespace
}  // namespace mpc

using namespace mpc;

extern "C" {

int mpc_comm_unique_id(void *id128) {
  if (!id128) return fail(MPC_ERR_INVALID, "mpc_comm_unique_id: null out pointer");
  NcclApi &api = nccl();
  if (!api.ok) return fail(MPC_ERR_COMM, "NCCL unavailable: %s", api.why);
  ncclUniqueId id;
  ncclResult_t r = api.GetUniqueId(&id);
  if (r) return nccl_fail(r, "ncclGetUniqueId");
  memcpy(id128, &id, sizeof(id));
  return MPC_OK;
}

int mpc_comm_init_timeout(mpc_device *dev, int nranks, int rank, const void *id128, int64_t timeout_ms,
                          mpc_comm **out) {
  int rc = enter(dev);
  if (rc) return rc;
  if (!id128 || !out) return fail(MPC_ERR_INVALID, "mpc_comm_init: null argument");
  if (nranks < 1 || rank < 0 || rank >= nranks) return fail(MPC_ERR_INVALID, "mpc_comm_init: rank %d of %d", rank, nranks);
  if (timeout_ms <= 0) return fail(MPC_ERR_INVALID, "mpc_comm_init: timeout %lld ms", (long long)timeout_ms);
  NcclApi &api = nccl();
  if (!api.ok) return fail(MPC_ERR_COMM, "NCCL unavailable: %s", api.why);
  ncclUniqueId id;
  memcpy(&id, id128, sizeof(id));
  NcclConfig cfg;  // non-blocking: the init runs on NCCL's own thread while this one keeps the deadline
  ncclComm_t c = nullptr;
  ncclResult_t r = api.CommInitRankConfig(&c, nranks, id, rank, &cfg);
  if (r != 0 && r != ncclInProgress) {
    if (c) api.CommAbort(c);
    return nccl_fail(r, "ncclCommInitRankConfig");
  }
  r = settle(c, timeout_ms);
  if (r != 0) {
    // The abort raises the communicator's abort flag, which NCCL's bootstrap waits poll, and
    // frees what the init had set up.
    api.CommAbort(c);
    if (r == ncclInProgress)
      return fail(MPC_ERR_TIMEOUT,
                  "mpc_comm_init: rank %d of %d: the communicator was not complete after %lld ms (a rank that "
                  "never joined?); it was aborted",
                  rank, nranks, (long long)timeout_ms);
    return nccl_fail(r, "ncclCommInitRankConfig");
  }
  *out = new mpc_comm{dev, c, nranks, rank, timeout_ms};
  return MPC_OK;
}

int mpc_comm_init(mpc_device *dev, int nranks, int rank, const void *id128, mpc_comm **out) {
  return mpc_comm_init_timeout(dev, nranks, rank, id128, kDefaultCommTimeoutMs, out);
}

int mpc_comm_destroy(mpc_comm *comm) {
  if (!comm) return MPC_OK;
  // Finalize (flushes the communicator's pending work; may complete asynchronously), then free.
  int rc = finish(comm, nccl().CommFinalize(comm->comm), "ncclCommFinalize");
  if (rc) {
    nccl().CommAbort(comm->comm);
    delete comm;
    return rc;
  }
  ncclResult_t r = nccl().CommDestroy(comm->comm);
  delete comm;
  return r ? nccl_fail(r, "ncclCommDestroy") : MPC_OK;
}

int mpc_comm_abort(mpc_comm *comm) {
  if (!comm) return MPC_OK;
  ncclResult_t r = nccl().CommAbort(comm->comm);
  delete comm;
  return r ? nccl_fail(r, "ncclCommAbort") : MPC_OK;
}

int mpc_allgather(mpc_comm *comm, const void *send, void *recv, size_t bytes, mpc_stream s) {
  if (!comm) return fail(MPC_ERR_INVALID, "mpc_allgather: null communicator");
  int rc = enter(comm->dev);
  if (rc) return rc;
  if (!send || !recv) return fail(MPC_ERR_INVALID, "mpc_allgather: null buffer");
  return finish(comm, nccl().AllGather(send, recv, bytes, ncclInt8, comm->comm, stream_of(comm->dev, s)),
                "ncclAllGather");
}

}  // extern "C"
