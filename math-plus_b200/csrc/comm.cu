// NCCL over NVLink / NVSwitch, one rank per process: the one exchange step of the path (the
// all-gather that reassembles a GEMM split over N across GPUs). NCCL is resolved at run time
// with dlopen("libnccl.so.2"), so a process that already loaded NCCL (torch.distributed) shares
// that copy instead of loading a second one.
#include <dlfcn.h>

#include <cstring>

#include "mpc_internal.h"

namespace mpc {
namespace {

typedef int ncclResult_t;
typedef void *ncclComm_t;
struct ncclUniqueId {
  char internal[128];
};
enum { ncclInt8 = 0 };

struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
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
    api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(dlsym(h, "ncclCommInitRank"));
    api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
    api.CommAbort = reinterpret_cast<decltype(api.CommAbort)>(dlsym(h, "ncclCommAbort"));
    api.AllGather = reinterpret_cast<decltype(api.AllGather)>(dlsym(h, "ncclAllGather"));
    api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
    api.ok = api.GetUniqueId && api.CommInitRank && api.CommDestroy && api.CommAbort && api.AllGather &&
             api.GetErrorString;
    if (!api.ok) snprintf(api.why, sizeof(api.why), "libnccl.so.2 lacks an expected symbol");
  });
  return api;
}

int nccl_fail(ncclResult_t r, const char *what) {
  return fail(MPC_ERR_COMM, "%s: %s", what, nccl().GetErrorString ? nccl().GetErrorString(r) : "NCCL error");
}

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

int mpc_comm_init(mpc_device *dev, int nranks, int rank, const void *id128, mpc_comm **out) {
  int rc = enter(dev);
  if (rc) return rc;
  if (!id128 || !out) return fail(MPC_ERR_INVALID, "mpc_comm_init: null argument");
  if (nranks < 1 || rank < 0 || rank >= nranks) return fail(MPC_ERR_INVALID, "mpc_comm_init: rank %d of %d", rank, nranks);
  NcclApi &api = nccl();
  if (!api.ok) return fail(MPC_ERR_COMM, "NCCL unavailable: %s", api.why);
  ncclUniqueId id;
  memcpy(&id, id128, sizeof(id));
  ncclComm_t c = nullptr;
  ncclResult_t r = api.CommInitRank(&c, nranks, id, rank);
  if (r) return nccl_fail(r, "ncclCommInitRank");
  *out = new mpc_comm{dev, c, nranks, rank};
  return MPC_OK;
}

int mpc_comm_destroy(mpc_comm *comm) {
  if (!comm) return MPC_OK;
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
  ncclResult_t r = nccl().AllGather(send, recv, bytes, ncclInt8, comm->comm, stream_of(comm->dev, s));
  return r ? nccl_fail(r, "ncclAllGather") : MPC_OK;
}

}  // extern "C"
