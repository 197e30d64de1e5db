#include "mpc_internal.h"
namespace mpc {
int sdpa_run(mpc_device *, const mpc_sdpa_desc *, const void *, const void *, const void *, const void *, void *,
             float *, cudaStream_t) {
  return fail(MPC_ERR_UNSUPPORTED, "mpc_sdpa: not built yet");
}
}  // namespace mpc
