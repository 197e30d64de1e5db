#include "mpc_internal.h"
using namespace mpc;
extern "C" {
int mpc_softmax(mpc_device *, const void *, int32_t, float *, int64_t, int64_t, int64_t, mpc_stream) { return fail(MPC_ERR_UNSUPPORTED, "not built yet"); }
int mpc_gelu(mpc_device *, const void *, int32_t, void *, int32_t, int64_t, mpc_stream) { return fail(MPC_ERR_UNSUPPORTED, "not built yet"); }
int mpc_add(mpc_device *, const void *, const void *, void *, int32_t, int64_t, int64_t, mpc_stream) { return fail(MPC_ERR_UNSUPPORTED, "not built yet"); }
int mpc_layer_norm(mpc_device *, const void *, int32_t, const float *, const float *, float, void *, int32_t, int64_t, int64_t, mpc_stream) { return fail(MPC_ERR_UNSUPPORTED, "not built yet"); }
int mpc_embedding(mpc_device *, const void *, int32_t, const int32_t *, void *, int64_t, int64_t, int64_t, int64_t *, mpc_stream) { return fail(MPC_ERR_UNSUPPORTED, "not built yet"); }
int mpc_cast(mpc_device *, const void *, int32_t, void *, int32_t, int64_t, mpc_stream) { return fail(MPC_ERR_UNSUPPORTED, "not built yet"); }
int mpc_comm_unique_id(void *) { return fail(MPC_ERR_UNSUPPORTED, "not built yet"); }
int mpc_comm_init(mpc_device *, int, int, const void *, mpc_comm **) { return fail(MPC_ERR_UNSUPPORTED, "not built yet"); }
int mpc_comm_destroy(mpc_comm *) { return MPC_OK; }
int mpc_comm_abort(mpc_comm *) { return MPC_OK; }
int mpc_allgather(mpc_comm *, const void *, void *, size_t, mpc_stream) { return fail(MPC_ERR_UNSUPPORTED, "not built yet"); }
}
