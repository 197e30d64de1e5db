"""Two ranks (torch.distributed.run): rank 1 never enters a peer barrier; rank 0's barrier kernel
gives up after a 200 ms wait limit and its synchronisation reports MPC_ERR_TIMEOUT. Both ranks
leave between steps with nothing in flight; the communicator is aborted, not destroyed."""
import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "math-plus_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)


def main():
    import ctypes as C

    import torch
    import torch.distributed as dist

    from tensor_cuda import _ffi as F
    from tensor_cuda.parallel import PeerGroup
    from tensor_cuda.runtime import Device

    rank, local = int(os.environ["RANK"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    dev = Device.shared(local)
    F.call("mpc_set_wait_timeout_ns", dev.handle, C.c_uint64(200_000_000))
    group = PeerGroup.from_torch(dev)
    buf = group.peer_buffer(1 << 20)
    buf.barrier()  # both ranks: a barrier that completes
    dev.sync()
    dist.barrier()
    if rank == 0:
        buf.barrier()  # rank 1 never arrives
        try:
            dev.sync()
            raise SystemExit("rank 0: the barrier completed without its peer")
        except F.MpcError as e:
            assert e.status == F.ERR_TIMEOUT, e
        F.call("mpc_device_clear_error", dev.handle)
        print("rank 0 timed out as expected", flush=True)
    else:
        print("rank 1 skipped the barrier", flush=True)
    dist.barrier()  # host-side: nothing of ours is in flight on either rank
    group.abort()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
