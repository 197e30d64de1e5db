"""Multi-GPU: one process per GPU, a communicator over NVLink, and the column-split GEMM.

The reference runs on one device; this module adds the one exchange step the GEMM path has when
it is split across GPUs: rank r of p computes ``C[:, r*n:(r+1)*n] = A @ B[:, r*n:(r+1)*n]`` and
every rank ends up with the whole ``C [m, p*n]``. Two ways to get there:

* ``ColumnSplitGemm(..., fused=True)`` (the default): one kernel per rank whose epilogue stores
  each finished output block into every rank's copy of C (the shard-major ``[p, m, n]`` view)
  through peer (IPC) mappings, so the NVLink transfer overlaps the tensor-core work; a local
  permute gives the row-major ``[m, p*n]`` when asked for (``mpc_gemm_allgather``);
* ``fused=False``: the GEMM into a local ``[m, n]`` shard, an NCCL all-gather into the
  shard-major ``[p, m, n]`` block, then a ``[p, m, n] -> [m, p, n]`` permute kernel.

Every other part of the path (batched GEMM, attention, a GPT-2 forward) shards over independent
batch entries and needs no collective: ``plan.batch_shard`` gives each rank its slice.
"""
from __future__ import annotations

import ctypes as C

from . import _ffi as F
from . import plan as P
from .runtime import Device, gemm_desc


def unique_id() -> bytes:
    """A fresh 128-byte NCCL id; rank 0 makes it and hands it to the others (any transport)."""
    F.load()
    buf = (C.c_uint8 * 128)()
    F.call("mpc_comm_unique_id", buf)
    return bytes(buf)


class PeerGroup:
    """One rank of a communicator (``mpc_comm``). Collective calls must be made by every rank in
    the same order."""

    def __init__(self, device: Device, rank: int, world: int, uid: bytes, timeout_ms: int | None = None):
        """Joins the group; with ``timeout_ms``, a group that is not complete in time (a rank that
        never joins) raises ``MpcError`` with status TIMEOUT instead of waiting (the default limit
        is 10 minutes)."""
        if len(uid) != 128:
            raise ValueError("PeerGroup: the id is 128 bytes (from unique_id() on one rank)")
        self.device, self.rank, self.world = device, rank, world
        h = C.c_void_p()
        uid_buf = (C.c_uint8 * 128).from_buffer_copy(uid)
        if timeout_ms is None:
            F.call("mpc_comm_init", device.handle, world, rank, uid_buf, C.byref(h))
        else:
            F.call("mpc_comm_init_timeout", device.handle, world, rank, uid_buf, int(timeout_ms), C.byref(h))
        self.handle = h.value

    @classmethod
    def from_torch(cls, device: Device, group=None) -> "PeerGroup":
        """Builds the communicator over an initialised torch.distributed group (its rank 0
        broadcasts the id)."""
        import torch.distributed as dist
        obj = [unique_id() if dist.get_rank(group) == 0 else None]
        dist.broadcast_object_list(obj, src=0, group=group)
        return cls(device, dist.get_rank(group), dist.get_world_size(group), obj[0])

    def allgather(self, send: int, recv: int, nbytes: int, stream=None) -> None:
        """``nbytes`` from every rank into ``recv`` (rank r's block at r * nbytes)."""
        F.call("mpc_allgather", self.handle, C.c_void_p(send), C.c_void_p(recv), nbytes, stream)

    def peer_buffer(self, nbytes: int) -> "PeerBuffer":
        return PeerBuffer(self, nbytes)

    def destroy(self) -> None:
        if self.handle is not None:
            F.call("mpc_comm_destroy", self.handle)
            self.handle = None

    def abort(self) -> None:
        if self.handle is not None:
            F.load().mpc_comm_abort(C.c_void_p(self.handle))
            self.handle = None


class PeerBuffer:
    """``nbytes`` of device memory on every rank, each rank's block mapped into every process."""

    def __init__(self, group: PeerGroup, nbytes: int):
        self.group, self.nbytes = group, int(nbytes)
        h = C.c_void_p()
        F.call("mpc_peer_buffer_create", group.handle, self.nbytes, C.byref(h))
        self.handle = h.value

    def ptr(self, rank: int | None = None) -> int:
        """Address of ``rank``'s block (default: this rank's) as mapped in this process."""
        p = C.c_void_p()
        F.call("mpc_peer_buffer_ptr", self.handle, self.group.rank if rank is None else rank, C.byref(p))
        return p.value

    def barrier(self, stream=None) -> None:
        F.call("mpc_peer_barrier", self.handle, stream)

    def destroy(self) -> None:
        if self.handle is not None:
            F.call("mpc_peer_buffer_destroy", self.handle)
            self.handle = None


class ColumnSplitGemm:
    """``C = A @ B`` with B's columns split over the group: this rank holds ``A [m, k]`` and its
    block ``B_r [k, n]`` (``b_layout=F.B_KN``) or ``[n, k]`` (``F.B_NK``); every rank gets the whole
    C, as row-major ``[m, p*n]`` (``layout="rows"``) or as the shard-major blocked view
    ``[p, m, n]`` (``layout="blocks"``). ``__call__`` returns its device address."""

    def __init__(self, group: PeerGroup, m: int, n: int, k: int, dtype_in: str = "bf16", dtype_out: str = "bf16",
                 b_layout: int = F.B_KN, fused: bool = True, layout: str = "rows"):
        if layout not in ("rows", "blocks"):
            raise ValueError(f"ColumnSplitGemm: layout {layout!r} (rows or blocks)")
        self.plan = P.column_split_plan(m, n * group.world, k, group.world, dtype_out)
        self.group, self.m, self.n, self.k, self.fused, self.layout = group, m, n, k, fused, layout
        self.desc = gemm_desc(m, n, k, F.DTYPE_CODES[dtype_in], F.DTYPE_CODES[dtype_out], b_layout)
        self.eo = F.DTYPE_BYTES[F.DTYPE_CODES[dtype_out]]
        total = m * n * group.world * self.eo
        dev = group.device
        # with one rank the blocked view [1, m, n] already is row-major
        self.rows = dev.alloc(total) if layout == "rows" and group.world > 1 else None
        if fused:
            self.blocks = group.peer_buffer(total)
            self.blocks_ptr = self.blocks.ptr()
        else:
            self.shard = dev.alloc(m * n * self.eo)
            self.blocks = dev.alloc(total)
            self.blocks_ptr = self.blocks.ptr
            self._shape = (C.c_int64 * 3)(group.world, m, n)
            self._perm = (C.c_int32 * 3)(*self.plan.gathered_to_output_perm())

    @property
    def out_ptr(self) -> int:
        return self.rows.ptr if self.rows is not None else self.blocks_ptr

    def __call__(self, a: int, b: int, stream=None) -> int:
        """Queues the step on ``stream``; returns the device address of this rank's whole C."""
        dev = self.group.device
        rows = C.c_void_p(self.rows.ptr) if self.rows is not None else None
        if self.fused:
            F.call("mpc_gemm_allgather", dev.handle, C.byref(self.desc), C.c_void_p(a), C.c_void_p(b), None,
                   self.blocks.handle, rows, stream)
            return self.out_ptr
        dev.gemm(self.desc, a, b, self.shard.ptr, None, stream)
        self.group.allgather(self.shard.ptr, self.blocks.ptr, self.m * self.n * self.eo, stream)
        if rows is not None:
            F.call("mpc_transpose", dev.handle, C.c_void_p(self.blocks.ptr), rows, self.eo, 3, self._shape,
                   self._perm, stream)
        return self.out_ptr

    def destroy(self) -> None:
        if self.fused:
            self.blocks.destroy()
        else:
            self.shard.free()
            self.blocks.free()
        if self.rows is not None:
            self.rows.free()


def gemm_multi_store(device: Device, desc: F.GemmDesc, a: int, b: int, dsts, ldc: int, col_offset: int,
                     bias: int | None = None, stream=None) -> None:
    """The product of ``desc`` stored into each row-major matrix of ``dsts`` (row pitch ``ldc``
    elements) at columns ``col_offset .. col_offset + n - 1``."""
    arr = (C.c_void_p * len(dsts))(*dsts)
    F.call("mpc_gemm_multi_store", device.handle, C.byref(desc), C.c_void_p(a), C.c_void_p(b),
           C.c_void_p(bias) if bias else None, arr, len(dsts), ldc, col_offset, stream)


__all__ = ["unique_id", "PeerGroup", "PeerBuffer", "ColumnSplitGemm", "gemm_multi_store"]
