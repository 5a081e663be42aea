"""One node, one process per GPU: the communicator and the expert-parallel plan.

``Comm`` wraps catnn_comm (include/catnn_b200.h): NCCL for the gradient
allreduce and the generic all-to-all, CUDA IPC peer mappings for the fused
MoE dispatch/combine kernels, and a device barrier with bounded waits. The
NCCL group id travels from rank 0 over the caller's torch.distributed
process group (gloo or nccl); nothing else crosses the host.

The reference runs one device handler per device in scoped worker threads
and moves tensors between devices on the host (crates/catnn-rt/src/dist.rs:
441-517, transfer.rs); it models expert parallelism as E/EP experts per rank
with a 2·top_k·H activation all-to-all per layer whose remote fraction is
(EP-1)/EP (crates/catnn-compile/src/spark_place.rs:119-131,196). The
functions below restate the partition this backend uses so that host code
and the CPU tests can check it: rank r trains sequences
[r·B/N, (r+1)·B/N) of the global batch and owns experts [r·E/N, (r+1)·E/N);
an expert's received rows are ordered by global (token, slot) pair, which is
the one-GPU permutation order, and padded to ``align`` rows per expert.
"""
import ctypes as C

import numpy as np

from . import _lib

COMM_ID_BYTES = 128


def shard(rank, world, batch, seq):
    """(first global token, token count) of rank's share of a [batch, seq] batch."""
    if batch % world:
        raise ValueError(f"batch {batch} is not divisible by {world} ranks")
    b = batch // world
    return rank * b * seq, b * seq


def expert_owner(e, experts, world):
    if experts % world:
        raise ValueError(f"experts {experts} is not divisible by {world} ranks")
    return e // (experts // world)


def ep_plan(counts_all, rank, align):
    """Host restatement of the device plan (moe_ep.cu k_ep_plan).

    counts_all: int array [world, E], pairs rank s routes to expert e.
    Returns (off_own [El+1], total_own [El], base [E]): row offsets of this
    rank's experts in its receive buffer, rows received per own expert, and
    for every expert the first row of this rank's pairs in the owner's buffer.
    """
    counts_all = np.asarray(counts_all, np.int64)
    world, E = counts_all.shape
    El = E // world
    off_own = np.zeros(El + 1, np.int64)
    total_own = np.zeros(El, np.int64)
    base = np.zeros(E, np.int64)
    off = 0
    for e in range(E):
        if e % El == 0:
            off = 0
        tot = int(counts_all[:, e].sum())
        base[e] = off + int(counts_all[:rank, e].sum())
        owner = e // El
        if owner == rank:
            off_own[e - rank * El] = off
            total_own[e - rank * El] = tot
        off += -(-tot // align) * align
        if owner == rank and e % El == El - 1:
            off_own[El] = off
    return off_own, total_own, base


def ep_dest_rows(idx, counts_all, rank, align):
    """Row of each local pair (idx [T, k] expert ids) in its owner's buffer:
    base[e] + rank of the pair among this rank's pairs for e, in pair order."""
    idx = np.asarray(idx).reshape(-1)
    _, _, base = ep_plan(counts_all, rank, align)
    seen = np.zeros(len(base), np.int64)
    dest = np.empty(idx.size, np.int64)
    for i, e in enumerate(idx):
        dest[i] = base[e] + seen[e]
        seen[e] += 1
    return dest


class Comm:
    """catnn_comm of this process (one rank, one GPU)."""

    def __init__(self, rank, world, device, group_id=None):
        import torch

        from . import ops
        self.rank, self.world, self.device = int(rank), int(world), int(device)
        self.ctx = ops.context(self.device)
        h = C.c_void_p()
        gid = None
        if world > 1:
            if group_id is None or len(group_id) != COMM_ID_BYTES:
                raise ValueError("world > 1 needs the 128-byte group id of rank 0")
            gid = C.create_string_buffer(bytes(group_id), COMM_ID_BYTES)
        with torch.cuda.device(self.device):
            _lib.call("catnn_comm_create", self.ctx.bind(), self.rank, self.world, gid, C.byref(h))
        self.handle = h

    @staticmethod
    def unique_id():
        buf = C.create_string_buffer(COMM_ID_BYTES)
        _lib.call("catnn_comm_unique_id", buf)
        return buf.raw

    @classmethod
    def from_process_group(cls, device, group=None):
        """Build the communicator of this rank of a torch.distributed group:
        rank 0 makes the NCCL id and broadcasts it over the group."""
        import torch.distributed as dist
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        obj = [cls.unique_id() if (rank == 0 and world > 1) else None]
        if world > 1:
            dist.broadcast_object_list(obj, src=0, group=group)
        return cls(rank, world, device, obj[0])

    def _bind(self):
        return self.ctx.bind()

    def set_timeout_ms(self, ms):
        self._bind()
        _lib.call("catnn_comm_set_timeout_ms", self.handle, int(ms))

    def allreduce(self, t):
        """In-place sum over ranks of a contiguous fp32/bf16 CUDA tensor."""
        import torch
        self._bind()
        dt = 1 if t.dtype == torch.bfloat16 else 0
        _lib.call("catnn_comm_allreduce", self.handle, C.c_void_p(t.data_ptr()), t.numel(), dt)
        return t

    def all_to_all(self, send, send_bytes, recv, recv_bytes):
        self._bind()
        sb = (C.c_int64 * self.world)(*[int(x) for x in send_bytes])
        rb = (C.c_int64 * self.world)(*[int(x) for x in recv_bytes])
        _lib.call("catnn_comm_all_to_all", self.handle, C.c_void_p(send.data_ptr()), sb, C.c_void_p(recv.data_ptr()),
                  rb)
        return recv

    def barrier(self):
        self._bind()
        _lib.call("catnn_comm_barrier", self.handle)

    def signal(self, peer, epoch):
        self._bind()
        _lib.call("catnn_comm_signal", self.handle, int(peer), int(epoch))

    def wait(self, peer, epoch):
        self._bind()
        _lib.call("catnn_comm_wait", self.handle, int(peer), int(epoch))

    def check(self):
        self._bind()
        _lib.call("catnn_comm_check", self.handle)

    def close(self):
        if getattr(self, "handle", None):
            self._bind()
            _lib.call("catnn_comm_destroy", self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
