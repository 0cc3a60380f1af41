"""The tensor-parallel group of a model split across the GPUs of one node
(include/webgllm_comm.h), through the library alone.

TensorGroup joins an NCCL group inside the library (wg_tp_init): the group's
all-reduces (row-parallel sums of prompt rows, the vocabulary-parallel
greedy pick) and the push exchange's set-up (wg_tp_comm: IPC handles
all-gathered through NCCL) need no PyTorch. Only the 128-byte group id has
to travel from one rank to the others, by any transport: `from_torch` uses
an existing torch.distributed group for that (and for nothing else), the
tests use a multiprocessing queue.

PushComm is the push all-reduce over a TensorGroup: a row-parallel matmul
pushes its partial sums into every rank's exchange buffer from its own
epilogue (`wg_q4_matmul_push`) and a following `wg_comm_reduce` (or
`wg_comm_reduce_norm`) sums them.
"""
from __future__ import annotations

import ctypes

from . import _lib
from ._lib import check

P = ctypes.c_void_p

WG_TP_F32, WG_TP_F16, WG_TP_BF16, WG_TP_I64 = 0, 1, 2, 3
WG_TP_SUM, WG_TP_MAX = 0, 1


def unique_id() -> bytes:
    """A new group id (ncclGetUniqueId), to be sent to every rank."""
    buf = (ctypes.c_ubyte * 128)()
    check(_lib.lib().wg_tp_unique_id(buf))
    return bytes(buf)


class TensorGroup:
    """This process's rank of a tensor-parallel group (one process per
    GPU); every rank passes the same `group_id`."""

    def __init__(self, ctx, rank: int, world: int, group_id: bytes):
        if len(group_id) != 128:
            raise ValueError("a group id has 128 bytes")
        self.ctx, self.rank, self.world = ctx, rank, world
        self.handle = P()
        idb = (ctypes.c_ubyte * 128).from_buffer_copy(group_id)
        check(_lib.lib().wg_tp_init(P(ctx.handle), world, rank, idb, ctypes.byref(self.handle)), ctx.handle)

    @classmethod
    def from_torch(cls, ctx, group=None) -> "TensorGroup":
        """Joins a group of the ranks of a torch.distributed group, which
        only carries the id from rank 0 to the others."""
        import torch.distributed as dist

        rank, world = dist.get_rank(group), dist.get_world_size(group)
        obj = [unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=dist.get_global_rank(group, 0) if group else 0, group=group)
        return cls(ctx, rank, world, obj[0])

    def all_reduce(self, t, op: str = "sum") -> None:
        """In place on the context's stream: sum (f32 / f16 / bf16) or max
        (int64) of a contiguous CUDA tensor."""
        import torch

        dt = {torch.float32: WG_TP_F32, torch.float16: WG_TP_F16, torch.bfloat16: WG_TP_BF16,
              torch.int64: WG_TP_I64}[t.dtype]
        if not t.is_contiguous():
            raise ValueError("all_reduce needs a contiguous tensor")
        code = WG_TP_SUM if op == "sum" else WG_TP_MAX
        check(_lib.lib().wg_tp_allreduce(P(self.ctx.handle), self.handle, P(t.data_ptr()), t.numel(), dt, code),
              self.ctx.handle)

    def barrier(self, timeout_ms: int = 0) -> None:
        check(_lib.lib().wg_tp_barrier(P(self.ctx.handle), self.handle, timeout_ms), self.ctx.handle)

    def push_comm(self, nbytes: int = 8 << 20) -> "PushComm":
        return PushComm(self, nbytes)

    def close(self) -> None:
        if self.handle is not None:
            _lib.lib().wg_tp_destroy(P(self.ctx.handle), self.handle)
            self.handle = None


class PushComm:
    """The push all-reduce over a TensorGroup (wg_tp_comm): this rank's
    exchange buffer of `nbytes` and its mappings of every peer's."""

    def __init__(self, group: TensorGroup, nbytes: int = 8 << 20):
        L = _lib.lib()
        self.group, self.ctx = group, group.ctx
        self.rank, self.world = group.rank, group.world
        self.handle = P()
        check(L.wg_tp_comm(P(self.ctx.handle), group.handle, nbytes, ctypes.byref(self.handle)), self.ctx.handle)
        n = ctypes.c_size_t()
        check(L.wg_comm_slot(self.handle, ctypes.byref(n)))
        self.slot = n.value

    def push(self, m, rows: int, x=None, pro=None):
        """Partial rows x W^T of matrix m (x a CUDA fp16/f32 tensor, or a
        wg_prologue) into every rank's buffer."""
        L = _lib.lib()
        if pro is not None:
            st = L.wg_q4_matmul_push(P(self.ctx.handle), P(m.handle), ctypes.byref(pro), None, 1, rows, self.handle)
        else:
            import torch

            xd = _lib.WG_F16 if x.dtype == torch.float16 else _lib.WG_F32
            st = L.wg_q4_matmul_push(P(self.ctx.handle), P(m.handle), None, P(x.data_ptr()), xd, rows, self.handle)
        check(st, self.ctx.handle)

    def reduce(self, out, rows: int, n: int):
        check(_lib.lib().wg_comm_reduce(P(self.ctx.handle), self.handle, rows, n, P(out.data_ptr())), self.ctx.handle)

    def reduce_norm(self, resid, weight, eps: float, resid_out, x_out, rows: int, k: int):
        """x_out (fp16) = rmsnorm(resid + the exchanged sum) * weight, and
        resid_out = resid + the sum: the all-reduce, residual add and norm in
        one launch."""
        check(_lib.lib().wg_comm_reduce_norm(P(self.ctx.handle), self.handle, rows, k, P(resid.data_ptr()),
                                             P(weight.data_ptr()), ctypes.c_float(eps), P(resid_out.data_ptr()),
                                             P(x_out.data_ptr())), self.ctx.handle)

    def close(self):
        """Collective: every rank of the group calls it."""
        if self.handle is None:
            return
        h, self.handle = self.handle, None
        check(_lib.lib().wg_comm_destroy(P(self.ctx.handle), h), self.ctx.handle)
