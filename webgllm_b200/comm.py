"""The push all-reduce exchange of a tensor-parallel group
(include/webgllm_comm.h), set up over torch.distributed.

Every rank allocates one IPC-shareable buffer, the 64-byte handles are
all-gathered, each rank maps its peers' buffers, and the library's
communicator then lets a row-parallel matmul push its partial sums into
every rank's buffer from its own epilogue (`wg_q4_matmul_push`) and a
following `wg_comm_reduce` sum them.
"""
from __future__ import annotations

import ctypes

from . import _lib
from ._lib import check

P = ctypes.c_void_p


class PushComm:
    def __init__(self, ctx, rank: int, world: int, group=None, nbytes: int = 8 << 20):
        import torch.distributed as dist

        L = _lib.lib()
        self.ctx, self.rank, self.world, self.group = ctx, rank, world, group
        self.own = P()
        handle = (ctypes.c_ubyte * 64)()
        check(L.wg_ipc_alloc(P(ctx.handle), nbytes, ctypes.byref(self.own), handle), ctx.handle)
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.opened = []
        ptrs = []
        for r in range(world):
            if r == rank:
                ptrs.append(self.own.value)
                continue
            q = P()
            hb = (ctypes.c_ubyte * 64).from_buffer_copy(handles[r])
            check(L.wg_ipc_open(P(ctx.handle), hb, ctypes.byref(q)), ctx.handle)
            self.opened.append(q.value)
            ptrs.append(q.value)
        arr = (P * world)(*ptrs)
        self.handle = P()
        check(L.wg_comm_init(P(ctx.handle), world, rank, arr, nbytes, ctypes.byref(self.handle)), ctx.handle)
        n = ctypes.c_size_t()
        check(L.wg_comm_slot(self.handle, ctypes.byref(n)))
        self.slot = n.value
        dist.barrier(group=group)

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
        import torch.distributed as dist

        if self.handle is None:
            return
        L = _lib.lib()
        L.wg_comm_destroy(P(self.ctx.handle), self.handle)
        self.handle = None
        dist.barrier(group=self.group)  # no rank still reads or writes a peer's buffer
        for q in self.opened:
            L.wg_ipc_close(P(self.ctx.handle), P(q))
        self.opened = []
        dist.barrier(group=self.group)  # every mapping of our buffer is closed
        L.wg_ipc_free(P(self.ctx.handle), self.own)
