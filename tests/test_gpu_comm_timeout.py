"""Failure detection of the tensor-parallel exchange, on one GPU.

A consumer of the push all-reduce (wg_comm_reduce) waits word by word for
every rank's partial, with a time limit (wg_comm_set_wait); when a peer never
pushes, the wait runs out, the launch ends, and the next wg_sync returns
WG_TIMEOUT (the reference's counterpart: GpuError on a lost context,
packages/webgllm/src/gpu/gl.ts:502, classified in src/worker-errors.ts:14-24).

Both ranks of a world-2 exchange live on one device here: two exchange
buffers, one communicator per rank. No kernel waits on another launch: the
"missing peer" is a slot that nothing writes (the failure is made on the
host, by not issuing rank 1's push), and in the working exchange both pushes
complete, in stream order, before either reduce starts.
"""
import ctypes
import time

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

import webgllm_b200 as wg  # noqa: E402
from webgllm_b200 import _lib  # noqa: E402

P = ctypes.c_void_p
N, K, M = 512, 2048, 2
NBYTES = 4 << 20


def exchange(ctx):
    """Two zeroed exchange buffers and the communicators of ranks 0 and 1."""
    L = _lib.lib()
    bufs = [torch.zeros(NBYTES, dtype=torch.uint8, device="cuda") for _ in range(2)]
    arr = (P * 2)(*[b.data_ptr() for b in bufs])
    comms = []
    for r in range(2):
        h = P()
        _lib.check(L.wg_comm_init(P(ctx.handle), 2, r, arr, NBYTES, ctypes.byref(h)), ctx.handle)
        comms.append(h)
    return bufs, comms


def halves(ctx):
    """Two K halves of one matrix (rank r holds columns [r K/2, (r+1) K/2))."""
    blocks = O.config_q4_0_blocks(N, K, 7).reshape(N, K // 32, 18)
    mats = []
    for r in range(2):
        part = np.ascontiguousarray(blocks[:, r * (K // 64):(r + 1) * (K // 64)]).reshape(-1)
        m = wg.newQuantMatrix(N, K // 2, ctx=ctx)
        wg.packQ4_0(m, 0, part, N)
        mats.append(m)
    return mats


def push(ctx, comm, m, x):
    _lib.check(_lib.lib().wg_q4_matmul_push(P(ctx.handle), P(m.handle), None, P(x.data_ptr()), _lib.WG_F16, M, comm),
               ctx.handle)


def test_exchange_sums_both_ranks_partials():
    ctx = wg.context(0)
    ctx.use_torch_stream()
    L = _lib.lib()
    mats = halves(ctx)
    x = torch.from_numpy(O.config_activations(M, K, 3)).to("cuda", torch.float16)
    xs = [x[:, :K // 2].contiguous(), x[:, K // 2:].contiguous()]
    want = sum(wg.matmul(xs[r], mats[r], out_dtype=torch.float32) for r in range(2))
    bufs, comms = exchange(ctx)
    for rnd in range(3):  # both parities of the slots, then the first again
        for r in range(2):
            push(ctx, comms[r], mats[r], xs[r])
        outs = [torch.full((M, N), float("nan"), device="cuda") for _ in range(2)]
        for r in range(2):
            _lib.check(L.wg_comm_reduce(P(ctx.handle), comms[r], M, N, P(outs[r].data_ptr())), ctx.handle)
        ctx.sync()
        for r in range(2):
            err = ((outs[r] - want).norm() / want.norm()).item()
            assert err <= 1e-6, f"round {rnd} rank {r}: {err:.2e}"
    for c in comms:
        L.wg_comm_destroy(P(ctx.handle), c)
    del bufs


def test_missing_peer_times_out_and_the_context_stays_usable():
    ctx = wg.context(0)
    ctx.use_torch_stream()
    L = _lib.lib()
    mats = halves(ctx)
    x = torch.from_numpy(O.config_activations(M, K, 4)).to("cuda", torch.float16)
    x0 = x[:, :K // 2].contiguous()
    bufs, comms = exchange(ctx)
    assert L.wg_comm_set_wait(comms[0], 0) == _lib.WG_INVALID_ARGUMENT
    _lib.check(L.wg_comm_set_wait(comms[0], 20_000_000))  # 20 ms
    ctx.sync()
    # rank 0 pushes; rank 1 never does (made on the host: its push is not issued)
    push(ctx, comms[0], mats[0], x0)
    out = torch.zeros((M, N), device="cuda")
    t0 = time.perf_counter()
    _lib.check(L.wg_comm_reduce(P(ctx.handle), comms[0], M, N, P(out.data_ptr())), ctx.handle)
    st = L.wg_sync(P(ctx.handle))
    waited = time.perf_counter() - t0
    assert st == _lib.WG_TIMEOUT, _lib.lib().wg_error_string(st)
    assert "wait ran out" in L.wg_last_error(P(ctx.handle)).decode()
    assert waited < 1.5, f"the timed-out reduce took {waited:.2f} s (limit 20 ms a wait)"
    # the flag is cleared and the context still computes
    assert L.wg_sync(P(ctx.handle)) == _lib.WG_OK
    y = wg.matmul(x0, mats[0], out_dtype=torch.float32)
    ctx.sync()
    ref = O.c_ref_f64(O.config_q4_0_blocks(N, K, 7).reshape(N, K // 32, 18)[:, :K // 64].reshape(-1),
                      x0.float().cpu().numpy(), N, K // 2)
    l2, mx = O.rel_errors(y.cpu().numpy(), ref)
    assert l2 <= O.TOL and mx <= O.TOL
    for c in comms:
        L.wg_comm_destroy(P(ctx.handle), c)
    del bufs
