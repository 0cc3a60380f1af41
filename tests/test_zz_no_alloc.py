"""wg_q4_matmul_static, the matmul entry point that allocates nothing.

Callers that cannot let a library allocate device memory (CUDA graph capture,
fixed memory budgets, decode loops that cannot take cudaMalloc's device
synchronisation) use it instead of wg_q4_matmul: its scratch is a fixed
32 MiB array in the library's device memory. These tests call it through the
C ABI and compare it with wg_q4_matmul, twice in a row (the array keeps the
previous call's contents), within the parity tolerance of the other tests.
This file is collected last, so a failure here comes after every other test
has run; it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

import webgllm_b200 as wg  # noqa: E402
from webgllm_b200 import _lib  # noqa: E402

DT = {torch.float32: _lib.WG_F32, torch.float16: _lib.WG_F16, torch.bfloat16: _lib.WG_BF16}


def call(fn, m, x, y):
    ctx = m.ctx
    ctx.use_torch_stream()
    st = fn(ctypes.c_void_p(ctx.handle), ctypes.c_void_p(m.handle), ctypes.c_void_p(x.data_ptr()), DT[x.dtype],
            x.shape[0], ctypes.c_void_p(y.data_ptr()), DT[y.dtype])
    _lib.check(st, ctx.handle)


@pytest.mark.parametrize("M,N,K,xdt", [
    (1, 512, 1024, torch.float16),      # GEMV: no scratch at all
    (8, 4096, 4096, torch.float16),     # the wide GEMV (x resident per CTA)
    (24, 512, 28672, torch.float16),    # 17..32 rows at long K: the GEMM, as wg_q4_matmul routes it
    (64, 512, 4096, torch.float16),     # GEMM with K split (reduced on chip): no scratch
    (256, 4096, 4096, torch.float32),   # config 1's M = 256, x converted to fp16 in the array
    (100, 384, 512, torch.float32),     # x converted to fp16 in the array
    (1024, 1024, 2048, torch.bfloat16), # no split, x conversion only
])
def test_static_scratch_matches_the_allocating_entry_point(M, N, K, xdt):
    L = _lib.lib()
    blocks = O.config_q4_0_blocks(N, K, M + N)
    m = wg.newQuantMatrix(N, K)
    wg.packQ4_0(m, 0, blocks, N)
    for call_no in range(2):
        x = torch.from_numpy(O.config_activations(M, K, M + call_no)).to("cuda", xdt)
        want = torch.empty((M, N), device="cuda", dtype=torch.float32)
        got = torch.full((M, N), float("nan"), device="cuda", dtype=torch.float32)
        call(L.wg_q4_matmul, m, x, want)
        call(L.wg_q4_matmul_static, m, x, got)
        torch.cuda.synchronize()
        l2, mx = O.rel_errors(got.cpu().numpy(), want.cpu().numpy())
        assert l2 <= O.TOL and mx <= O.TOL, f"call {call_no}: {l2:.2e} {mx:.2e}"
        ref = O.c_ref_f64(blocks, x.float().cpu().numpy(), N, K)
        l2, mx = O.rel_errors(got.cpu().numpy(), ref)
        assert l2 <= O.TOL and mx <= O.TOL, f"call {call_no} vs fp64: {l2:.2e} {mx:.2e}"


def test_static_scratch_rejects_needs_beyond_its_size():
    # f32 x of 4096 x 8192 needs a 64 MiB fp16 copy: more than the 32 MiB array.
    L = _lib.lib()
    N, K, M = 16, 8192, 4096
    m = wg.newQuantMatrix(N, K)
    x = torch.zeros((M, K), device="cuda", dtype=torch.float32)
    y = torch.zeros((M, N), device="cuda", dtype=torch.float32)
    m.ctx.use_torch_stream()
    st = L.wg_q4_matmul_static(ctypes.c_void_p(m.ctx.handle), ctypes.c_void_p(m.handle),
                               ctypes.c_void_p(x.data_ptr()), _lib.WG_F32, M, ctypes.c_void_p(y.data_ptr()),
                               _lib.WG_F32)
    assert st == _lib.WG_UNSUPPORTED
    msg = L.wg_last_error(ctypes.c_void_p(m.ctx.handle)).decode()
    assert "scratch" in msg and str(32 << 20) in msg
