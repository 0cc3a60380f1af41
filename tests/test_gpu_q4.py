"""Parity of the CUDA path with the oracle, through the C ABI.

Repacks are bit-exact (matrixRow read back from the device equals the
oracle's matrixRow of the reference's QuantMatrix). Matmul outputs must be
within the north star's rel 1e-3 of BOTH oracle modes (fp64 exact, and the
reference shader's fp16-partial emulation), measured as
||y - ref||_2 / ||ref||_2 and max|y - ref| / max|ref|.
"""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

import webgllm_b200 as wg  # noqa: E402

TOL = O.TOL


def make(N, K, seed):
    blocks = O.config_q4_0_blocks(N, K, seed)
    m = wg.newQuantMatrix(N, K)
    wg.packQ4_0(m, 0, blocks, N)
    host = O.HostQuantMatrix(N, K)
    O.c_pack_q4_0(host, 0, blocks, N)
    return blocks, m, host


def check_close(y, ref, what):
    l2, mx = O.rel_errors(y, ref)
    assert l2 <= TOL and mx <= TOL, f"{what}: l2 {l2:.3e} max {mx:.3e}"
    return l2, mx


def run(m, x_np, x_dtype=torch.float16, y_dtype=torch.float32):
    x = torch.from_numpy(x_np).to("cuda", dtype=x_dtype)
    y = wg.matmul(x, m, out_dtype=y_dtype)
    torch.cuda.synchronize()
    return y.float().cpu().numpy(), x.float().cpu().numpy()


# ---------------------------------------------------------------- repack


@pytest.mark.parametrize("N,K", [(4, 32), (12, 96), (16, 64), (64, 256), (260, 160), (2048, 2048)])
def test_pack_q4_0_round_trip_is_bit_exact(N, K):
    _, m, host = make(N, K, N * 7 + K)
    for n in sorted({0, 1, N // 2, N - 1, min(N - 1, 17)}):
        assert np.array_equal(wg.matrixRow(m, n), O.c_matrix_row(host, n)), n


def test_pack_in_parts_with_permutation_matches_one_pack():
    # Parts of 4 and 20 rows: the boundary falls inside a 16-row tile.
    N, K = 24, 128
    blocks = O.config_q4_0_blocks(N, K, 5)
    perm = np.array([3, 0, 2, 1], dtype=np.int32)
    m = wg.newQuantMatrix(N, K)
    wg.packQ4_0(m, 4, blocks[: 4 * (K // 32) * 18], 4, perm)
    wg.packQ4_0(m, 8, blocks[8 * (K // 32) * 18:], N - 8)
    host = O.HostQuantMatrix(N, K)
    O.c_pack_q4_0(host, 4, blocks[: 4 * (K // 32) * 18], 4, perm)
    O.c_pack_q4_0(host, 8, blocks[8 * (K // 32) * 18:], N - 8)
    for n in range(N):
        assert np.array_equal(wg.matrixRow(m, n), O.c_matrix_row(host, n)), n
    # rows 0..3 were never written: weight 0
    assert not wg.matrixRow(m, 2).any()


def test_pack_errors_follow_the_reference():
    m = wg.newQuantMatrix(8, 64)
    with pytest.raises(wg.RangeError):
        wg.packQ4_0(m, 6, np.zeros(4 * 2 * 18, np.uint8), 4)
    with pytest.raises(wg.ShapeError, match="too short"):
        wg.packQ4_0(m, 0, np.zeros(4 * 2 * 18 - 1, np.uint8), 4)


def _nbits(N, K, seed):
    rng = np.random.default_rng(seed)
    blocks = K // 32
    quant = rng.integers(0, 256, N * blocks * 16, dtype=np.uint8)
    scales = (np.abs(rng.standard_normal(N * blocks)) * 0.02 / 8).astype(np.float16).view(np.uint8)
    zp = rng.integers(0, 256, N * ((blocks + 1) // 2), dtype=np.uint8)
    return quant, scales, zp


@pytest.mark.parametrize("N,K", [(8, 64), (20, 96), (64, 2048)])
def test_pack_matmulnbits_with_zero_points_round_trip(N, K):
    quant, scales, zp = _nbits(N, K, N + K)
    m = wg.newQuantMatrix(N, K, withZeros=True)
    wg.packMatMulNBits(m, 0, quant, scales, zp, N)
    host = O.HostQuantMatrix(N, K, with_zeros=True)
    O.c_pack_matmulnbits(host, 0, quant, scales, zp, N)
    for n in range(0, N, max(1, N // 9)):
        assert np.array_equal(wg.matrixRow(m, n), O.c_matrix_row(host, n)), n


def test_write_quantmatrix_round_trip():
    N, K = 36, 192
    quant, scales, zp = _nbits(N, K, 9)
    host = O.HostQuantMatrix(N, K, with_zeros=True)
    O.c_pack_matmulnbits(host, 0, quant, scales, zp, N)
    m = wg.newQuantMatrix(N, K, withZeros=True)
    wg.writeMatrix(m, host.quants, host.scales, host.zeros)
    for n in range(N):
        assert np.array_equal(wg.matrixRow(m, n), O.c_matrix_row(host, n)), n


# ---------------------------------------------------------------- decode GEMV


def test_config0_gemv_fp32():
    # x fp32 [1 x 2048] ~ N(0,1), W 2048 x 2048 Q4_0, seed 0.
    N = K = 2048
    blocks, m, host = make(N, K, 0)
    x = O.config_activations(1, K, 0)
    y, _ = run(m, x, torch.float32, torch.float32)
    check_close(y, O.c_ref_f64(blocks, x, N, K), "vs fp64")
    check_close(y, O.c_split_emulate(host, x), "vs shader emulation")


@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 7, 8, 9, 12, 16, 17, 24, 31, 32])
def test_gemv_rows(M):
    N, K = 512, 1024
    blocks, m, host = make(N, K, M)
    y, x16 = run(m, O.config_activations(M, K, M))
    check_close(y, O.c_ref_f64(blocks, x16, N, K), f"M={M} vs fp64")
    check_close(y, O.c_split_emulate(host, x16), f"M={M} vs emulation")


@pytest.mark.parametrize("N,K", [(4, 32), (12, 96), (20, 160), (36, 64), (100, 4096),
                                 (2560, 2048), (2048, 5632), (256, 14336), (4, 32768),
                                 # K in one CTA up to 128 tiles (formerly cluster splits)
                                 (1024, 2048), (512, 1600), (64, 3520), (1536, 4608), (128, 8192)])
def test_gemv_shapes(N, K):
    blocks, m, host = make(N, K, N + K)
    for M in (1, 5):
        y, x16 = run(m, O.config_activations(M, K, 3))
        check_close(y, O.c_ref_f64(blocks, x16, N, K), f"{N}x{K} M={M}")


_SPLIT_CHILD = """
import sys
sys.path.insert(0, sys.argv[1])
import torch, oracle as O, webgllm_b200 as wg
for N, K, M in [(1024, 2048, 1), (512, 1600, 2), (64, 3520, 1), (1536, 4608, 3), (256, 14336, 1), (4, 32768, 1)]:
    blocks = O.config_q4_0_blocks(N, K, N + K)
    m = wg.newQuantMatrix(N, K)
    wg.packQ4_0(m, 0, blocks, N)
    x = torch.from_numpy(O.config_activations(M, K, 3)).to("cuda", torch.float16)
    y = wg.matmul(x, m, out_dtype=torch.float32)
    torch.cuda.synchronize()
    l2, mx = O.rel_errors(y.cpu().numpy(), O.c_ref_f64(blocks, x.float().cpu().numpy(), N, K))
    assert l2 <= O.TOL and mx <= O.TOL, f"{N}x{K} M={M}: {l2:.3e} {mx:.3e}"
print("ok")
"""


def test_gemv_cluster_split_path():
    # The tile-column GEMV splits K over a thread-block cluster only where a
    # CTA's range does not fit (K > 8192 at one row); WG_GEMV_SPLIT_PCT=100
    # restores the split of small grids and WG_GEMV_WIDE=0 keeps every shape
    # on the tile-column kernel, so that the cluster reduction (including
    # clusters whose last CTA has a shorter range) stays checked. The
    # settings are read once per process: a child process runs the cases.
    import os
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent
    env = dict(os.environ, WG_GEMV_SPLIT_PCT="100", WG_GEMV_WIDE="0")
    r = subprocess.run([sys.executable, "-c", _SPLIT_CHILD, str(root)], env=env, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout[-2000:] + r.stderr[-2000:]


@pytest.mark.parametrize("M,N,K", [(1, 4096, 14336),   # one stage: a column at a time
                                   (8, 28672, 4096),   # three stages, ~12 columns a CTA
                                   (8, 6144, 4096), (4, 4096, 4096), (2, 20480, 2048),
                                   (3, 2560, 8192), (8, 4096, 14336)])  # the last: K split over a cluster
def test_wide_gemv_many_columns(M, N, K):
    # shapes where the wide GEMV's CTAs walk several tile columns through
    # their shared-memory stages (the two warp groups alternate columns)
    blocks, m, host = make(N, K, M * 7 + N)
    y, x16 = run(m, O.config_activations(M, K, 5))
    check_close(y, O.c_ref_f64(blocks, x16, N, K), f"{M}x{N}x{K} vs fp64")
    if N * K <= 4096 * 4096:
        check_close(y, O.c_split_emulate(host, x16), f"{M}x{N}x{K} vs emulation")


@pytest.mark.parametrize("xd", ["float32", "float16", "bfloat16"])
@pytest.mark.parametrize("yd", ["float32", "float16", "bfloat16"])
def test_gemv_dtypes(xd, yd):
    N, K = 256, 512
    blocks, m, host = make(N, K, 11)
    xt, yt = getattr(torch, xd), getattr(torch, yd)
    y, xq = run(m, O.config_activations(3, K, 11), xt, yt)
    ref = O.c_ref_f64(blocks, xq, N, K)
    if yd == "bfloat16":  # bf16 storage itself rounds at 2^-9
        l2, mx = O.rel_errors(y, ref)
        assert l2 <= 4e-3 and mx <= 4e-3
    else:
        check_close(y, ref, f"{xd}->{yd}")


def test_gemv_zero_points():
    N, K = 1024, 2048
    quant, scales, zp = _nbits(N, K, 4)
    m = wg.newQuantMatrix(N, K, withZeros=True)
    wg.packMatMulNBits(m, 0, quant, scales, zp, N)
    host = O.HostQuantMatrix(N, K, with_zeros=True)
    O.c_pack_matmulnbits(host, 0, quant, scales, zp, N)
    W = np.stack([O.c_matrix_row(host, n) for n in range(N)]).astype(np.float64)
    for M in (1, 6, 20):
        y, x16 = run(m, O.config_activations(M, K, M))
        check_close(y, x16.astype(np.float64) @ W.T, f"zeros M={M} vs fp64")
        check_close(y, O.c_split_emulate(host, x16), f"zeros M={M} vs emulation")


def test_fp16_output_saturates_like_packh2():
    # Scales of 64 and codes 15: |y| far above 65504 -> +-65504 (kernels.ts:32-36).
    N, K = 16, 256
    blk = np.zeros((N * K // 32, 18), np.uint8)
    blk[:, 0:2] = np.array([64.0], np.float16).view(np.uint8)
    blk[:, 2:] = 0xFF
    m = wg.newQuantMatrix(N, K)
    wg.packQ4_0(m, 0, blk.reshape(-1), N)
    x = np.full((1, K), 100.0, np.float32)
    y, _ = run(m, x, torch.float32, torch.float16)
    assert np.all(np.abs(y) == 65504.0)


def test_empty_batch_is_a_no_op():
    _, m, _ = make(16, 64, 1)
    x = torch.zeros((0, 64), device="cuda", dtype=torch.float16)
    y = wg.matmul(x, m)
    assert y.shape == (0, 16)


# ---------------------------------------------------------------- config 1 sweep


@pytest.mark.parametrize("s,M", list(enumerate([1, 4, 16, 64, 256, 1024])))
def test_config1_sweep(s, M):
    # K = N = 4096, x fp16 ~ N(0,1), seed s for shape s.
    N = K = 4096
    blocks, m, host = make(N, K, s)
    y, x16 = run(m, O.config_activations(M, K, s))
    ref = O.c_ref_f64(blocks, x16, N, K)
    check_close(y, ref, f"config 1 M={M} vs fp64")
    emul = O.c_split_emulate(host, x16) if M <= 8 else O.c_prefill_emulate(host, x16)
    check_close(y, emul, f"config 1 M={M} vs emulation")


# ---------------------------------------------------------------- prefill GEMM (tcgen05)


@pytest.mark.parametrize("M,N,K", [
    (33, 128, 128),      # smallest GEMM row count, one CTA
    (64, 128, 128),
    (64, 512, 4096),     # few tiles: K split across CTAs (a cluster, reduced on chip)
    (256, 4096, 4096),   # config 1's M = 256: a 4-way K split
    (65, 128, 256),      # second token tile, partial
    (129, 100, 96),      # N not a multiple of 128 (TMA fills), K % 64 == 32
    (300, 1024, 2048),
    (1024, 512, 512),    # few tiles: a 2-way K split
    (1024, 4096, 1024),  # K unsplit, 256 CTAs
    (520, 4144, 2080),   # the last weight tile partial (N % 128 = 48), K % 64 == 32
    (96, 2560, 2048),    # a q|k|v-shaped matrix
])
def test_gemm_parity(M, N, K):
    blocks, m, host = make(N, K, M + N + K)
    y, x16 = run(m, O.config_activations(M, K, M))
    check_close(y, O.c_ref_f64(blocks, x16, N, K), f"GEMM {M}x{N}x{K} vs fp64")
    check_close(y, O.c_prefill_emulate(host, x16), f"GEMM {M}x{N}x{K} vs f16 route")


@pytest.mark.parametrize("M,N", [(100, 256), (600, 4096)])  # K split / unsplit
def test_gemm_zero_points(M, N):
    K = 1024
    quant, scales, zp = _nbits(N, K, 8)
    m = wg.newQuantMatrix(N, K, withZeros=True)
    wg.packMatMulNBits(m, 0, quant, scales, zp, N)
    host = O.HostQuantMatrix(N, K, with_zeros=True)
    O.c_pack_matmulnbits(host, 0, quant, scales, zp, N)
    W = np.stack([O.c_matrix_row(host, n) for n in range(N)]).astype(np.float64)
    y, x16 = run(m, O.config_activations(M, K, 5))
    check_close(y, x16.astype(np.float64) @ W.T, "GEMM zeros vs fp64")


@pytest.mark.parametrize("xd,yd", [("float32", "float16"), ("bfloat16", "float32"), ("float16", "bfloat16")])
def test_gemm_dtypes(xd, yd):
    N, K, M = 384, 512, 70
    blocks, m, host = make(N, K, 21)
    y, xq = run(m, O.config_activations(M, K, 2), getattr(torch, xd), getattr(torch, yd))
    ref = O.c_ref_f64(blocks, xq, N, K)
    tol = 4e-3 if yd == "bfloat16" else TOL
    l2, mx = O.rel_errors(y, ref)
    assert l2 <= tol and mx <= tol, f"{xd}->{yd}: {l2:.2e} {mx:.2e}"


def test_gemm_repeated_calls_are_deterministic():
    N, K, M = 512, 1024, 256
    _, m, _ = make(N, K, 3)
    x = torch.from_numpy(O.config_activations(M, K, 3)).to("cuda", torch.float16)
    a = wg.matmul(x, m, out_dtype=torch.float32)
    b = wg.matmul(x, m, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_gemm_pair_kernel_parity():
    """The 2-SM (cta_group::2) GEMM, opt-in through WG_GEMM_PAIR=1 (read once
    per process, hence a child process): the same products as the fp32
    product of the dequantised weights within the suite's two measures (rel
    L2 and max |error| / max |ref| <= 1e-3)."""
    import subprocess
    import sys

    code = r'''
import sys, torch
sys.path.insert(0, ".")
import webgllm_b200 as wg
from webgllm_b200.model import quantize_q4_0, dequantize_q4_0
c = wg.context(); c.use_torch_stream()
worst = worst_max = 0.0
for (M, N, K) in [(256, 256, 256), (300, 512, 1024), (1024, 4096, 4096), (77, 768, 2048)]:
    g = torch.Generator(device="cuda"); g.manual_seed(M + N + K)
    w = torch.randn((N, K), generator=g, device="cuda") * 0.02
    bl = quantize_q4_0(w)
    m = wg.newQuantMatrix(N, K); wg.packQ4_0(m, 0, bl, N)
    x = torch.randn((M, K), generator=g, device="cuda").half()
    y = wg.matmul(x, m, out_dtype=torch.float32)
    c.sync()
    ref = x.float() @ dequantize_q4_0(bl, N, K).t()
    worst = max(worst, ((y - ref).norm() / ref.norm()).item())
    worst_max = max(worst_max, ((y - ref).abs().max() / ref.abs().max()).item())
print(worst, worst_max)
'''
    import os

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, WG_GEMM_PAIR="1")
    out = subprocess.run([sys.executable, "-c", code], cwd=root, env=env, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    l2, mx = map(float, out.stdout.strip().splitlines()[-1].split())
    assert l2 <= TOL and mx <= TOL, f"pair kernel: l2 {l2:.3e} max {mx:.3e}"


# ---------------------------------------------------------------- recorded steps (wg_graph_*)


def test_recorded_step_replays_the_calls():
    # A recorded sequence of matmuls (GEMV rows, wide GEMV rows and the GEMM,
    # as a decode step mixes them) replays to the same bytes as the same calls
    # made one by one, reading the inputs' current contents at every replay.
    import ctypes

    from webgllm_b200 import _lib

    L = _lib.lib()
    cases = []
    for i, (M, N, K) in enumerate([(1, 4096, 4096), (8, 2048, 4096), (64, 512, 4096)]):
        _, m, _ = make(N, K, 40 + i)
        x = torch.empty((M, K), device="cuda", dtype=torch.float16)
        cases.append((m, x, torch.empty((M, N), device="cuda"), torch.empty((M, N), device="cuda")))
    ctx = cases[0][0].ctx
    h = ctypes.c_void_p(ctx.handle)
    ctx.set_stream(None)  # the context's own stream (torch's default one is the legacy stream)

    def calls(into):
        for m, x, ya, yb in cases:
            y = ya if into == 0 else yb
            _lib.check(L.wg_q4_matmul(h, ctypes.c_void_p(m.handle), ctypes.c_void_p(x.data_ptr()), _lib.WG_F16,
                                      x.shape[0], ctypes.c_void_p(y.data_ptr()), _lib.WG_F32), ctx.handle)

    try:
        for _, x, _, _ in cases:
            x.zero_()
        torch.cuda.synchronize()
        calls(0)  # first calls of each kind outside the recording
        _lib.check(L.wg_sync(h), ctx.handle)
        g = ctypes.c_void_p()
        _lib.check(L.wg_graph_begin(h), ctx.handle)
        calls(1)
        _lib.check(L.wg_graph_end(h, ctypes.byref(g)), ctx.handle)
        assert g.value
        try:
            for rep in range(2):
                for j, (_, x, _, _) in enumerate(cases):
                    x.copy_(torch.from_numpy(O.config_activations(x.shape[0], x.shape[1], 10 * rep + j)))
                torch.cuda.synchronize()
                calls(0)
                _lib.check(L.wg_graph_launch(h, g), ctx.handle)
                _lib.check(L.wg_sync(h), ctx.handle)
                for m, x, ya, yb in cases:
                    assert torch.equal(ya, yb), f"replay {rep}, M={x.shape[0]}"
                    assert ya.abs().max().item() > 0
        finally:
            _lib.check(L.wg_graph_free(h, g), ctx.handle)
        # A call that waits spoils a recording; the end reports it, returns no
        # graph, and the context works on.
        _lib.check(L.wg_graph_begin(h), ctx.handle)
        assert L.wg_sync(h) != _lib.WG_OK
        g2 = ctypes.c_void_p()
        assert L.wg_graph_end(h, ctypes.byref(g2)) == _lib.WG_CUDA_ERROR and not g2.value
        assert b"recording failed" in L.wg_last_error(h)
        calls(0)
        _lib.check(L.wg_sync(h), ctx.handle)
    finally:
        ctx.use_torch_stream()
