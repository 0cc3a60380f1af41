"""CPU oracle for the Q4 matmul path. TEST INFRASTRUCTURE ONLY.

Two restatements of webgllm's 4-bit matmul arithmetic, used to check the CUDA
library and to time a CPU baseline:

* ``q4_oracle.c`` (built by ``oracle/Makefile`` into ``oracle/_build``), called
  through ctypes by the ``c_*`` functions here;
* numpy mirrors (``np_*``) of the same functions, written independently, used
  to cross-check the C at small sizes.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s cpu_baseline /
reference legs import this package, as the checker or as the timed CPU
baseline. The product (``webgllm_b200``) never imports it.

Reference citations are paths inside the webgllm package (packages/webgllm/).
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"

_lib = None


def build() -> Path:
    """Compile q4_oracle.c with the committed Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        build()
    L = ctypes.CDLL(str(LIB_PATH))
    P = ctypes.c_void_p
    i32, sz, f = ctypes.c_int, ctypes.c_size_t, ctypes.c_float
    L.orc_to_half.argtypes = [f]
    L.orc_to_half.restype = ctypes.c_uint16
    L.orc_to_half_bench.argtypes = [f]
    L.orc_to_half_bench.restype = ctypes.c_uint16
    L.orc_from_half.argtypes = [ctypes.c_uint16]
    L.orc_from_half.restype = f
    L.orc_check_shape.argtypes = [i32, i32]
    L.orc_pack_q4_0.argtypes = [i32, i32, P, P, i32, P, sz, i32, P]
    L.orc_pack_matmulnbits.argtypes = [i32, i32, P, P, P, i32, P, sz, P, sz, P, sz, i32, P]
    L.orc_quants_from_raw.argtypes = [P, i32, i32, P]
    L.orc_quants_from_raw.restype = None
    L.orc_matrix_row.argtypes = [i32, i32, P, P, P, i32, P]
    L.orc_matrix_row.restype = None
    L.orc_q4_ref_f64.argtypes = [P, P, i32, i32, i32, P, i32]
    L.orc_q4_ref_f64.restype = None
    L.orc_split_slices.argtypes = [i32, i32, P, P]
    L.orc_split_slices.restype = None
    L.orc_quad_slices.argtypes = [i32, i32, P, P]
    L.orc_quad_slices.restype = None
    L.orc_q4_split_emulate.argtypes = [i32, i32, P, P, P, P, i32, P, i32]
    L.orc_q4_split_emulate.restype = None
    L.orc_q4_prefill_emulate.argtypes = [i32, i32, P, P, P, P, i32, P, i32]
    L.orc_q4_prefill_emulate.restype = None
    L.orc_quantize_q4_0.argtypes = [P, i32, i32, P]
    L.orc_quantize_q4_0.restype = None
    L.orc_max_threads.restype = i32
    _lib = L
    return L


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


class OracleError(ValueError):
    """A status code from the C oracle (values as include/webgllm_q4.h)."""

    MESSAGES = {
        1: "invalid argument",
        2: "invalid shape: N must be a multiple of 4 and K of 32",
        3: "rows are outside the matrix",
        4: "data is too short",
    }

    def __init__(self, code: int):
        super().__init__(self.MESSAGES.get(code, f"oracle status {code}"))
        self.code = code


# --------------------------------------------------------------------------
# QuantMatrix (src/weights.ts:153-178) as host arrays


class HostQuantMatrix:
    """The reference's QuantMatrix for 4-bit weights, on the host.

    ``quants`` u32 words ((g*blocks + b)*4 + r)*4 + w, ``scales`` fp16 bits
    (g*blocks + b)*4 + r, ``zeros`` u8 or None (8 everywhere), as
    src/weights.ts:5-21 lays them out.
    """

    def __init__(self, N: int, K: int, with_zeros: bool = False):
        st = lib().orc_check_shape(N, K)
        if st:
            raise OracleError(st)
        self.N, self.K, self.bits = N, K, 4
        blocks = K // 32
        self.quants = np.zeros(N * blocks * 4, dtype=np.uint32)
        self.scales = np.zeros(N * blocks, dtype=np.uint16)
        self.zeros = np.full(N * blocks, 8, dtype=np.uint8) if with_zeros else None


def c_to_half(v: float) -> int:
    return int(lib().orc_to_half(float(v)))


def c_to_half_bench(v: float) -> int:
    return int(lib().orc_to_half_bench(float(v)))


def c_from_half(h: int) -> float:
    return float(lib().orc_from_half(int(h) & 0xFFFF))


def c_pack_q4_0(m: HostQuantMatrix, row0: int, src: np.ndarray, rows: int, src_rows=None) -> None:
    """src/repack.ts:60-87."""
    src = np.ascontiguousarray(src, dtype=np.uint8)
    perm = None if src_rows is None else np.ascontiguousarray(src_rows, dtype=np.int32)
    st = lib().orc_pack_q4_0(m.N, m.K, _p(m.quants), _p(m.scales), row0, _p(src), src.nbytes, rows, _p(perm))
    if st:
        raise OracleError(st)


def c_pack_matmulnbits(m: HostQuantMatrix, row0: int, quant, scale_bytes, zp, rows: int, src_rows=None) -> None:
    """src/repack.ts:342-392."""
    quant = np.ascontiguousarray(quant, dtype=np.uint8)
    scale_bytes = np.ascontiguousarray(scale_bytes, dtype=np.uint8)
    zp_a = None if zp is None else np.ascontiguousarray(zp, dtype=np.uint8)
    perm = None if src_rows is None else np.ascontiguousarray(src_rows, dtype=np.int32)
    st = lib().orc_pack_matmulnbits(
        m.N, m.K, _p(m.quants), _p(m.scales), _p(m.zeros), row0,
        _p(quant), quant.nbytes, _p(scale_bytes), scale_bytes.nbytes,
        _p(zp_a), 0 if zp_a is None else zp_a.nbytes, rows, _p(perm))
    if st:
        raise OracleError(st)


def c_quants_from_raw(raw: np.ndarray, N: int, K: int) -> np.ndarray:
    """src/repack.ts:216-242."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    out = np.zeros(N * (K // 32) * 4, dtype=np.uint32)
    lib().orc_quants_from_raw(_p(raw), N, K, _p(out))
    return out


def c_matrix_row(m: HostQuantMatrix, n: int) -> np.ndarray:
    """src/repack.ts:865-891."""
    out = np.zeros(m.K, dtype=np.float32)
    lib().orc_matrix_row(m.N, m.K, _p(m.quants), _p(m.scales), _p(m.zeros), n, _p(out))
    return out


def c_ref_f64(blocks: np.ndarray, act: np.ndarray, N: int, K: int, threads: int = 0) -> np.ndarray:
    """bench/gpu-bench-worker.js:41-55: fp64 sums from GGUF Q4_0 blocks."""
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    act = np.ascontiguousarray(act, dtype=np.float32).reshape(-1, K)
    M = act.shape[0]
    out = np.zeros((M, N), dtype=np.float64)
    lib().orc_q4_ref_f64(_p(blocks), _p(act), M, N, K, _p(out), threads)
    return out


def split_slices(N: int, K: int) -> tuple[int, int]:
    """src/engine.ts:5316-5327 (kbSlice, slices) of the decode split matmul."""
    a, b = ctypes.c_int(), ctypes.c_int()
    lib().orc_split_slices(N, K, ctypes.byref(a), ctypes.byref(b))
    return a.value, b.value


def quad_slices(N: int, K: int) -> tuple[int, int]:
    """src/engine.ts:4957-4967 (kbSlice, slices) of the prompt matmul."""
    a, b = ctypes.c_int(), ctypes.c_int()
    lib().orc_quad_slices(N, K, ctypes.byref(a), ctypes.byref(b))
    return a.value, b.value


def c_split_emulate(m: HostQuantMatrix, act: np.ndarray, threads: int = 0) -> np.ndarray:
    """The decode matmul as the reference's shader computes it (fp16
    activations, fp32 block sums, fp16 K-slice partials)."""
    act = np.ascontiguousarray(act, dtype=np.float32).reshape(-1, m.K)
    M = act.shape[0]
    out = np.zeros((M, m.N), dtype=np.float32)
    lib().orc_q4_split_emulate(m.N, m.K, _p(m.quants), _p(m.scales), _p(m.zeros), _p(act), M, _p(out), threads)
    return out


def c_prefill_emulate(m: HostQuantMatrix, act: np.ndarray, threads: int = 0) -> np.ndarray:
    """The prompt matmul's f16 route (fp16 weights and activations, fp32
    slice sums, fp16 slice outputs)."""
    act = np.ascontiguousarray(act, dtype=np.float32).reshape(-1, m.K)
    M = act.shape[0]
    out = np.zeros((M, m.N), dtype=np.float32)
    lib().orc_q4_prefill_emulate(m.N, m.K, _p(m.quants), _p(m.scales), _p(m.zeros), _p(act), M, _p(out), threads)
    return out


def c_quantize_q4_0(w: np.ndarray) -> np.ndarray:
    """Float rows to GGUF Q4_0 blocks (the llama.cpp Q4_0 rule)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, K = w.shape
    out = np.zeros(N * (K // 32) * 18, dtype=np.uint8)
    lib().orc_quantize_q4_0(_p(w), N, K, _p(out))
    return out


def max_threads() -> int:
    return int(lib().orc_max_threads())


# --------------------------------------------------------------------------
# numpy mirrors (independent restatements, for cross-checking the C)


def np_from_half(h: np.ndarray) -> np.ndarray:
    return np.asarray(h, dtype=np.uint16).view(np.float16).astype(np.float32)


def np_pack_q4_0(N: int, K: int, src: np.ndarray, src_rows=None):
    """src/repack.ts:60-87 for a whole matrix: (quants u32, scales u16)."""
    blocks = K // 32
    b = np.asarray(src, dtype=np.uint8)[: N * blocks * 18].reshape(N, blocks, 18)
    if src_rows is not None:
        b = b[np.asarray(src_rows)]
    scales = b[:, :, 0].astype(np.uint16) | (b[:, :, 1].astype(np.uint16) << 8)
    nib = np.ascontiguousarray(b[:, :, 2:]).view(np.uint32).reshape(N, blocks, 4)
    # (g, r, b, w) -> (g, b, r, w)
    q = nib.reshape(N // 4, 4, blocks, 4).transpose(0, 2, 1, 3).reshape(-1)
    s = scales.reshape(N // 4, 4, blocks).transpose(0, 2, 1).reshape(-1)
    return np.ascontiguousarray(q), np.ascontiguousarray(s)


def np_matrix_row(N: int, K: int, quants: np.ndarray, scales: np.ndarray, zeros, n: int) -> np.ndarray:
    """src/repack.ts:865-891."""
    blocks = K // 32
    g, r = n >> 2, n & 3
    qb = quants.view(np.uint8).reshape(N // 4, blocks, 4, 16)[g, :, r, :]
    lo = (qb & 15).astype(np.float32)
    hi = (qb >> 4).astype(np.float32)
    s = np_from_half(scales.reshape(N // 4, blocks, 4)[g, :, r])
    z = 8.0 if zeros is None else zeros.reshape(N // 4, blocks, 4)[g, :, r].astype(np.float32)[:, None]
    w = np.concatenate([lo, hi], axis=1)
    return (s[:, None] * (w - z)).reshape(-1).astype(np.float32)


def np_dequant_gguf(blocks: np.ndarray, N: int, K: int) -> np.ndarray:
    """All weights of GGUF Q4_0 blocks as float64 (d * (q - 8))."""
    kb = K // 32
    b = np.asarray(blocks, dtype=np.uint8)[: N * kb * 18].reshape(N, kb, 18)
    d = np_from_half(b[:, :, 0].astype(np.uint16) | (b[:, :, 1].astype(np.uint16) << 8)).astype(np.float64)
    q = b[:, :, 2:]
    w = np.concatenate([(q & 15), (q >> 4)], axis=2).astype(np.float64) - 8.0
    return (w * d[:, :, None]).reshape(N, K)


def np_ref_f64(blocks: np.ndarray, act: np.ndarray, N: int, K: int) -> np.ndarray:
    """bench/gpu-bench-worker.js:41-55, vectorised (summation order differs
    from the C; agreement is to fp64 rounding)."""
    W = np_dequant_gguf(blocks, N, K)
    return np.asarray(act, dtype=np.float64).reshape(-1, K) @ W.T


def mulberry32(seed: int):
    """bench/gpu-bench-worker.js:18-27: the bench's seeded generator."""
    a = seed & 0xFFFFFFFF

    def rand() -> float:
        nonlocal a
        a = (a + 0x6D2B79F5) & 0xFFFFFFFF
        t = a
        t = _imul(t ^ (t >> 15), t | 1)
        t ^= (t + _imul(t ^ (t >> 7), t | 61)) & 0xFFFFFFFF
        return ((t ^ (t >> 14)) & 0xFFFFFFFF) / 4294967296.0

    return rand


def _imul(a: int, b: int) -> int:
    return (a * b) & 0xFFFFFFFF


def bench_random_q4_0(N: int, K: int, rand) -> np.ndarray:
    """bench/gpu-bench-worker.js:30-39: random Q4_0 blocks, scales
    toHalf(0.004 + rand() * 0.02) with the bench's toHalf."""
    nb = N * (K // 32)
    out = np.zeros(nb * 18, dtype=np.uint8)
    for b in range(nb):
        h = c_to_half_bench(np.float32(0.004 + rand() * 0.02))
        out[b * 18] = h & 255
        out[b * 18 + 1] = h >> 8
        for j in range(16):
            out[b * 18 + 2 + j] = int(rand() * 256) & 255
    return out


# --------------------------------------------------------------------------
# Synthetic inputs of the BASELINE configs (numpy default_rng, seeded)


def config_q4_0_blocks(N: int, K: int, seed: int) -> np.ndarray:
    """Config 0/1 weights: per block d = fp16(|N(0,1)| * 0.02 / 8), codes
    uniform on 0..15, packed GGUF style (byte j: w[j] low, w[j+16] high)."""
    rng = np.random.default_rng(seed)
    nb = N * (K // 32)
    d = (np.abs(rng.standard_normal(nb)) * 0.02 / 8).astype(np.float16)
    q = rng.integers(0, 16, size=(nb, 32), dtype=np.uint8)
    out = np.zeros((nb, 18), dtype=np.uint8)
    out[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    out[:, 2:] = q[:, :16] | (q[:, 16:] << 4)
    return out.reshape(-1)


def config_activations(M: int, K: int, seed: int, dtype=np.float32) -> np.ndarray:
    rng = np.random.default_rng(seed + 1_000_003)
    return rng.standard_normal((M, K)).astype(dtype)


def rel_errors(y: np.ndarray, ref: np.ndarray) -> tuple[float, float]:
    """(||y - ref||_2 / ||ref||_2, max|y - ref| / max|ref|): the two parity
    measures, both of which must be <= 1e-3."""
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    nref = float(np.linalg.norm(ref))
    mref = float(np.max(np.abs(ref))) if ref.size else 0.0
    if ref.size == 0:
        return 0.0, 0.0
    l2 = float(np.linalg.norm(y - ref)) / (nref if nref > 0 else 1.0)
    mx = float(np.max(np.abs(y - ref))) / (mref if mref > 0 else 1.0)
    return l2, mx


TOL = 1e-3  # rel 1e-3 on matmul outputs
