"""The reference's 4-bit matmul interface, over the B200 library.

Names, arguments and errors follow webgllm (paths inside packages/webgllm/):

* ``newQuantMatrix(N, K, bits, withZeros)``: src/repack.ts:14-35, the matrix
  now lives on the device (the engine's allocateMatrix, src/engine.ts:2381);
* ``packQ4_0(m, row0, src, rows, srcRows)``: src/repack.ts:60-87;
* ``packMatMulNBits(m, row0, quant, scaleBytes, zp, rows, srcRows)``:
  src/repack.ts:342-392;
* ``writeMatrix(m, quants, scales, zeros)``: src/engine.ts:3355, for a
  QuantMatrix already packed on the host (src/weights.ts:5-21);
* ``matrixRow(m, n)``: src/repack.ts:865-891;
* ``project(a, w, out, rows)`` / ``matmul(...)``: src/engine.ts:4677 and
  :4969, out = a . w^T.

Every call goes through libwebgllm_b200.so (include/webgllm_q4.h); device
buffers are torch CUDA tensors, and the library runs on torch's current
stream so that its work is ordered with the caller's.
"""
from __future__ import annotations

import ctypes
import threading

import numpy as np

from . import _lib
from ._lib import WG_BF16, WG_F16, WG_F32, GpuError, RangeError, ShapeError, check

__all__ = [
    "Context", "QuantMatrix", "newQuantMatrix", "packQ4_0", "packMatMulNBits",
    "writeMatrix", "matrixRow", "project", "matmul", "GpuError", "RangeError", "ShapeError",
]


class Context:
    """One device and one stream (the reference's Gpu, src/gpu/gl.ts:108)."""

    def __init__(self, device: int = 0):
        self.device = device
        h = ctypes.c_void_p()
        check(_lib.lib().wg_init(device, ctypes.byref(h)))
        self.handle = h.value

    def close(self) -> None:
        if self.handle:
            _lib.lib().wg_destroy(self.handle)
            self.handle = None

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass

    def _check(self, status: int) -> None:
        check(status, self.handle)

    def use_torch_stream(self) -> None:
        import torch

        s = torch.cuda.current_stream(self.device).cuda_stream
        # torch's default stream is the legacy NULL stream; NULL would select
        # the context's own (non-blocking, unordered) stream, so name the
        # legacy stream by its handle, cudaStreamLegacy.
        self._check(_lib.lib().wg_set_stream(self.handle, ctypes.c_void_p(s if s else _CUDA_STREAM_LEGACY)))

    def set_stream(self, stream: int | None) -> None:
        self._check(_lib.lib().wg_set_stream(self.handle, ctypes.c_void_p(stream or 0)))

    def set_option(self, option: int, value: int) -> None:
        """wg_set_option (e.g. WG_OPT_EXACT_ROWS)."""
        self._check(_lib.lib().wg_set_option(self.handle, option, value))

    def sync(self) -> None:
        self._check(_lib.lib().wg_sync(self.handle))

    # raw memory (the C ABI's own buffers, for callers without torch)
    def alloc(self, nbytes: int) -> int:
        p = ctypes.c_void_p()
        self._check(_lib.lib().wg_alloc(self.handle, nbytes, ctypes.byref(p)))
        return p.value

    def free(self, ptr: int) -> None:
        self._check(_lib.lib().wg_free(self.handle, ctypes.c_void_p(ptr)))

    def host_alloc(self, nbytes: int) -> int:
        p = ctypes.c_void_p()
        self._check(_lib.lib().wg_host_alloc(self.handle, nbytes, ctypes.byref(p)))
        return p.value

    def host_free(self, ptr: int) -> None:
        self._check(_lib.lib().wg_host_free(self.handle, ctypes.c_void_p(ptr)))

    def upload(self, dst: int, src: int, nbytes: int) -> None:
        self._check(_lib.lib().wg_upload(self.handle, ctypes.c_void_p(dst), ctypes.c_void_p(src), nbytes))

    def read(self, host: int, src: int, nbytes: int) -> None:
        self._check(_lib.lib().wg_read(self.handle, ctypes.c_void_p(host), ctypes.c_void_p(src), nbytes))


_CUDA_STREAM_LEGACY = 1  # cudaStreamLegacy

_contexts: dict[int, Context] = {}
_ctx_lock = threading.Lock()


def context(device: int | None = None) -> Context:
    """The per-device default context."""
    if device is None:
        import torch

        device = torch.cuda.current_device()
    with _ctx_lock:
        ctx = _contexts.get(device)
        if ctx is None:
            ctx = _contexts[device] = Context(device)
        return ctx


class QuantMatrix:
    """A 4-bit matrix on the device (the reference's QuantMatrix,
    src/weights.ts:153-178, with bits 4): N rows of K weights, each
    scale * (q - zero) of its 32-weight block."""

    def __init__(self, ctx: Context, handle: int, N: int, K: int, with_zeros: bool):
        self.ctx, self.handle = ctx, handle
        self.N, self.K, self.bits = N, K, 4
        self.with_zeros = with_zeros

    @property
    def device_bytes(self) -> int:
        n, k, b = ctypes.c_int(), ctypes.c_int(), ctypes.c_size_t()
        check(_lib.lib().wg_q4_info(ctypes.c_void_p(self.handle), ctypes.byref(n), ctypes.byref(k), ctypes.byref(b)))
        return b.value

    def free(self) -> None:
        if self.handle:
            self.ctx._check(_lib.lib().wg_q4_free(self.ctx.handle, ctypes.c_void_p(self.handle)))
            self.handle = None

    def __del__(self):  # pragma: no cover
        try:
            self.free()
        except Exception:
            pass


def _u8(a) -> np.ndarray:
    return np.ascontiguousarray(np.frombuffer(memoryview(a).cast("B"), dtype=np.uint8)
                                if not isinstance(a, np.ndarray) else a.view(np.uint8).reshape(-1))


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def newQuantMatrix(N: int, K: int, bits: int = 4, withZeros: bool = False, ctx: Context | None = None) -> QuantMatrix:
    """src/repack.ts:14-35 on the device (every weight starts at 0)."""
    if bits != 4:
        raise GpuError(_lib.WG_UNSUPPORTED, f"only 4-bit matrices run on the B200 path (got {bits})")
    # src/repack.ts:21-24, before touching a device
    if N % 4 != 0:
        raise ShapeError(_lib.WG_INVALID_SHAPE, f"matrix rows ({N}) must be a multiple of 4")
    if K % 32 != 0:
        raise ShapeError(_lib.WG_INVALID_SHAPE, f"matrix columns ({K}) must be a multiple of 32")
    ctx = ctx or context()
    ctx.use_torch_stream() if _torch_ready() else None
    h = ctypes.c_void_p()
    ctx._check(_lib.lib().wg_q4_new(ctx.handle, N, K, 1 if withZeros else 0, ctypes.byref(h)))
    return QuantMatrix(ctx, h.value, N, K, withZeros)


def packQ4_0(m: QuantMatrix, row0: int, src, rows: int, srcRows=None) -> None:
    """src/repack.ts:60-87: `rows` rows of Q4_0 blocks into rows
    [row0, row0 + rows) of m; srcRows[i] names destination row i's source.
    `src` is host bytes or a contiguous uint8 CUDA tensor (read in place)."""
    perm = None if srcRows is None else np.ascontiguousarray(np.asarray(srcRows, dtype=np.int32))
    if getattr(src, "is_cuda", False):
        if not src.is_contiguous():
            raise GpuError(_lib.WG_INVALID_ARGUMENT, "device Q4_0 source must be contiguous")
        nbytes = src.numel() * src.element_size()
        m.ctx._check(_lib.lib().wg_q4_pack_q4_0(m.ctx.handle, ctypes.c_void_p(m.handle), row0,
                                                ctypes.c_void_p(src.data_ptr()), nbytes, rows, _ptr(perm)))
        return
    s = _u8(src)
    m.ctx._check(_lib.lib().wg_q4_pack_q4_0(m.ctx.handle, ctypes.c_void_p(m.handle), row0, _ptr(s), s.nbytes, rows, _ptr(perm)))


def packMatMulNBits(m: QuantMatrix, row0: int, quant, scaleBytes, zp, rows: int, srcRows=None) -> None:
    """src/repack.ts:342-392 (onnxruntime MatMulNBits, bits 4, block 32)."""
    q, sb = _u8(quant), _u8(scaleBytes)
    z = None if zp is None else _u8(zp)
    perm = None if srcRows is None else np.ascontiguousarray(np.asarray(srcRows, dtype=np.int32))
    m.ctx._check(_lib.lib().wg_q4_pack_nbits(
        m.ctx.handle, ctypes.c_void_p(m.handle), row0, _ptr(q), q.nbytes, _ptr(sb), sb.nbytes,
        _ptr(z), 0 if z is None else z.nbytes, rows, _ptr(perm)))


def writeMatrix(m: QuantMatrix, quants: np.ndarray, scales: np.ndarray, zeros: np.ndarray | None = None) -> None:
    """src/engine.ts:3355 for a host QuantMatrix (src/weights.ts:5-21)."""
    blocks = m.N * (m.K // 32)
    q = np.ascontiguousarray(quants, dtype=np.uint32)
    s = np.ascontiguousarray(scales, dtype=np.uint16)
    if q.size < blocks * 4 or s.size < blocks:
        raise ShapeError(_lib.WG_DATA_TOO_SHORT, "QuantMatrix data is too short")
    z = None if zeros is None else np.ascontiguousarray(zeros, dtype=np.uint8)
    if z is not None and z.size < blocks:
        raise ShapeError(_lib.WG_DATA_TOO_SHORT, "QuantMatrix zeros are too short")
    m.ctx._check(_lib.lib().wg_q4_write_quantmatrix(m.ctx.handle, ctypes.c_void_p(m.handle), _ptr(q), _ptr(s), _ptr(z)))


def matrixRow(m: QuantMatrix, n: int) -> np.ndarray:
    """src/repack.ts:865-891: row n as floats, read back from the device."""
    out = np.zeros(m.K, dtype=np.float32)
    m.ctx._check(_lib.lib().wg_q4_matrix_row(m.ctx.handle, ctypes.c_void_p(m.handle), n, _ptr(out)))
    return out


_DTYPES = None


def _dtype_code(t) -> int:
    global _DTYPES
    import torch

    if _DTYPES is None:
        _DTYPES = {torch.float32: WG_F32, torch.float16: WG_F16, torch.bfloat16: WG_BF16}
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise GpuError(_lib.WG_INVALID_ARGUMENT, f"unsupported dtype {t.dtype}") from None


def _torch_ready() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False


def matmul(a, w: QuantMatrix, out=None, rows: int | None = None, out_dtype=None):
    """out = a . w^T (src/engine.ts:4969) for `rows` rows of a (default all).

    a: CUDA tensor [rows, K] (float32 / float16 / bfloat16); out: CUDA tensor
    [rows, N] or None (allocated, dtype out_dtype, default a's). Returns out.
    """
    import torch

    rows = a.shape[0] if rows is None else rows
    if a.dim() != 2 or a.shape[1] != w.K:
        raise ShapeError(_lib.WG_INVALID_SHAPE, f"activations {tuple(a.shape)} do not match K = {w.K}")
    if not a.is_contiguous():
        a = a.contiguous()
    if out is None:
        out = torch.empty((rows, w.N), dtype=out_dtype or a.dtype, device=a.device)
    if out.shape[0] < rows or out.shape[1] != w.N or not out.is_contiguous():
        raise ShapeError(_lib.WG_INVALID_SHAPE, f"output {tuple(out.shape)} does not hold {rows} x {w.N}")
    ctx = w.ctx
    ctx.use_torch_stream()
    ctx._check(_lib.lib().wg_q4_matmul(ctx.handle, ctypes.c_void_p(w.handle), ctypes.c_void_p(a.data_ptr()),
                                       _dtype_code(a), rows, ctypes.c_void_p(out.data_ptr()), _dtype_code(out)))
    return out


def project(a, w: QuantMatrix, out=None, rows: int | None = None):
    """src/engine.ts:4677: the same product; the reference's split/prompt
    choice by row count is made inside the library."""
    return matmul(a, w, out, rows)
