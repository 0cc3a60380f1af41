"""ctypes binding of libwebgllm_b200.so (include/webgllm_q4.h).

The library is the product: there is no fallback. If the shared object is
missing, importing the binding raises, with the command that builds it.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libwebgllm_b200.so"

# include/webgllm_q4.h: enum wg_status, enum wg_dtype
WG_OK = 0
WG_INVALID_ARGUMENT = 1
WG_INVALID_SHAPE = 2
WG_OUT_OF_RANGE = 3
WG_DATA_TOO_SHORT = 4
WG_OUT_OF_MEMORY = 5
WG_CUDA_ERROR = 6
WG_TIMEOUT = 7
WG_DEVICE_LOST = 8
WG_UNSUPPORTED = 9
WG_NO_DEVICE = 10

WG_F32, WG_F16, WG_BF16 = 0, 1, 2
WG_PRO_RMSNORM, WG_PRO_SWIGLU = 1, 2
WG_EPI_SWIGLU_PAIRS = 1
WG_OPT_EXACT_ROWS = 1


class wg_prologue(ctypes.Structure):
    """include/webgllm_q4.h wg_prologue."""
    _fields_ = [("kind", ctypes.c_int), ("a", ctypes.c_void_p), ("b", ctypes.c_void_p),
                ("weight", ctypes.c_void_p), ("eps", ctypes.c_float), ("resid_out", ctypes.c_void_p),
                ("stats", ctypes.c_void_p)]

_P = ctypes.c_void_p
_I = ctypes.c_int
_SZ = ctypes.c_size_t
_PP = ctypes.POINTER(ctypes.c_void_p)

# name -> (restype, argtypes), in the header's order
SIGNATURES = {
    "wg_init": (_I, [_I, _PP]),
    "wg_destroy": (_I, [_P]),
    "wg_set_stream": (_I, [_P, _P]),
    "wg_set_option": (_I, [_P, _I, _I]),
    "wg_alloc": (_I, [_P, _SZ, _PP]),
    "wg_free": (_I, [_P, _P]),
    "wg_host_alloc": (_I, [_P, _SZ, _PP]),
    "wg_host_free": (_I, [_P, _P]),
    "wg_upload": (_I, [_P, _P, _P, _SZ]),
    "wg_read": (_I, [_P, _P, _P, _SZ]),
    "wg_sync": (_I, [_P]),
    "wg_q4_new": (_I, [_P, _I, _I, _I, _PP]),
    "wg_q4_free": (_I, [_P, _P]),
    "wg_q4_info": (_I, [_P, ctypes.POINTER(_I), ctypes.POINTER(_I), ctypes.POINTER(_SZ)]),
    "wg_q4_pack_q4_0": (_I, [_P, _P, _I, _P, _SZ, _I, _P]),
    "wg_q4_pack_nbits": (_I, [_P, _P, _I, _P, _SZ, _P, _SZ, _P, _SZ, _I, _P]),
    "wg_q4_write_quantmatrix": (_I, [_P, _P, _P, _P, _P]),
    "wg_q4_matrix_row": (_I, [_P, _P, _I, _P]),
    "wg_q4_matmul": (_I, [_P, _P, _P, _I, _I, _P, _I]),
    "wg_q4_matmul_static": (_I, [_P, _P, _P, _I, _I, _P, _I]),
    "wg_q4_matmul_fused": (_I, [_P, _P, _P, _I, _P, _I]),
    "wg_q4_matmul_ex": (_I, [_P, _P, _P, _P, _I, _I, _P, _I, _I]),
    "wg_q4_matmul_residual": (_I, [_P, _P, _P, _P, _I, _I, _P, _P]),
    "wg_trace": (_I, [_P, _P, _SZ]),
    "wg_trace_count": (_I, [_P, ctypes.POINTER(_SZ)]),
    "wg_graph_begin": (_I, [_P]),
    "wg_graph_end": (_I, [_P, _PP]),
    "wg_graph_launch": (_I, [_P, _P]),
    "wg_graph_free": (_I, [_P, _P]),
    # include/webgllm_decoder.h
    "wg_embed": (_I, [_P, _P, _I, _P, _I, _I, _P]),
    "wg_rmsnorm": (_I, [_P, _P, _P, _P, ctypes.c_float, _I, _I, _P, _I]),
    "wg_rope_kv": (_I, [_P, _P, _I, _I, _I, _I, _I, _P, ctypes.c_float, _P, _P, ctypes.c_float, _P, _P, _P, _I]),
    "wg_attention": (_I, [_P, _P, _I, _I, _I, _I, _I, _P, _P, _I, _P, _P]),
    "wg_rope_attention": (_I, [_P, _P, _I, _I, _I, _I, _P, ctypes.c_float, _P, _P, ctypes.c_float, _P, _P, _I, _P]),
    "wg_swiglu": (_I, [_P, _P, _I, _I, _P, _I]),
    "wg_swiglu_pairs": (_I, [_P, _P, _I, _I, _P, _I]),
    "wg_short_conv": (_I, [_P, _P, _I, _I, _I, _I, _P, _P, _P, _I]),
    "wg_short_conv_prefixes": (_I, [_P, _P, _I, _I, _I, _I, _P, _P, _P, _I, _P, _I, _I]),
    "wg_conv_restore": (_I, [_P, _P, _I, _I, _I, _I, _P, _P, _P]),
    "wg_head": (_I, [_P, _P, _I, _I, _P, _I, _P, _P]),
    "wg_head_rmsnorm": (_I, [_P, _P, _P, _P, ctypes.c_float, _I, _I, _I, _P, _I, _I, _P, _P, _P]),
    "wg_pick_keys": (_I, [_P, _P, _I, _P]),
    "wg_argmax": (_I, [_P, _P, _I, _I, _P]),
    "wg_add_i32": (_I, [_P, _P, _I, _I]),
    "wg_spec_accept": (_I, [_P, _P, _P, _I, _I, _P, _P, _P, _P, _P, _I, _P, _P]),
    # include/webgllm_comm.h
    "wg_ipc_alloc": (_I, [_P, _SZ, _PP, _P]),
    "wg_ipc_free": (_I, [_P, _P]),
    "wg_ipc_open": (_I, [_P, _P, _PP]),
    "wg_ipc_close": (_I, [_P, _P]),
    "wg_comm_init": (_I, [_P, _I, _I, _P, _SZ, _PP]),
    "wg_comm_destroy": (_I, [_P, _P]),
    "wg_comm_set_wait": (_I, [_P, ctypes.c_ulonglong]),
    "wg_comm_slot": (_I, [_P, ctypes.POINTER(_SZ)]),
    "wg_q4_matmul_push": (_I, [_P, _P, _P, _P, _I, _I, _P]),
    "wg_comm_reduce": (_I, [_P, _P, _I, _I, _P]),
    "wg_comm_reduce_norm": (_I, [_P, _P, _I, _I, _P, _P, ctypes.c_float, _P, _P]),
    "wg_tp_unique_id": (_I, [_P]),
    "wg_tp_init": (_I, [_P, _I, _I, _P, _PP]),
    "wg_tp_destroy": (_I, [_P, _P]),
    "wg_tp_info": (_I, [_P, ctypes.POINTER(_I), ctypes.POINTER(_I)]),
    "wg_tp_allreduce": (_I, [_P, _P, _P, _SZ, _I, _I]),
    "wg_tp_barrier": (_I, [_P, _P, _I]),
    "wg_tp_comm": (_I, [_P, _P, _SZ, _PP]),
    "wg_error_string": (ctypes.c_char_p, [_I]),
    "wg_last_error": (ctypes.c_char_p, [_P]),
}

_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """The loaded library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m webgllm_b200.build` "
                "(the Q4 path has no CPU fallback)")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


class GpuError(RuntimeError):
    """A failed library call (the reference's GpuError, src/gpu/types.ts:14)."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


class RangeError(GpuError, IndexError):
    """Rows outside the matrix (src/repack.ts:52-53 throws RangeError)."""


class ShapeError(GpuError, ValueError):
    """N % 4 or K % 32, or data too short (src/repack.ts:21-24, :69)."""


def error_for(code: int, message: str) -> GpuError:
    if code == WG_OUT_OF_RANGE:
        return RangeError(code, message)
    if code in (WG_INVALID_SHAPE, WG_DATA_TOO_SHORT):
        return ShapeError(code, message)
    return GpuError(code, message)


def check(status: int, ctx: int | None = None) -> None:
    if status == WG_OK:
        return
    L = lib()
    detail = L.wg_last_error(ctx).decode() if ctx else ""
    name = L.wg_error_string(status).decode()
    raise error_for(status, detail or name)
