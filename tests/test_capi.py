"""The C ABI library without a GPU: it loads, exports every entry point
include/webgllm_q4.h declares, and the host-side checks behave as the
reference's (src/repack.ts:21-24) before any device is touched."""
import ctypes
import re
from pathlib import Path

import pytest

from webgllm_b200 import _lib
import webgllm_b200 as wg

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    names = []
    for h in sorted((ROOT / "include").glob("*.h")):
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names += re.findall(r"^\s*(?:int|const char \*|void)\s*\*?\s*(wg_\w+)\s*\(", text, flags=re.M)
    return names


def test_header_declares_the_abi():
    names = declared_symbols()
    assert "wg_q4_matmul" in names and "wg_q4_pack_q4_0" in names
    assert len(names) == len(set(names))


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    for name in declared_symbols():
        assert hasattr(L, name), name
    # and the binding covers them all
    assert set(declared_symbols()) <= set(_lib.SIGNATURES)


def test_error_strings():
    L = _lib.lib()
    assert L.wg_error_string(0) == b"ok"
    assert L.wg_error_string(_lib.WG_DEVICE_LOST) == b"the GPU context was lost"
    assert L.wg_error_string(_lib.WG_OUT_OF_MEMORY) == b"out of memory"
    assert L.wg_error_string(12345) == b"unknown status"


def test_null_arguments_are_rejected_without_a_device():
    L = _lib.lib()
    assert L.wg_init(0, None) == _lib.WG_INVALID_ARGUMENT
    assert L.wg_destroy(None) == _lib.WG_INVALID_ARGUMENT
    assert L.wg_sync(None) == _lib.WG_INVALID_ARGUMENT
    assert L.wg_q4_matmul(None, None, None, 0, 1, None, 0) == _lib.WG_INVALID_ARGUMENT
    assert L.wg_q4_info(None, None, None, None) == _lib.WG_INVALID_ARGUMENT
    assert L.wg_graph_begin(None) == _lib.WG_INVALID_ARGUMENT
    assert L.wg_graph_end(None, None) == _lib.WG_INVALID_ARGUMENT
    assert L.wg_graph_launch(None, None) == _lib.WG_INVALID_ARGUMENT
    assert L.wg_graph_free(None, None) == _lib.WG_INVALID_ARGUMENT
    assert L.wg_last_error(None) == b""


def test_init_reports_a_missing_device_as_a_status():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = ctypes.c_void_p()
    assert _lib.lib().wg_init(0, ctypes.byref(h)) == _lib.WG_NO_DEVICE
    assert not h.value


@pytest.mark.parametrize("N,K,msg", [(6, 64, "matrix rows (6) must be a multiple of 4"),
                                     (8, 48, "matrix columns (48) must be a multiple of 32")])
def test_new_quant_matrix_shape_errors(N, K, msg):
    with pytest.raises(wg.ShapeError, match=re.escape(msg)):
        wg.newQuantMatrix(N, K)


def test_only_4_bit_matrices():
    with pytest.raises(wg.GpuError):
        wg.newQuantMatrix(8, 64, bits=8)


def test_error_classes():
    e = _lib.error_for(_lib.WG_OUT_OF_RANGE, "rows 6..10 are outside the matrix")
    assert isinstance(e, IndexError) and isinstance(e, wg.GpuError)
    assert isinstance(_lib.error_for(_lib.WG_DATA_TOO_SHORT, "x"), ValueError)


def test_tensor_parallel_group_id_without_a_gpu():
    """wg_tp_unique_id loads NCCL (libnccl.so.2) on first use and needs no
    device: the id a host sends to every rank of a group."""
    from webgllm_b200.comm import unique_id

    a, b = unique_id(), unique_id()
    assert len(a) == 128 and a != b
    L = _lib.lib()
    assert L.wg_tp_unique_id(None) == _lib.WG_INVALID_ARGUMENT
    assert L.wg_tp_init(None, 2, 0, ctypes.create_string_buffer(128), ctypes.byref(ctypes.c_void_p())) \
        == _lib.WG_INVALID_ARGUMENT
