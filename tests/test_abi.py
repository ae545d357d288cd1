"""The C-ABI library builds for sm_100a, loads, and exports every symbol that
include/qmm.h declares; host-only entry points validate like `Linear::load`
(src/quant.rs:43-77).  No compute calls: this file needs no GPU."""
import ctypes
import os
import re

import pytest

from qwen_imager_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "qmm.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^QMM_API\s+(?:const\s+)?\w+\s+\*?\s*(qmm_\w+)\s*\(", text, re.M)))


def test_header_declares_the_binding_table():
    assert declared_symbols() == sorted(_lib.EXPORTED_SYMBOLS)


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.qmm_abi_version() == 2


@pytest.mark.gpu
def test_library_device_code_is_sm100():
    # The runtime's own report for one of the library's kernels
    # (cudaFuncGetAttributes): built for compute capability 10.0.
    lib = _lib.load()
    binary, ptx = ctypes.c_int32(), ctypes.c_int32()
    _lib.check(lib.qmm_binary_version(ctypes.byref(binary), ctypes.byref(ptx)))
    assert binary.value == 100 and ptx.value == 100, (binary.value, ptx.value)


@pytest.mark.parametrize("input,output,scales,packed,expect", [
    (192, 96, (96, 3), (96, 24), (4, 64)),
    (192, 96, (96, 3), (96, 48), (8, 64)),
    (4096, 1024, (1024, 128), (1024, 256), (2, 32)),
    (3072, 18432, (18432, 48), (18432, 384), (4, 64)),
])
def test_infer_layout_accepts_mlx_packs(input, output, scales, packed, expect):
    assert _lib.infer_layout(input, output, scales, packed) == expect


@pytest.mark.parametrize("input,output,scales,packed", [
    (128, 96, (96, 3), (96, 24)),   # groups do not divide the input
    (192, 96, (96, 3), (96, 20)),   # truncated packing (reference test, src/quant.rs:804-806)
    (192, 96, (95, 3), (96, 24)),   # scales rows
    (192, 96, (96, 0), (96, 24)),   # no groups
    (192, 96, (96, 3), (96, 18)),   # 3-bit
    (192, 96, (96, 3), (96, 96)),   # 16-bit
])
def test_infer_layout_rejects_bad_packing(input, output, scales, packed):
    with pytest.raises(_lib.QmmError) as e:
        _lib.infer_layout(input, output, scales, packed)
    assert e.value.status == _lib.QMM_ERR_BAD_SHAPE


def test_validate_rejects_null_and_misaligned_weights():
    lib = _lib.load()
    w = _lib.QmmWeight(None, None, None, 96, 192, 4, 64)
    assert lib.qmm_validate(ctypes.byref(w)) == _lib.QMM_ERR_INVALID_ARGUMENT
    assert b"null" in lib.qmm_last_error()
    w = _lib.QmmWeight(0x1008, 0x2000, 0x3000, 96, 192, 4, 64)
    assert lib.qmm_validate(ctypes.byref(w)) == _lib.QMM_ERR_MISALIGNED
    w = _lib.QmmWeight(0x1000, 0x2000, 0x3000, 96, 192, 3, 64)
    assert lib.qmm_validate(ctypes.byref(w)) == _lib.QMM_ERR_BAD_SHAPE
    w = _lib.QmmWeight(0x1000, 0x2000, 0x3000, 96, 192, 4, 50)
    assert lib.qmm_validate(ctypes.byref(w)) == _lib.QMM_ERR_BAD_SHAPE
    w = _lib.QmmWeight(0x1000, 0x2000, 0x3000, 96, 192, 4, 64)
    assert lib.qmm_validate(ctypes.byref(w)) == _lib.QMM_OK
    assert lib.qmm_validate(None) == _lib.QMM_ERR_INVALID_ARGUMENT


def test_compute_entry_points_fail_loudly_without_a_device():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    lib = _lib.load()
    w = _lib.QmmWeight(0x1000, 0x2000, 0x3000, 96, 192, 4, 64)
    st = lib.qmm_linear(ctypes.byref(w), 0x4000, 5, None, 0x8000, None)
    assert st == _lib.QMM_ERR_CUDA
    st = lib.qmm_dequantize(ctypes.byref(w), 0x8000, 0, None)
    assert st == _lib.QMM_ERR_CUDA


def test_splitk_workspace_size_and_argument_checks_without_a_device():
    from qwen_imager_b200 import _lib
    lib = _lib.load()
    import ctypes
    w = _lib.QmmWeight(16, 16, 16, 96, 640, 4, 64)
    assert lib.qmm_splitk_workspace_bytes(ctypes.byref(w), 8, 2) == 2 * 8 * 96 * 4
    assert lib.qmm_splitk_workspace_bytes(ctypes.byref(w), 8, 1) == 0
    # split count outside [1, 16] and a null workspace are argument errors, found before any device access
    assert lib.qmm_linear_splitk(ctypes.byref(w), 16, 8, None, 1 << 20, 0, 0, 0, None) == _lib.QMM_ERR_INVALID_ARGUMENT
    assert lib.qmm_linear_splitk(ctypes.byref(w), 16, 8, None, 1 << 20, 2, 0, 0, None) == _lib.QMM_ERR_INVALID_ARGUMENT
