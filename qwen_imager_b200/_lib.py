"""ctypes binding of libqmm.so (include/qmm.h).

This is the same binding a foreign host language would write against the C ABI:
plain structs, raw device pointers, a stream handle.  The library is built
in-tree (qwen_imager_b200/_build/libqmm.so); if it is missing and nvcc is
available it is built on first use, otherwise loading fails with QmmError.
There is no CPU implementation behind it.
"""
from __future__ import annotations

import ctypes
import os
import threading

from . import build as _build

QMM_OK = 0
QMM_ERR_INVALID_ARGUMENT = 1
QMM_ERR_BAD_SHAPE = 2
QMM_ERR_UNSUPPORTED = 3
QMM_ERR_MISALIGNED = 4
QMM_ERR_CUDA = 5
QMM_ERR_TIMEOUT = 6

STATUS_NAMES = {
    QMM_OK: "QMM_OK",
    QMM_ERR_INVALID_ARGUMENT: "QMM_ERR_INVALID_ARGUMENT",
    QMM_ERR_BAD_SHAPE: "QMM_ERR_BAD_SHAPE",
    QMM_ERR_UNSUPPORTED: "QMM_ERR_UNSUPPORTED",
    QMM_ERR_MISALIGNED: "QMM_ERR_MISALIGNED",
    QMM_ERR_CUDA: "QMM_ERR_CUDA",
    QMM_ERR_TIMEOUT: "QMM_ERR_TIMEOUT",
}

QMM_DTYPE_BF16 = 0
QMM_DTYPE_F32 = 1

QMM_ACT_NONE = 0
QMM_ACT_GELU_TANH = 1
QMM_ACT_SILU = 2

QMM_PATH_AUTO = 0
QMM_PATH_GEMV = 1
QMM_PATH_GEMM = 2
QMM_PATH_GEMM_PAIR = 3
QMM_PATH_GEMM_F16 = 4

QMM_EPILOGUE_RESIDUAL_MUL = 0x100

# Every symbol include/qmm.h declares.
EXPORTED_SYMBOLS = (
    "qmm_abi_version",
    "qmm_last_error",
    "qmm_infer_layout",
    "qmm_validate",
    "qmm_dequantize",
    "qmm_linear",
    "qmm_linear_ex",
    "qmm_device_error",
    "qmm_launch_count",
    "qmm_gemm_splits",
    "qmm_splitk_workspace_bytes",
    "qmm_linear_splitk",
    "qmm_linear_splitk_static",
    "qmm_layernorm_modulate",
    "qmm_residual_layernorm_modulate",
    "qmm_set_sm_budget",
    "qmm_static_scratch_bytes",
    "qmm_binary_version",
    "qmm_debug_gemm_stall",
    "qmm_set_weights_immutable",
    "qmm_tp_signal_ready",
    "qmm_tp_reduce_norm_gather",
    "qmm_tp_wait_gathered",
)


class QmmError(RuntimeError):
    """A non-OK qmm_status, with the library's message."""

    def __init__(self, status: int, message: str):
        self.status = status
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")


class QmmWeight(ctypes.Structure):
    _fields_ = [
        ("packed", ctypes.c_void_p),
        ("scales", ctypes.c_void_p),
        ("biases", ctypes.c_void_p),
        ("n", ctypes.c_int64),
        ("k", ctypes.c_int64),
        ("bits", ctypes.c_int32),
        ("group", ctypes.c_int32),
    ]


class QmmEpilogue(ctypes.Structure):
    _fields_ = [
        ("bias", ctypes.c_void_p),
        ("gate", ctypes.c_void_p),
        ("residual", ctypes.c_void_p),
        ("activation", ctypes.c_int32),
    ]


QMM_TP_MAX_RANKS = 8


class QmmTpPeers(ctypes.Structure):
    _fields_ = [
        ("world", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("part", ctypes.c_void_p * QMM_TP_MAX_RANKS),
        ("gathered", ctypes.c_void_p * QMM_TP_MAX_RANKS),
        ("counters", ctypes.c_void_p * QMM_TP_MAX_RANKS),
    ]


class QmmTpNorm(ctypes.Structure):
    _fields_ = [
        ("bias", ctypes.c_void_p * 2),
        ("gate", ctypes.c_void_p * 2),
        ("shift", ctypes.c_void_p * 2),
        ("scale", ctypes.c_void_p * 2),
        ("split", ctypes.c_int64),
        ("eps", ctypes.c_float),
    ]


_lock = threading.Lock()
_lib = None


def library_path() -> str:
    return _build.LIB


def load() -> ctypes.CDLL:
    """Loads libqmm.so (building it first when stale and nvcc exists)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if _build.is_stale():
            try:
                _build.build()
            except Exception as exc:  # no nvcc, or a compile error
                if not os.path.exists(_build.LIB):
                    raise QmmError(QMM_ERR_CUDA, f"libqmm.so is not built and cannot be built: {exc}")
        if not os.path.exists(_build.LIB):
            raise QmmError(QMM_ERR_CUDA, f"libqmm.so not found at {_build.LIB}")
        lib = ctypes.CDLL(_build.LIB)
        vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32
        wp = ctypes.POINTER(QmmWeight)
        ep = ctypes.POINTER(QmmEpilogue)
        lib.qmm_abi_version.restype = i32
        lib.qmm_abi_version.argtypes = []
        lib.qmm_last_error.restype = ctypes.c_char_p
        lib.qmm_last_error.argtypes = []
        lib.qmm_launch_count.restype = ctypes.c_uint64
        lib.qmm_launch_count.argtypes = []
        lib.qmm_infer_layout.restype = i32
        lib.qmm_infer_layout.argtypes = [i64, i64, i64, i64, i64, i64,
                                         ctypes.POINTER(i32), ctypes.POINTER(i32)]
        lib.qmm_validate.restype = i32
        lib.qmm_validate.argtypes = [wp]
        lib.qmm_dequantize.restype = i32
        lib.qmm_dequantize.argtypes = [wp, vp, i32, vp]
        lib.qmm_linear.restype = i32
        lib.qmm_linear.argtypes = [wp, vp, i64, ep, vp, vp]
        lib.qmm_linear_ex.restype = i32
        lib.qmm_linear_ex.argtypes = [wp, vp, i64, ep, vp, i32, vp]
        lib.qmm_gemm_splits.restype = i32
        lib.qmm_gemm_splits.argtypes = [wp, i64]
        lib.qmm_splitk_workspace_bytes.restype = ctypes.c_uint64
        lib.qmm_splitk_workspace_bytes.argtypes = [wp, i64, i32]
        lib.qmm_linear_splitk.restype = i32
        lib.qmm_linear_splitk.argtypes = [wp, vp, i64, ep, vp, i32, vp, ctypes.c_uint64, vp]
        lib.qmm_set_sm_budget.restype = i32
        lib.qmm_set_sm_budget.argtypes = [i32]
        lib.qmm_layernorm_modulate.restype = i32
        lib.qmm_layernorm_modulate.argtypes = [vp, i64, i64, vp, vp, ctypes.c_float, vp, vp]
        lib.qmm_residual_layernorm_modulate.restype = i32
        lib.qmm_residual_layernorm_modulate.argtypes = [vp, i64, i64, vp, vp, vp, vp, vp, ctypes.c_float, vp, vp]
        lib.qmm_linear_splitk_static.restype = i32
        lib.qmm_linear_splitk_static.argtypes = [wp, vp, i64, ep, vp, i32, vp]
        lib.qmm_static_scratch_bytes.restype = ctypes.c_uint64
        lib.qmm_static_scratch_bytes.argtypes = []
        tpp, tpn = ctypes.POINTER(QmmTpPeers), ctypes.POINTER(QmmTpNorm)
        lib.qmm_tp_signal_ready.restype = i32
        lib.qmm_tp_signal_ready.argtypes = [tpp, vp]
        lib.qmm_tp_reduce_norm_gather.restype = i32
        lib.qmm_tp_reduce_norm_gather.argtypes = [tpp, ctypes.c_uint64, i64, i64, vp, tpn, i32, i32, vp]
        lib.qmm_tp_wait_gathered.restype = i32
        lib.qmm_tp_wait_gathered.argtypes = [tpp, ctypes.c_uint64, vp]
        lib.qmm_set_weights_immutable.restype = i32
        lib.qmm_set_weights_immutable.argtypes = [i32]
        lib.qmm_debug_gemm_stall.restype = i32
        lib.qmm_debug_gemm_stall.argtypes = [i32, ctypes.c_uint64]
        lib.qmm_binary_version.restype = i32
        lib.qmm_binary_version.argtypes = [ctypes.POINTER(i32), ctypes.POINTER(i32)]
        lib.qmm_device_error.restype = i32
        lib.qmm_device_error.argtypes = [vp, ctypes.POINTER(ctypes.c_uint32)]
        _lib = lib
        return lib


def check(status: int) -> None:
    if status != QMM_OK:
        msg = load().qmm_last_error().decode(errors="replace")
        raise QmmError(status, msg)


def launch_count() -> int:
    return int(load().qmm_launch_count())


def infer_layout(input: int, output: int, scales_shape, packed_shape):
    bits, group = ctypes.c_int32(), ctypes.c_int32()
    check(load().qmm_infer_layout(input, output, scales_shape[0], scales_shape[1],
                                  packed_shape[0], packed_shape[1],
                                  ctypes.byref(bits), ctypes.byref(group)))
    return bits.value, group.value
