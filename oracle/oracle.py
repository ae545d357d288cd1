"""ORACLE -- test infrastructure, not product code.

Python access to the CPU restatement of image-forger's quantized-linear path
(oracle/qmm_oracle.c) plus an independent numpy twin of its dequantization.
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module; the qwen_imager_b200 package never does.

bf16 arrays are numpy uint16 holding raw bf16 bits; packed weights are uint32.

Reference algorithm (paths relative to the reference repository):
  src/quant.rs:555-573   dequantize (f32 arithmetic, bf16 by round-to-nearest-even)
  src/quant.rs:105-113   forward_f32: f32 W, f32 x, f32 GEMM, f32 bias
  src/quant.rs:119       result cast to bf16
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libqmm_oracle.so")
_lock = threading.Lock()
_lib = None

_u16p = ctypes.POINTER(ctypes.c_uint16)
_u32p = ctypes.POINTER(ctypes.c_uint32)
_f32p = ctypes.POINTER(ctypes.c_float)
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32


def build() -> str:
    """Compiles oracle/qmm_oracle.c with oracle/Makefile; returns the .so path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    with _lock:
        if _lib is None:
            src = os.path.join(_HERE, "qmm_oracle.c")
            if (not os.path.exists(_LIB_PATH)
                    or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src)):
                build()
            l = ctypes.CDLL(_LIB_PATH)
            l.oracle_dequantize_f32.argtypes = [_u32p, _u16p, _u16p, _i64, _i64, _i32, _i32, _f32p]
            l.oracle_dequantize_bf16.argtypes = [_u32p, _u16p, _u16p, _i64, _i64, _i32, _i32, _u16p]
            l.oracle_matmul_f32.argtypes = [_f32p, _f32p, _u16p, _i64, _i64, _i64, _f32p]
            l.oracle_epilogue_bf16.argtypes = [_f32p, _u16p, _u16p, _i32, _i64, _i64, _u16p]
            l.oracle_bf16_from_f32_array.argtypes = [_f32p, _u16p, _i64]
            l.oracle_f32_from_bf16_array.argtypes = [_u16p, _f32p, _i64]
            l.oracle_set_threads.argtypes = [_i32]
            l.oracle_get_threads.restype = _i32
            _lib = l
    return _lib


def _p(a: np.ndarray, t):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(t)


def _opt(a, t):
    return None if a is None else _p(a, t)


def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.uint16)
    return (a.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    """Round to nearest even (half::bf16::from_f32)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty(a.shape, dtype=np.uint16)
    lib().oracle_bf16_from_f32_array(_p(a, _f32p), _p(out, _u16p), a.size)
    return out


def dequantize_f32(packed, scales, biases, bits: int, group: int) -> np.ndarray:
    packed = np.ascontiguousarray(packed, dtype=np.uint32)
    n = packed.shape[0]
    k = packed.shape[1] * 32 // bits
    out = np.empty((n, k), dtype=np.float32)
    lib().oracle_dequantize_f32(_p(packed, _u32p), _p(np.ascontiguousarray(scales), _u16p),
                                _p(np.ascontiguousarray(biases), _u16p), n, k, bits, group,
                                _p(out, _f32p))
    return out


def dequantize_bf16(packed, scales, biases, bits: int, group: int) -> np.ndarray:
    packed = np.ascontiguousarray(packed, dtype=np.uint32)
    n = packed.shape[0]
    k = packed.shape[1] * 32 // bits
    out = np.empty((n, k), dtype=np.uint16)
    lib().oracle_dequantize_bf16(_p(packed, _u32p), _p(np.ascontiguousarray(scales), _u16p),
                                 _p(np.ascontiguousarray(biases), _u16p), n, k, bits, group,
                                 _p(out, _u16p))
    return out


def dequantize_numpy(packed, scales, biases, bits: int, group: int) -> np.ndarray:
    """Independent numpy twin of src/quant.rs:555-573 returning bf16 bits."""
    packed = np.asarray(packed, dtype=np.uint32)
    n, words = packed.shape
    per_word = 32 // bits
    k = words * per_word
    shifts = (np.arange(per_word, dtype=np.uint32) * bits)[None, None, :]
    q = ((packed[:, :, None] >> shifts) & np.uint32((1 << bits) - 1)).reshape(n, k)
    g = np.arange(k) // group
    s = bf16_to_f32(scales)[:, g]
    o = bf16_to_f32(biases)[:, g]
    w = (s * q.astype(np.float32)).astype(np.float32) + o
    return _f32_to_bf16_numpy(w.astype(np.float32))


def _f32_to_bf16_numpy(a: np.ndarray) -> np.ndarray:
    """Round to nearest even, written independently of the C oracle (finite inputs)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    return ((u + (((u >> 16) & 1) + 0x7FFF)) >> 16).astype(np.uint16)


def matmul_f32(x_f32: np.ndarray, w_f32: np.ndarray, bias=None) -> np.ndarray:
    x_f32 = np.ascontiguousarray(x_f32, dtype=np.float32)
    w_f32 = np.ascontiguousarray(w_f32, dtype=np.float32)
    m, k = x_f32.shape
    n = w_f32.shape[0]
    y = np.empty((m, n), dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.uint16)
    lib().oracle_matmul_f32(_p(x_f32, _f32p), _p(w_f32, _f32p), _opt(b, _u16p), m, n, k,
                            _p(y, _f32p))
    return y


def linear_f32(x_bf16, packed, scales, biases, bits: int, group: int, bias=None) -> np.ndarray:
    """`Linear::forward_f32` (src/quant.rs:105-113): f32 result [m, n]."""
    x = bf16_to_f32(np.asarray(x_bf16, dtype=np.uint16).reshape(-1, np.asarray(x_bf16).shape[-1]))
    w = dequantize_f32(packed, scales, biases, bits, group)
    return matmul_f32(x, w, bias)


def linear_bf16(x_bf16, packed, scales, biases, bits: int, group: int, bias=None) -> np.ndarray:
    """The reference CPU forward: forward_f32 then cast to bf16 (src/quant.rs:119)."""
    return f32_to_bf16(linear_f32(x_bf16, packed, scales, biases, bits, group, bias))


def epilogue_bf16(y_f32, gate=None, residual=None, activation: int = 0) -> np.ndarray:
    """residual + gate * act(y_f32), f32 arithmetic, one rounding to bf16."""
    y_f32 = np.ascontiguousarray(y_f32, dtype=np.float32)
    m, n = y_f32.shape
    out = np.empty((m, n), dtype=np.uint16)
    g = None if gate is None else np.ascontiguousarray(gate, dtype=np.uint16)
    r = None if residual is None else np.ascontiguousarray(residual, dtype=np.uint16)
    lib().oracle_epilogue_bf16(_p(y_f32, _f32p), _opt(g, _u16p), _opt(r, _u16p), activation,
                               m, n, _p(out, _u16p))
    return out


def quantize_affine(w_f32: np.ndarray, bits: int, group: int = 64):
    """Affine group quantizer with the formula the benchmark configurations state:
    per group, scale = (max - min) / (2^bits - 1), bias = min, both stored bf16,
    q = clamp(round((w - bias) / scale), 0, 2^bits - 1), codes packed
    little-end-first into uint32 words.  Returns (packed, scales, biases)."""
    w = np.asarray(w_f32, dtype=np.float32)
    n, k = w.shape
    levels = (1 << bits) - 1
    wg = w.reshape(n, k // group, group)
    lo = wg.min(axis=2)
    hi = wg.max(axis=2)
    scale_b = f32_to_bf16(((hi - lo) / levels).astype(np.float32))
    bias_b = f32_to_bf16(lo)
    s = bf16_to_f32(scale_b)[:, :, None]
    b = bf16_to_f32(bias_b)[:, :, None]
    safe = np.where(s == 0, 1.0, s)
    q = np.clip(np.rint((wg - b) / safe), 0, levels).astype(np.uint32).reshape(n, k)
    per_word = 32 // bits
    q = q.reshape(n, k // per_word, per_word)
    shifts = (np.arange(per_word, dtype=np.uint32) * bits)[None, None, :]
    packed = np.bitwise_or.reduce(q << shifts, axis=2).astype(np.uint32)
    return packed, scale_b, bias_b


def reference_forward_cpu(x_bf16, packed, scales, biases, bits: int, group: int, bias=None,
                          threads: int = 0) -> np.ndarray:
    """The reference's CPU forward as it runs per call (src/quant.rs:105-113, 119):
    re-dequantize W to f32 (row-parallel, like rayon's par_chunks_mut), x to f32,
    f32 GEMM plus f32 bias, cast to bf16.  The f32 GEMM of Candle's third-party
    `gemm` crate is stood in for by torch's multi-threaded CPU matmul.
    Used as the timed CPU baseline; returns bf16 bits."""
    import torch

    if threads:
        lib().oracle_set_threads(threads)
        torch.set_num_threads(threads)
    w = torch.from_numpy(dequantize_f32(packed, scales, biases, bits, group))
    x = torch.from_numpy(bf16_to_f32(np.asarray(x_bf16, dtype=np.uint16)))
    y = x @ w.T
    if bias is not None:
        y = y + torch.from_numpy(bf16_to_f32(np.asarray(bias, dtype=np.uint16)))
    return f32_to_bf16(y.numpy())
