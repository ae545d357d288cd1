"""Failure detection on the GPU without a fault: a GEMM whose copy producer
withholds one k-block (qmm_debug_gemm_stall) has its bounded waits run out
after a short limit.  The launch ends by itself, having drained its copies and
MMAs and freed its tensor memory; qmm_device_error reports QMM_ERR_TIMEOUT;
and the next normal launch on the same context is bit-identical to one made
before.  (The reference surfaces failures as `candle_core::Error`s,
src/quant.rs:438-451; the device-side waits have no counterpart there.)"""
import ctypes

import numpy as np
import pytest
import torch

from qmm_testutil import from_dev_bf16, make_linear, random_layer, sin_input, to_dev_u16
from qwen_imager_b200 import _lib, device_error

pytestmark = pytest.mark.gpu

TIMEOUT_CODES = {1, 2, 3, 4, 5}  # producer, dequant, MMA, epilogue, drain


def _layer(m, k, n, bits, seed):
    packed, scales, offsets, bias = random_layer(n, k, bits, 64, seed=seed, bias=True)
    return make_linear(packed, scales, offsets, bias, bits, 64), to_dev_u16(sin_input(m, k))


@pytest.mark.parametrize("m,k,n,bits,withhold,residual", [
    (1024, 3072, 3072, 4, 2, False),    # one tile per CTA, stalls in its first tile
    (1024, 3072, 3072, 8, 0, False),    # nothing issued at all
    (4096, 3072, 3072, 4, 100, True),   # stalls in a CTA's third tile, residual chunks in flight
])
def test_gemm_wait_expiry_is_reported_and_the_context_recovers(m, k, n, bits, withhold, residual):
    lib = _lib.load()
    lin, x = _layer(m, k, n, bits, seed=m + withhold)
    res = to_dev_u16(sin_input(m, n)) if residual else None
    assert device_error() == 0
    before = lin.forward_fused(x, residual=res, path=_lib.QMM_PATH_GEMM, splits=1)
    torch.cuda.synchronize()
    assert device_error() == 0
    _lib.check(lib.qmm_debug_gemm_stall(withhold, 50_000_000))  # 50 ms wait limit
    try:
        y = torch.zeros((m, n), dtype=torch.bfloat16, device="cuda")
        lin.forward_fused(x, residual=res, path=_lib.QMM_PATH_GEMM, splits=1, out=y)
        code = ctypes.c_uint32()
        status = lib.qmm_device_error(torch.cuda.current_stream().cuda_stream, ctypes.byref(code))
        assert status == _lib.QMM_ERR_TIMEOUT, status
        assert code.value in TIMEOUT_CODES, code.value
        assert b"device-side wait expired" in lib.qmm_last_error()
    finally:
        _lib.check(lib.qmm_debug_gemm_stall(-1, 0))
    assert device_error() == 0  # read and cleared
    after = lin.forward_fused(x, residual=res, path=_lib.QMM_PATH_GEMM, splits=1)
    torch.cuda.synchronize()
    assert device_error() == 0
    assert np.array_equal(from_dev_bf16(after), from_dev_bf16(before))


def test_stall_hook_rejects_out_of_range_limits():
    lib = _lib.load()
    assert lib.qmm_debug_gemm_stall(-2, 0) == _lib.QMM_ERR_INVALID_ARGUMENT
    assert lib.qmm_debug_gemm_stall(1, 1000) == _lib.QMM_ERR_INVALID_ARGUMENT  # under 1 ms
    assert lib.qmm_debug_gemm_stall(1, 5_000_000_000) == _lib.QMM_ERR_INVALID_ARGUMENT  # over 4 s
    _lib.check(lib.qmm_debug_gemm_stall(-1, 0))
