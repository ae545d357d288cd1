"""The no-allocation split-K entry point (qmm_linear_splitk_static), for
callers that cannot call cudaMalloc (plug-ins whose host owns all device
memory, paths that must not synchronize the device), against the
caller-workspace entry point (qmm_linear_splitk): the same kernels give the
same results on two calls in a row through the shared static scratch, and
requests beyond the scratch's 16 MiB are refused.  Both paths run the same
kernels in the same summation order, so their outputs must be bit-identical;
the scratch is first left holding another shape's partials, so that a
reliance on old contents would show.  Kept in its own file, collected last,
so it runs both alone and after every other test."""
import ctypes

import numpy as np
import pytest
import torch

from qmm_testutil import from_dev_bf16, make_linear, random_layer, sin_input, to_dev_u16
from qwen_imager_b200 import _lib

pytestmark = pytest.mark.gpu


def _call_workspace(lib, lin, x, m, splits, y):
    w = lin.affine.c_weight()
    nbytes = int(lib.qmm_splitk_workspace_bytes(ctypes.byref(w), m, splits))
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.qmm_linear_splitk(ctypes.byref(w), x.data_ptr(), m, None, y.data_ptr(), splits, ws.data_ptr(),
                                     nbytes, st))


def _call_static(lib, lin, x, m, splits, y):
    w = lin.affine.c_weight()
    st = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.qmm_linear_splitk_static(ctypes.byref(w), x.data_ptr(), m, None, y.data_ptr(), splits, st))


def _leave_other_partials(lib):
    """A static-scratch call of another shape and split count, so that the
    scratch holds unrelated partial sums when the checked calls begin."""
    packed, scales, offsets, bias = random_layer(1536, 2048, 4, 64, seed=99, bias=False)
    lin = make_linear(packed, scales, offsets, bias, 4, 64)
    m = 96
    x = to_dev_u16(np.full((m, 2048), 0x3F80, dtype=np.uint16))  # every x = 1.0
    y = torch.empty((m, 1536), dtype=torch.bfloat16, device="cuda")
    _call_static(lib, lin, x, m, 8, y)
    torch.cuda.synchronize()


@pytest.mark.parametrize("m,k,n,bits,splits", [(256, 3072, 3072, 4, 3), (200, 1024, 768, 8, 4)])
def test_static_scratch_matches_caller_workspace_twice(oracle, m, k, n, bits, splits):
    lib = _lib.load()
    packed, scales, offsets, bias = random_layer(n, k, bits, 64, seed=m + n, bias=True)
    lin = make_linear(packed, scales, offsets, bias, bits, 64)
    x = to_dev_u16(sin_input(m, k))
    ref = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    _call_workspace(lib, lin, x, m, splits, ref)
    torch.cuda.synchronize()
    want = from_dev_bf16(ref)
    assert np.isfinite(oracle.bf16_to_f32(want)).all()
    _leave_other_partials(lib)
    for _ in range(2):  # two calls in a row reuse the same scratch
        y = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
        _call_static(lib, lin, x, m, splits, y)
        torch.cuda.synchronize()
        # same kernels, same summation order: bit-identical to the workspace path
        assert np.array_equal(from_dev_bf16(y), want)


def test_static_scratch_refuses_oversize_requests():
    lib = _lib.load()
    cap = int(lib.qmm_static_scratch_bytes())
    assert cap == 16 << 20
    packed, scales, offsets, bias = random_layer(4096, 1024, 4, 64, seed=2, bias=False)
    lin = make_linear(packed, scales, offsets, bias, 4, 64)
    m, splits = 4096, 2  # 2 * 4096 * 4096 * 4 bytes = 128 MiB
    x = torch.zeros((m, 1024), dtype=torch.bfloat16, device="cuda")
    y = torch.empty((m, 4096), dtype=torch.bfloat16, device="cuda")
    w = lin.affine.c_weight()
    status = lib.qmm_linear_splitk_static(ctypes.byref(w), x.data_ptr(), m, None, y.data_ptr(), splits,
                                          torch.cuda.current_stream().cuda_stream)
    assert status == _lib.QMM_ERR_UNSUPPORTED
    assert b"static scratch" in lib.qmm_last_error()
    # sizes whose byte count would not fit 64 bits are refused the same way,
    # and split counts outside [1, 16] before any size arithmetic
    big = _lib.QmmWeight(w.packed, w.scales, w.biases, 2**40, 1024, 4, 64)
    assert lib.qmm_linear_splitk_static(ctypes.byref(big), x.data_ptr(), 2**40, None, y.data_ptr(), 16,
                                        torch.cuda.current_stream().cuda_stream) == _lib.QMM_ERR_UNSUPPORTED
    assert lib.qmm_linear_splitk_static(ctypes.byref(w), x.data_ptr(), m, None, y.data_ptr(), 17,
                                        torch.cuda.current_stream().cuda_stream) == _lib.QMM_ERR_INVALID_ARGUMENT
