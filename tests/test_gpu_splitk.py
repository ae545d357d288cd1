"""Split-K GEMM (qmm_linear_splitk) on B200: the small-m shapes of the DiT
text stream and of tensor-parallel shards, against the oracle.  Each split's
f32 partials are summed by a second kernel that applies the epilogue, so the
result keeps the GEMM's contract: within one bf16 rounding of
bf16(x . dequantize_bf16(W)^T + bias), and exact for x = I."""
import ctypes

import numpy as np
import pytest
import torch

from qmm_testutil import (assert_one_rounding, from_dev_bf16, make_linear, random_layer, sin_input,
                          to_dev_u16)
from test_gpu_linear import bf16_weight_reference
from qwen_imager_b200 import _lib

pytestmark = pytest.mark.gpu


def run_split(lin, x_np, splits, **kw):
    y = lin.forward_fused(to_dev_u16(x_np), path=_lib.QMM_PATH_GEMM, splits=splits, **kw)
    torch.cuda.synchronize()
    return from_dev_bf16(y)


@pytest.mark.parametrize("m,k,n,bits", [(256, 3072, 3072, 4), (37, 4096, 1024, 8), (512, 1536, 3072, 8),
                                        (200, 12288, 3072, 4), (1, 640, 96, 4), (193, 384, 1152, 8)])
@pytest.mark.parametrize("splits", [1, 2, 3, 4, 6, 8])
def test_splitk_matches_bf16_weight_reference(oracle, m, k, n, bits, splits):
    if (k // 64) % splits:
        pytest.skip("split count does not divide the k-blocks")
    packed, scales, offsets, bias = random_layer(n, k, bits, 64, seed=m + k + n + splits, bias=True)
    lin = make_linear(packed, scales, offsets, bias, bits, 64)
    x = sin_input(m, k)
    got = run_split(lin, x, splits)
    assert_one_rounding(got, bf16_weight_reference(oracle, x, packed, scales, offsets, bias, bits, 64), oracle)


@pytest.mark.parametrize("splits", [2, 4])
def test_splitk_identity_probe_is_exact(oracle, splits):
    n, k, bits = 200, 1024, 4
    packed, scales, offsets, bias = random_layer(n, k, bits, 64, seed=77, bias=True)
    lin = make_linear(packed, scales, offsets, bias, bits, 64)
    eye = torch.eye(k, dtype=torch.bfloat16, device="cuda")
    got = from_dev_bf16(lin.forward_fused(eye, path=_lib.QMM_PATH_GEMM, splits=splits))
    w = oracle.bf16_to_f32(oracle.dequantize_bf16(packed, scales, offsets, bits, 64))
    want = oracle.f32_to_bf16(w.T + oracle.bf16_to_f32(bias)[None, :])
    assert np.array_equal(got, want)


@pytest.mark.parametrize("activation,act_code", [(None, 0), ("gelu_tanh", 1), ("silu", 2)])
def test_splitk_fused_epilogue_and_residual_alias(oracle, activation, act_code):
    m, k, n, bits = 256, 1536, 768, 4
    packed, scales, offsets, bias = random_layer(n, k, bits, 64, seed=90 + act_code, bias=True)
    rng = np.random.default_rng(91)
    gate = oracle.f32_to_bf16(rng.standard_normal(n).astype(np.float32))
    residual = oracle.f32_to_bf16(rng.standard_normal((m, n)).astype(np.float32))
    lin = make_linear(packed, scales, offsets, bias, bits, 64)
    x = sin_input(m, k)
    buf = to_dev_u16(residual)  # y aliases the residual
    lin.forward_fused(to_dev_u16(x), path=_lib.QMM_PATH_GEMM, splits=3, gate=to_dev_u16(gate), residual=buf,
                      activation=activation, out=buf)
    torch.cuda.synchronize()
    y = bf16_weight_reference(oracle, x, packed, scales, offsets, bias, bits, 64)
    ref = oracle.epilogue_bf16(y, gate, residual, act_code)
    d = np.abs(oracle.bf16_to_f32(from_dev_bf16(buf)) - oracle.bf16_to_f32(ref))
    assert d.max() <= np.abs(oracle.bf16_to_f32(ref)).max() * 2.0**-7


def test_recommended_splits_for_dit_text_stream_and_full_image():
    lib = _lib.load()

    def splits(m, k, n, bits):
        packed, scales, offsets, bias = random_layer(n, k, bits, 64, seed=1, bias=False)
        lin = make_linear(packed, scales, offsets, bias, bits, 64)
        w = lin.affine.c_weight()
        return lib.qmm_gemm_splits(ctypes.byref(w), m)

    assert splits(256, 3072, 3072, 4) > 1        # text-stream out-proj: 48 tiles
    assert splits(256, 12288, 3072, 4) > 1       # text-stream FFN-down
    assert splits(4352, 3072, 12288, 8) == 1     # image FFN-up: 2208 tiles
    assert splits(4096, 3072, 3072, 4) == 1


def test_splitk_argument_errors():
    lib = _lib.load()
    packed, scales, offsets, bias = random_layer(96, 640, 4, 64, seed=3, bias=False)
    lin = make_linear(packed, scales, offsets, bias, 4, 64)
    w = lin.affine.c_weight()
    x = torch.zeros((8, 640), dtype=torch.bfloat16, device="cuda")
    y = torch.empty((8, 96), dtype=torch.bfloat16, device="cuda")
    ws = torch.empty(1 << 20, dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    # 10 k-blocks do not split 3 ways
    assert lib.qmm_linear_splitk(ctypes.byref(w), x.data_ptr(), 8, None, y.data_ptr(), 3, ws.data_ptr(),
                                 ws.numel(), st) == _lib.QMM_ERR_INVALID_ARGUMENT
    # workspace too small
    assert lib.qmm_linear_splitk(ctypes.byref(w), x.data_ptr(), 8, None, y.data_ptr(), 2, ws.data_ptr(),
                                 100, st) == _lib.QMM_ERR_INVALID_ARGUMENT
    # workspace overlapping y
    assert lib.qmm_linear_splitk(ctypes.byref(w), x.data_ptr(), 8, None, y.data_ptr(), 2, y.data_ptr(),
                                 1 << 20, st) == _lib.QMM_ERR_INVALID_ARGUMENT
    assert lib.qmm_linear_splitk(ctypes.byref(w), x.data_ptr(), 8, None, y.data_ptr(), 2, ws.data_ptr(),
                                 ws.numel(), st) == _lib.QMM_OK
    torch.cuda.synchronize()
