"""Fused quantized linear (GEMV and tcgen05 GEMM) against the oracle.

Restates the reference's `fused_metal_matmul_matches_dequantized_weights`
(src/quant.rs:741-792): the same shapes (ragged m and n, a tile-sized k),
4 and 8 bits, a bias on 8-bit layers, x = sin(0.37 i).  The bar is the one
the benchmark contract states against the reference's f32 CPU path
(src/quant.rs:105-119): max|d| / max|ref| <= 1e-2 and mean|d| / max|ref| <= 1e-3,
normalised by max|ref| like the reference test (src/quant.rs:768-775).
Tighter checks pin the GEMM to the bf16 weights it consumes: with x = I the
output is exactly bf16(W^T + bias) (every weight element checked bit for bit),
and for random x it is within one bf16 rounding of
bf16(x . dequantize_bf16(W)^T + bias) up to f32 accumulation order.
"""
import numpy as np
import pytest
import torch

from qmm_testutil import (assert_one_rounding, bf16_ulp_diff, from_dev_bf16, make_linear,
                          random_layer, rel_errors, sin_input, to_dev_u16)
from qwen_imager_b200 import _lib

pytestmark = pytest.mark.gpu

MAX_REL = 1e-2
MEAN_REL = 1e-3
REFERENCE_SHAPES = [(37, 4096, 1024), (130, 1152, 3456), (1, 128, 96), (64, 64, 64), (200, 4096, 12288)]


def run(lin, x_np, path=_lib.QMM_PATH_AUTO, **kw):
    y = lin.forward_fused(to_dev_u16(x_np), path=path, **kw)
    torch.cuda.synchronize()
    return from_dev_bf16(y)


def oracle_f32(oracle, x, packed, scales, offsets, bias, bits, group):
    return oracle.linear_f32(x, packed, scales, offsets, bits, group, bias)


def bf16_weight_reference(oracle, x, packed, scales, offsets, bias, bits, group):
    """x . W^T + bias with W rounded to bf16 exactly as dequantize_bf16 rounds it."""
    w = oracle.bf16_to_f32(oracle.dequantize_bf16(packed, scales, offsets, bits, group))
    return oracle.matmul_f32(oracle.bf16_to_f32(x).reshape(x.shape), w, bias)


@pytest.mark.parametrize("m,k,n", REFERENCE_SHAPES)
@pytest.mark.parametrize("bits", [4, 8])
def test_fused_linear_matches_oracle(oracle, m, k, n, bits):
    packed, scales, offsets, bias = random_layer(n, k, bits, 64, seed=m + n + bits, bias=bits == 8)
    lin = make_linear(packed, scales, offsets, bias, bits, 64)
    x = sin_input(m, k)
    got = run(lin, x)
    assert got.shape == (m, n)
    ref = oracle_f32(oracle, x, packed, scales, offsets, bias, bits, 64)
    mx, mean = rel_errors(got, ref)
    assert mx < MAX_REL and mean < MEAN_REL, (mx, mean)


@pytest.mark.parametrize("path", [_lib.QMM_PATH_GEMM, _lib.QMM_PATH_GEMM_PAIR])
@pytest.mark.parametrize("m,k,n", REFERENCE_SHAPES)
@pytest.mark.parametrize("bits", [4, 8])
def test_gemm_consumes_exact_bf16_weights(oracle, m, k, n, bits, path):
    packed, scales, offsets, bias = random_layer(n, k, bits, 64, seed=7 * m + n + bits, bias=True)
    lin = make_linear(packed, scales, offsets, bias, bits, 64)
    x = sin_input(m, k)
    got = run(lin, x, path=path)
    assert_one_rounding(got, bf16_weight_reference(oracle, x, packed, scales, offsets, bias, bits, 64), oracle)


@pytest.mark.parametrize("bits,group,n,k", [(4, 64, 200, 1152), (8, 64, 300, 640), (4, 32, 130, 512),
                                            (8, 128, 64, 1024), (4, 64, 1024, 4096)])
def test_gemm_identity_probe_reproduces_every_weight(oracle, bits, group, n, k):
    """x = I (k tokens, one-hot rows): every output is one weight plus the bias,
    with no accumulation error, so y must equal bf16(W^T + bias) exactly."""
    packed, scales, offsets, bias = random_layer(n, k, bits, group, seed=n + k + bits, bias=True)
    lin = make_linear(packed, scales, offsets, bias, bits, group)
    eye = torch.eye(k, dtype=torch.bfloat16, device="cuda")
    got = from_dev_bf16(lin.forward_fused(eye, path=_lib.QMM_PATH_GEMM))
    got_pair = from_dev_bf16(lin.forward_fused(eye, path=_lib.QMM_PATH_GEMM_PAIR))
    assert np.array_equal(got_pair, got)
    w = oracle.bf16_to_f32(oracle.dequantize_bf16(packed, scales, offsets, bits, group))
    ref = oracle.f32_to_bf16(w.T + oracle.bf16_to_f32(bias)[None, :])
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("m", [1, 2, 3, 5, 8, 13, 16])
@pytest.mark.parametrize("bits", [2, 4, 8])
def test_gemv_small_m(oracle, m, bits):
    k, n = 640, 300
    packed, scales, offsets, bias = random_layer(n, k, bits, 64, seed=m * 10 + bits)
    lin = make_linear(packed, scales, offsets, bias, bits, 64)
    x = sin_input(m, k)
    got = run(lin, x, path=_lib.QMM_PATH_GEMV)
    # f32 weights, f32 accumulation: within one bf16 rounding of the oracle
    assert_one_rounding(got, oracle_f32(oracle, x, packed, scales, offsets, bias, bits, 64), oracle)


@pytest.mark.parametrize("path", [_lib.QMM_PATH_GEMM, _lib.QMM_PATH_GEMM_PAIR])
@pytest.mark.parametrize("m", [1, 17, 100, 191, 192, 193, 385])
@pytest.mark.parametrize("n", [64, 200, 1000])
def test_gemm_ragged_edges(oracle, m, n, path):
    k, bits = 320, 4
    packed, scales, offsets, bias = random_layer(n, k, bits, 64, seed=m + 31 * n)
    lin = make_linear(packed, scales, offsets, bias, bits, 64)
    x = sin_input(m, k)
    got = run(lin, x, path=path)
    assert_one_rounding(got, bf16_weight_reference(oracle, x, packed, scales, offsets, bias, bits, 64), oracle)


@pytest.mark.parametrize("bits,group", [(4, 32), (4, 128), (8, 32), (8, 128), (4, 256)])
def test_gemm_group_sizes(oracle, bits, group):
    m, k, n = 150, 512, 256
    packed, scales, offsets, bias = random_layer(n, k, bits, group, seed=bits * group)
    lin = make_linear(packed, scales, offsets, bias, bits, group)
    x = sin_input(m, k)
    got = run(lin, x, path=_lib.QMM_PATH_GEMM)
    assert_one_rounding(got, bf16_weight_reference(oracle, x, packed, scales, offsets, bias, bits, group), oracle)


def test_two_bit_gemm_falls_back_to_dense(oracle):
    """2-bit has no fused GEMM, like the reference's fused kernel (src/quant.rs:783-790):
    forward dequantizes and runs a dense GEMM instead."""
    m, k, n = 40, 128, 64
    packed, scales, offsets, _ = random_layer(n, k, 2, 64, seed=5, bias=False)
    lin = make_linear(packed, scales, offsets, None, 2, 64)
    x = sin_input(m, k)
    with pytest.raises(_lib.QmmError) as e:
        run(lin, x, path=_lib.QMM_PATH_GEMM)
    assert e.value.status == _lib.QMM_ERR_UNSUPPORTED
    got = run(lin, x)
    ref = oracle_f32(oracle, x, packed, scales, offsets, None, 2, 64)
    mx, mean = rel_errors(got, ref)
    assert mx < MAX_REL and mean < MEAN_REL


@pytest.mark.parametrize("path", [_lib.QMM_PATH_GEMV, _lib.QMM_PATH_GEMM])
@pytest.mark.parametrize("activation,act_code", [(None, 0), ("gelu_tanh", 1), ("silu", 2)])
def test_fused_epilogue(oracle, path, activation, act_code):
    m = 7 if path == _lib.QMM_PATH_GEMV else 77
    k, n, bits = 256, 384, 8
    packed, scales, offsets, bias = random_layer(n, k, bits, 64, seed=11 + act_code)
    rng = np.random.default_rng(12)
    gate = oracle.f32_to_bf16(rng.standard_normal(n).astype(np.float32))
    residual = oracle.f32_to_bf16(rng.standard_normal((m, n)).astype(np.float32))
    lin = make_linear(packed, scales, offsets, bias, bits, 64)
    x = sin_input(m, k)
    got = run(lin, x, path=path, gate=to_dev_u16(gate), residual=to_dev_u16(residual), activation=activation)
    if path == _lib.QMM_PATH_GEMM:
        y = bf16_weight_reference(oracle, x, packed, scales, offsets, bias, bits, 64)
    else:
        y = oracle_f32(oracle, x, packed, scales, offsets, bias, bits, 64)
    ref = oracle.epilogue_bf16(y, gate, residual, act_code)
    ulps = bf16_ulp_diff(got, ref)
    d = np.abs(oracle.bf16_to_f32(got) - oracle.bf16_to_f32(ref))
    assert not ((ulps > 2) & (d > np.abs(oracle.bf16_to_f32(ref)).max() * 2.0**-10)).any()


def test_residual_may_alias_output(oracle):
    m, k, n, bits = 64, 256, 128, 4
    packed, scales, offsets, bias = random_layer(n, k, bits, 64, seed=99)
    lin = make_linear(packed, scales, offsets, bias, bits, 64)
    rng = np.random.default_rng(1)
    residual = oracle.f32_to_bf16(rng.standard_normal((m, n)).astype(np.float32))
    buf = to_dev_u16(residual)
    lin.forward_fused(to_dev_u16(sin_input(m, k)), residual=buf, out=buf)
    torch.cuda.synchronize()
    y = bf16_weight_reference(oracle, sin_input(m, k), packed, scales, offsets, bias, bits, 64)
    ref = oracle.epilogue_bf16(y, None, residual, 0)
    d = np.abs(oracle.bf16_to_f32(from_dev_bf16(buf)) - oracle.bf16_to_f32(ref))
    assert d.max() <= np.abs(oracle.bf16_to_f32(ref)).max() * 2.0**-7


def test_empty_input_and_leading_dims(oracle):
    packed, scales, offsets, bias = random_layer(96, 128, 4, 64, seed=1)
    lin = make_linear(packed, scales, offsets, bias, 4, 64)
    y = lin.forward(torch.empty((0, 128), dtype=torch.bfloat16, device="cuda"))
    assert tuple(y.shape) == (0, 96)
    x = sin_input(6, 128)
    y3 = lin.forward(to_dev_u16(x).reshape(2, 3, 128))
    assert tuple(y3.shape) == (2, 3, 96)
    assert np.array_equal(from_dev_bf16(y3.reshape(6, 96)), run(lin, x))


def test_device_error_word_is_clear():
    from qwen_imager_b200 import device_error
    assert device_error() == 0


def test_argument_errors_are_reported():
    import ctypes
    lib = _lib.load()
    packed, scales, offsets, bias = random_layer(96, 128, 4, 64, seed=2)
    lin = make_linear(packed, scales, offsets, bias, 4, 64)
    w = lin.affine.c_weight()
    x = torch.zeros((4, 128), dtype=torch.bfloat16, device="cuda")
    y = torch.zeros((4, 96), dtype=torch.bfloat16, device="cuda")
    assert lib.qmm_linear(ctypes.byref(w), x.data_ptr(), 4, None, None, None) == _lib.QMM_ERR_INVALID_ARGUMENT
    assert lib.qmm_linear(ctypes.byref(w), x.data_ptr() + 2, 4, None, y.data_ptr(), None) == _lib.QMM_ERR_MISALIGNED
    assert lib.qmm_linear(ctypes.byref(w), x.data_ptr(), -1, None, y.data_ptr(), None) == _lib.QMM_ERR_BAD_SHAPE
    assert lib.qmm_linear(ctypes.byref(w), x.data_ptr(), 4, None, x.data_ptr(), None) == _lib.QMM_ERR_INVALID_ARGUMENT
    assert lib.qmm_linear_ex(ctypes.byref(w), x.data_ptr(), 4, None, y.data_ptr(), 9, None) == _lib.QMM_ERR_INVALID_ARGUMENT
    with pytest.raises(_lib.QmmError):
        lin.forward(torch.zeros((4, 100), dtype=torch.bfloat16, device="cuda"))
    with pytest.raises(_lib.QmmError):  # f64 activations: no kernel and no dense route serves them
        lin.forward(torch.zeros((4, 128), dtype=torch.float64, device="cuda"))
    # f16 activations run the GEMM with fp16 operands (tests/test_gpu_f16_operands.py).
    assert lin.forward(torch.zeros((4, 128), dtype=torch.float16, device="cuda")).dtype == torch.bfloat16
