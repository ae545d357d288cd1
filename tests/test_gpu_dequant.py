"""GPU dequantization is bit-exact with the reference unpacking
(src/quant.rs:555-573): against MLX's own golden vectors and against the
oracle on random layers of every supported layout."""
import numpy as np
import pytest
import torch

from qmm_testutil import from_dev_bf16, make_linear, random_layer

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("bits", [4, 8])
def test_gpu_dequantize_matches_mlx_golden(golden, bits):
    p = f"q{bits}"
    lin = make_linear(golden[p + ".weight"], golden[p + ".scales"], golden[p + ".biases"], None, bits, 64)
    w = lin.dense()[0]
    assert w.dtype == torch.bfloat16 and tuple(w.shape) == (96, 192)
    assert np.array_equal(from_dev_bf16(w), golden[p + ".dequantized"])


@pytest.mark.parametrize("bits,group", [(2, 32), (2, 64), (4, 32), (4, 64), (4, 128), (8, 32), (8, 64), (8, 128)])
def test_gpu_dequantize_matches_oracle(oracle, bits, group):
    packed, scales, offsets, _ = random_layer(200, 640, bits, group, seed=bits + group)
    lin = make_linear(packed, scales, offsets, None, bits, group)
    got = from_dev_bf16(lin.affine.dequantize(torch.bfloat16))
    assert np.array_equal(got, oracle.dequantize_bf16(packed, scales, offsets, bits, group))
    got32 = lin.affine.dequantize(torch.float32).cpu().numpy()
    assert np.array_equal(got32.view(np.uint32), oracle.dequantize_f32(packed, scales, offsets, bits, group).view(np.uint32))


def test_gpu_dequantize_extreme_offsets(oracle):
    """Offsets far below or above the scale (where a single-rounding fused
    multiply-add in bf16 would differ from the reference's f32-then-bf16)."""
    rng = np.random.default_rng(3)
    n, k, bits, group = 64, 256, 8, 64
    packed = rng.integers(0, 2**32, size=(n, k * bits // 32), dtype=np.uint64).astype(np.uint32)
    s = rng.choice([1.0078125, -1.0078125, 3.0, 0.5], size=(n, k // group)).astype(np.float32)
    o = (rng.choice([1e-12, -1e-12, 2.0**-40, 7.0, -1e3], size=(n, k // group))).astype(np.float32)
    scales, offsets = oracle.f32_to_bf16(s), oracle.f32_to_bf16(o)
    lin = make_linear(packed, scales, offsets, None, bits, group)
    got = from_dev_bf16(lin.affine.dequantize(torch.bfloat16))
    assert np.array_equal(got, oracle.dequantize_bf16(packed, scales, offsets, bits, group))
