"""The oracle (CPU restatement of the reference path) pinned to MLX's own
golden vectors, as the reference's `cpu_dequantization_matches_mlx` does
(src/quant.rs:668-694): dequantization exact, matmul within 0.02."""
import numpy as np
import pytest


@pytest.mark.parametrize("bits", [4, 8])
def test_oracle_dequantize_is_bit_exact_with_mlx(golden, oracle, bits):
    p = f"q{bits}"
    dq = oracle.dequantize_bf16(golden[p + ".weight"], golden[p + ".scales"], golden[p + ".biases"], bits, 64)
    assert dq.shape == (96, 192)
    assert np.array_equal(dq, golden[p + ".dequantized"])


@pytest.mark.parametrize("bits", [4, 8])
def test_numpy_twin_is_bit_exact_with_mlx(golden, oracle, bits):
    p = f"q{bits}"
    dq = oracle.dequantize_numpy(golden[p + ".weight"], golden[p + ".scales"], golden[p + ".biases"], bits, 64)
    assert np.array_equal(dq, golden[p + ".dequantized"])


@pytest.mark.parametrize("bits", [4, 8])
def test_oracle_matmul_matches_mlx(golden, oracle, bits):
    p = f"q{bits}"
    y = oracle.linear_bf16(golden["x"], golden[p + ".weight"], golden[p + ".scales"], golden[p + ".biases"], bits, 64)
    err = np.abs(oracle.bf16_to_f32(y) - oracle.bf16_to_f32(golden[p + ".y"])).max()
    assert err < 0.02, err


@pytest.mark.parametrize("bits,group", [(2, 32), (2, 64), (4, 32), (4, 64), (4, 128), (8, 64), (8, 128)])
def test_c_oracle_and_numpy_twin_agree(oracle, bits, group):
    rng = np.random.default_rng(bits * 1000 + group)
    n, k = 37, 512
    packed = rng.integers(0, 2**32, size=(n, k * bits // 32), dtype=np.uint64).astype(np.uint32)
    scales = oracle.f32_to_bf16(((rng.random((n, k // group)) - 0.5) * 0.02).astype(np.float32))
    biases = oracle.f32_to_bf16(((rng.random((n, k // group)) - 0.5) * 0.1).astype(np.float32))
    a = oracle.dequantize_bf16(packed, scales, biases, bits, group)
    b = oracle.dequantize_numpy(packed, scales, biases, bits, group)
    assert np.array_equal(a, b)
    f = oracle.dequantize_f32(packed, scales, biases, bits, group)
    assert np.array_equal(oracle.f32_to_bf16(f), a)


def test_bf16_rounding_is_nearest_even(oracle):
    # 1 + 2^-8 is the midpoint between bf16 1.0 and 1.0078125: ties to even -> 1.0
    x = np.array([1.0 + 2.0**-8, 1.0 + 3 * 2.0**-8, -(1.0 + 2.0**-8), 1.0 + 2.0**-8 + 2.0**-20], dtype=np.float32)
    got = oracle.f32_to_bf16(x)
    assert list(got) == [0x3F80, 0x3F82, 0xBF80, 0x3F81]


@pytest.mark.parametrize("bits", [4, 8])
def test_quantize_affine_roundtrip(oracle, bits):
    rng = np.random.default_rng(7)
    w = (rng.standard_normal((16, 256)) * 0.02).astype(np.float32)
    packed, scales, biases = oracle.quantize_affine(w, bits, 64)
    assert packed.shape == (16, 256 * bits // 32)
    deq = oracle.bf16_to_f32(oracle.dequantize_bf16(packed, scales, biases, bits, 64))
    step = oracle.bf16_to_f32(scales).repeat(64, axis=1)
    assert np.all(np.abs(deq - w) <= step + 2.0**-8 * np.abs(w))


def test_epilogue_oracle(oracle):
    y = np.array([[0.5, -1.0], [2.0, 0.0]], dtype=np.float32)
    gate = oracle.f32_to_bf16(np.array([2.0, 0.5], dtype=np.float32))
    res = oracle.f32_to_bf16(np.array([[1.0, 1.0], [1.0, 1.0]], dtype=np.float32))
    out = oracle.bf16_to_f32(oracle.epilogue_bf16(y, gate, res, 0))
    assert np.allclose(out, [[2.0, 0.5], [5.0, 1.0]])
    silu = oracle.bf16_to_f32(oracle.epilogue_bf16(y, None, None, 2))
    assert np.allclose(silu, y / (1 + np.exp(-y)), rtol=1e-2)
