"""The quantized linear at the shapes of its other callers, against the oracle.

- Qwen3-VL text layers (src/text.rs:183-237): hidden 4096, no bias.
  - q_proj and o_proj: 4096 -> 4096;
  - k_proj and v_proj: 4096 -> 1024 (8 KV heads of 128, grouped-query attention);
  - MLP gate/up: 4096 -> 12288; MLP down: 12288 -> 4096.

  Prompts have ragged lengths, and decoding runs at m = 1.
- The DiT prefix pass (src/dit.rs:117-250). It runs the text prefix, at ragged token counts, through the
  block linears of the 3072-wide DiT:
  - QKV: 3072 -> 9216 with bias;
  - out: 3072 -> 3072 with gate and residual;
  - FFN up: 3072 -> 12288 with GELU-tanh;
  - FFN down: 12288 -> 3072 with gate and residual.

The bar is the benchmark contract's against the reference's f32 CPU path (src/quant.rs:105-119):
max|d| / max|ref| <= 1e-2 and mean|d| / max|ref| <= 1e-3.
"""
import numpy as np
import pytest

from qmm_testutil import from_dev_bf16, make_linear, random_layer, rel_errors, sin_input, to_dev_u16

pytestmark = pytest.mark.gpu

MAX_REL = 1e-2
MEAN_REL = 1e-3

TEXT_LAYERS = [(4096, 4096), (4096, 1024), (4096, 12288), (12288, 4096)]


def run(lin, x, **kw):
    import torch

    y = lin.forward_fused(to_dev_u16(x), **kw)
    torch.cuda.synchronize()
    return from_dev_bf16(y)


@pytest.mark.parametrize("k,n", TEXT_LAYERS)
@pytest.mark.parametrize("m", [1, 7, 77, 333])
@pytest.mark.parametrize("bits", [4, 8])
def test_text_encoder_layers(oracle, k, n, m, bits):
    packed, scales, offsets, _ = random_layer(n, k, bits, 64, seed=k + n + m + bits, bias=False)
    lin = make_linear(packed, scales, offsets, None, bits, 64)
    x = sin_input(m, k)
    got = run(lin, x)
    assert got.shape == (m, n)
    mx, mean = rel_errors(got, oracle.linear_f32(x, packed, scales, offsets, bits, 64, None))
    assert mx < MAX_REL and mean < MEAN_REL, (mx, mean)


# (k, n, epilogue) of the DiT block linears the prefix pass runs.
DIT_LAYERS = [(3072, 9216, "bias"), (3072, 3072, "gate_residual"), (3072, 12288, "gelu"),
              (12288, 3072, "gate_residual")]


@pytest.mark.parametrize("k,n,epilogue", DIT_LAYERS)
@pytest.mark.parametrize("m", [5, 77, 300])
def test_dit_prefix_pass_layers(oracle, k, n, epilogue, m):
    rng = np.random.default_rng(k + n + m)
    packed, scales, offsets, bias = random_layer(n, k, 4, 64, seed=k * 7 + n + m, bias=epilogue == "bias")
    lin = make_linear(packed, scales, offsets, bias, 4, 64)
    x = sin_input(m, k)
    y = oracle.linear_f32(x, packed, scales, offsets, 4, 64, bias)
    if epilogue == "gate_residual":
        gate = oracle.f32_to_bf16(rng.standard_normal(n).astype(np.float32))
        residual = oracle.f32_to_bf16(rng.standard_normal((m, n)).astype(np.float32))
        got = run(lin, x, gate=to_dev_u16(gate), residual=to_dev_u16(residual))
        ref = oracle.bf16_to_f32(oracle.epilogue_bf16(y, gate, residual, 0))
    elif epilogue == "gelu":
        got = run(lin, x, activation="gelu_tanh")
        ref = oracle.bf16_to_f32(oracle.epilogue_bf16(y, None, None, 1))
    else:
        got = run(lin, x)
        ref = y
    mx, mean = rel_errors(got, ref)
    assert mx < MAX_REL and mean < MEAN_REL, (mx, mean)
