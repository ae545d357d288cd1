"""The GEMM with fp16 operands (QMM_PATH_GEMM_F16): x in fp16 and the
dequantized weights rounded to fp16 (11 significant bits) instead of bf16 (8),
so the product is closer to the reference's CPU path, which keeps the
weights in f32 (src/quant.rs:105-113).  Checked against the oracle:
  - an identity input reproduces every fp16-rounded weight plus the bias,
    rounded once to bf16, exactly;
  - outputs within one bf16 rounding of the f32 product of the fp16-rounded
    weights;
  - at the full FFN-up configuration, mean|d| / mean|ref| against the
    reference's own bf16 output is below 1e-3 (recorded beside the bf16
    operands' figure).
"""
import json
import os

import numpy as np
import pytest
import torch

from qmm_testutil import assert_one_rounding, from_dev_bf16, make_linear, random_layer, sin_input
from qwen_imager_b200.synthetic import gaussian, quantized_linear

pytestmark = pytest.mark.gpu
RECORD = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "gpurun_out",
                      "config_parity.jsonl")


def _f16_weights(oracle, packed, scales, offsets, bits, group):
    """The oracle's f32 dequantization (s * q + o) rounded to fp16 (RNE), as f32."""
    return oracle.dequantize_f32(packed, scales, offsets, bits, group).astype(np.float16).astype(np.float32)


@pytest.mark.parametrize("bits", [4, 8])
def test_identity_reproduces_fp16_weights(oracle, bits):
    n, k = 200, 256
    packed, scales, offsets, bias = random_layer(n, k, bits, 64, seed=60 + bits)
    lin = make_linear(packed, scales, offsets, bias, bits, 64)
    x = torch.eye(k, dtype=torch.float16, device="cuda")
    y = lin.forward_fused(x, operands="fp16")
    torch.cuda.synchronize()
    w16 = _f16_weights(oracle, packed, scales, offsets, bits, 64)
    want = oracle.f32_to_bf16((w16.T + oracle.bf16_to_f32(bias)[None, :]).astype(np.float32))
    assert np.array_equal(from_dev_bf16(y), want)


@pytest.mark.parametrize("m,k,n,bits", [(37, 4096, 1024, 4), (200, 3072, 1536, 8), (300, 1152, 3456, 4),
                                        (17, 64, 64, 8)])
def test_fp16_operands_within_one_rounding(oracle, m, k, n, bits):
    packed, scales, offsets, bias = random_layer(n, k, bits, 64, seed=m + k + bits)
    lin = make_linear(packed, scales, offsets, bias, bits, 64)
    x = sin_input(m, k)
    xd = torch.from_numpy(oracle.bf16_to_f32(x)).cuda().to(torch.bfloat16)
    y = lin.forward_fused(xd, operands="fp16")
    torch.cuda.synchronize()
    x16 = oracle.bf16_to_f32(x).astype(np.float16).astype(np.float32)
    ref = oracle.matmul_f32(x16, _f16_weights(oracle, packed, scales, offsets, bits, 64), bias)
    assert_one_rounding(from_dev_bf16(y), ref, oracle)


def test_fp16_operands_at_the_ffn_up_configuration(oracle):
    m, k, n = 4352, 3072, 12288
    lin = quantized_linear(n, k, 8, seed=20)
    g = torch.Generator(device="cuda")
    g.manual_seed(21)
    x = gaussian((m, k), 1.0, g, "cuda").to(torch.bfloat16)
    rows = np.random.default_rng(5).choice(m, size=256, replace=False)
    a = lin.affine
    packed = a.packed.view(torch.int32).cpu().numpy().view(np.uint32)
    scales, offsets = from_dev_bf16(a.scales), from_dev_bf16(a.offsets)
    xr = from_dev_bf16(x)[rows]
    ref_bf16 = oracle.bf16_to_f32(oracle.linear_bf16(xr, packed, scales, offsets, 8, 64)).astype(np.float64)
    out = {}
    for operands in ("bf16", "fp16"):
        y = lin.forward_fused(x, operands=operands)
        torch.cuda.synchronize()
        got = oracle.bf16_to_f32(from_dev_bf16(y)[rows]).astype(np.float64)
        d = np.abs(got - ref_bf16)
        out[operands] = (d.max() / np.abs(ref_bf16).max(), d.mean() / np.abs(ref_bf16).max(),
                         d.mean() / np.abs(ref_bf16).mean())
    os.makedirs(os.path.dirname(RECORD), exist_ok=True)
    with open(RECORD, "a") as f:
        for operands, (mx, mean, mm) in out.items():
            f.write(json.dumps({"case": f"config2 FFN-up vs the reference's bf16 output, {operands} operands",
                                "max_rel": mx, "mean_rel": mean, "mean_over_mean": mm}) + "\n")
    mx, mean, mm = out["fp16"]
    assert mx <= 1e-2 and mean <= 1e-3 and mm < 1e-3, out
    assert mm < out["bf16"][2], out
