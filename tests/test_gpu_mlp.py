"""The SwiGLU MLP caller (src/ops.rs:183-208) and the epilogue mode it uses,
plus f32 activations, against the oracle.

- QMM_EPILOGUE_RESIDUAL_MUL: y = r * (gate * act(x W^T + b)), one rounding,
  on every kernel family (tensor-core and FMA GEMVs, the tcgen05 GEMM with its
  TMA and element residual paths, split-K).
- SwiGlu.forward = down(silu(gate(x)) * up(x)) in 4096-token chunks, against
  the oracle's composition of the same three linears; chunk boundaries do not
  change the result.
- f32 inputs (the reference's qmm_f32 kernels, src/quant.rs:324-325, tested at
  1e-5, src/quant.rs:774): the weight dequantized to f32 and an f32 GEMM, with
  an f32 result, within 1e-5 of the oracle's f32 product.
"""
import numpy as np
import pytest
import torch

from qmm_testutil import assert_one_rounding, from_dev_bf16, make_linear, random_layer, sin_input, to_dev_u16
from qwen_imager_b200 import _lib
from qwen_imager_b200.ops import SwiGlu

pytestmark = pytest.mark.gpu


def _host(lin):
    a = lin.affine
    return (a.packed.view(torch.int32).cpu().numpy().view(np.uint32), from_dev_bf16(a.scales),
            from_dev_bf16(a.offsets), None if a.bias is None else from_dev_bf16(a.bias))


def _oracle_mul(oracle, x, lin, r, act=0):
    packed, scales, offsets, bias = _host(lin)
    y = oracle.linear_f32(x, packed, scales, offsets, lin.affine.bits, lin.affine.group, bias)
    if act == 2:
        y = y / (1.0 + np.exp(-y.astype(np.float64)))
    return (oracle.bf16_to_f32(r).astype(np.float64) * y).astype(np.float32)


@pytest.mark.parametrize("m,k,n,bits,path,splits", [
    (1, 3072, 1536, 4, _lib.QMM_PATH_AUTO, None),    # tensor-core GEMV
    (5, 1024, 768, 8, _lib.QMM_PATH_AUTO, None),     # FMA GEMV
    (300, 1024, 1536, 4, _lib.QMM_PATH_GEMM, 1),      # GEMM, TMA residual chunks
    (300, 1024, 1532, 8, _lib.QMM_PATH_GEMM, 1),      # GEMM, n % 8 != 0: element residual loads
    (256, 3072, 1024, 4, _lib.QMM_PATH_GEMM, 4),      # split-K reduction
])
def test_residual_mul_epilogue(oracle, m, k, n, bits, path, splits):
    packed, scales, offsets, bias = random_layer(n, k, bits, 64, seed=m + n, bias=True)
    lin = make_linear(packed, scales, offsets, bias, bits, 64)
    x = sin_input(m, k)
    r = oracle.f32_to_bf16(np.cos(np.arange(m * n, dtype=np.float64) * 0.11).astype(np.float32).reshape(m, n))
    y = lin.forward_fused(to_dev_u16(x), residual=to_dev_u16(r), residual_mul=True, path=path, splits=splits)
    torch.cuda.synchronize()
    assert_one_rounding(from_dev_bf16(y), _oracle_mul(oracle, x, lin, r), oracle)


def test_residual_mul_rejects_unknown_flags():
    import ctypes
    lib = _lib.load()
    packed, scales, offsets, bias = random_layer(128, 256, 4, 64, seed=1, bias=False)
    lin = make_linear(packed, scales, offsets, bias, 4, 64)
    x = to_dev_u16(sin_input(32, 256))
    y = torch.empty((32, 128), dtype=torch.bfloat16, device="cuda")
    w = lin.affine.c_weight()
    ep = _lib.QmmEpilogue(None, None, None, 0x200)
    assert lib.qmm_linear(ctypes.byref(w), x.data_ptr(), 32, ctypes.byref(ep), y.data_ptr(),
                          torch.cuda.current_stream().cuda_stream) == _lib.QMM_ERR_INVALID_ARGUMENT


def _swiglu(dim, hidden, bits, seed, chunk):
    lins = []
    for i, (n, k) in enumerate(((hidden, dim), (hidden, dim), (dim, hidden))):
        packed, scales, offsets, _ = random_layer(n, k, bits, 64, seed=seed + i, bias=False)
        lins.append(make_linear(packed, scales, offsets, None, bits, 64))
    return SwiGlu(*lins, chunk=chunk)


def _oracle_swiglu(oracle, x, mlp):
    pg, sg, og, _ = _host(mlp.gate)
    g = oracle.epilogue_bf16(oracle.linear_f32(x, pg, sg, og, mlp.gate.affine.bits, 64), activation=2)
    h = oracle.f32_to_bf16(_oracle_mul(oracle, x, mlp.up, g))
    pd, sd, od, _ = _host(mlp.down)
    return oracle.linear_f32(h, pd, sd, od, mlp.down.affine.bits, 64), h


@pytest.mark.parametrize("m,dim,hidden,bits,chunk", [
    (300, 4096, 12288, 4, 4096),   # the reference DiT's MLP widths (src/dit.rs:32), one chunk
    (333, 1024, 3072, 8, 128),     # several chunks, a ragged last one
    (1, 1024, 3072, 4, 4096),      # a single token: GEMVs
])
def test_swiglu_matches_oracle_composition(oracle, m, dim, hidden, bits, chunk):
    mlp = _swiglu(dim, hidden, bits, seed=m, chunk=chunk)
    x = sin_input(m, dim)
    y = mlp.forward(to_dev_u16(x).reshape(1, m, dim))
    torch.cuda.synchronize()
    assert y.shape == (1, m, dim)
    ref, _h = _oracle_swiglu(oracle, x, mlp)
    got = oracle.bf16_to_f32(from_dev_bf16(y.reshape(m, dim))).astype(np.float64)
    d = np.abs(got - ref)
    mx, mean = d.max() / np.abs(ref).max(), d.mean() / np.abs(ref).max()
    assert mx <= 1e-2 and mean <= 1e-3, (mx, mean)


def test_swiglu_chunking_does_not_change_the_result():
    mlp = _swiglu(1024, 3072, 4, seed=7, chunk=4096)
    x = to_dev_u16(sin_input(500, 1024))
    whole = mlp.forward(x)
    mlp.chunk = 96
    chunked = mlp.forward(x)
    torch.cuda.synchronize()
    assert torch.equal(whole, chunked)


@pytest.mark.parametrize("m,k,n,bits", [(37, 4096, 1024, 4), (130, 1152, 3456, 8), (1, 128, 96, 4),
                                        (64, 64, 64, 8)])
def test_f32_activations_match_the_f32_oracle(oracle, m, k, n, bits):
    packed, scales, offsets, bias = random_layer(n, k, bits, 64, seed=m * 3 + bits, bias=(bits == 8))
    lin = make_linear(packed, scales, offsets, bias, bits, 64)
    x32 = np.sin(np.arange(m * k, dtype=np.float64) * 0.37).astype(np.float32).reshape(m, k)
    y = lin.forward(torch.from_numpy(x32).cuda().reshape(1, m, k))
    torch.cuda.synchronize()
    assert y.dtype == torch.float32 and y.shape == (1, m, n)
    w = oracle.dequantize_f32(packed, scales, offsets, bits, 64).astype(np.float64)
    ref = x32.astype(np.float64) @ w.T
    if bias is not None:
        ref += oracle.bf16_to_f32(bias)
    err = np.abs(y.reshape(m, n).cpu().numpy() - ref).max() / np.abs(ref).max()
    assert err < 1e-5, err
