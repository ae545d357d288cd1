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


def _oracle_mul(oracle, x, lin, r, bf16_weights=False):
    """r * (x W^T + b) in f32: W in f32 as the oracle path has it (the GEMVs'
    arithmetic), or rounded to bf16 as the tcgen05 GEMM consumes it."""
    packed, scales, offsets, bias = _host(lin)
    bits, group = lin.affine.bits, lin.affine.group
    if bf16_weights:
        w = oracle.bf16_to_f32(oracle.dequantize_bf16(packed, scales, offsets, bits, group))
        y = oracle.matmul_f32(oracle.bf16_to_f32(x), w, bias)
    else:
        y = oracle.linear_f32(x, packed, scales, offsets, bits, group, bias)
    return (oracle.bf16_to_f32(r).astype(np.float64) * y).astype(np.float32)


@pytest.mark.parametrize("m,k,n,bits,group,path,splits", [
    (1, 3072, 1536, 4, 64, _lib.QMM_PATH_AUTO, None),    # tensor-core GEMV
    (5, 1024, 768, 8, 64, _lib.QMM_PATH_AUTO, None),     # tensor-core GEMV, 8-bit
    (5, 1024, 768, 8, 32, _lib.QMM_PATH_AUTO, None),     # FMA GEMV (group 32)
    (300, 1024, 1536, 4, 64, _lib.QMM_PATH_GEMM, 1),      # GEMM, TMA residual chunks
    (300, 1024, 1532, 8, 64, _lib.QMM_PATH_GEMM, 1),      # GEMM, n % 8 != 0: element residual loads
    (256, 3072, 1024, 4, 64, _lib.QMM_PATH_GEMM, 4),      # split-K reduction
])
def test_residual_mul_epilogue(oracle, m, k, n, bits, group, path, splits):
    packed, scales, offsets, bias = random_layer(n, k, bits, group, seed=m + n, bias=True)
    lin = make_linear(packed, scales, offsets, bias, bits, group)
    x = sin_input(m, k)
    r = oracle.f32_to_bf16(np.cos(np.arange(m * n, dtype=np.float64) * 0.11).astype(np.float32).reshape(m, n))
    y = lin.forward_fused(to_dev_u16(x), residual=to_dev_u16(r), residual_mul=True, path=path, splits=splits)
    torch.cuda.synchronize()
    gemm = path == _lib.QMM_PATH_GEMM
    assert_one_rounding(from_dev_bf16(y), _oracle_mul(oracle, x, lin, r, bf16_weights=gemm), oracle)


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


def _rel(got_bf16, ref, oracle):
    d = np.abs(oracle.bf16_to_f32(got_bf16).astype(np.float64) - np.asarray(ref, dtype=np.float64))
    return d.max() / np.abs(ref).max(), d.mean() / np.abs(ref).max()


@pytest.mark.parametrize("m,dim,hidden,bits,chunk", [
    (300, 4096, 12288, 4, 4096),   # the reference DiT's MLP widths (src/dit.rs:32), one chunk
    (333, 1024, 3072, 8, 128),     # several chunks, a ragged last one
    (1, 1024, 3072, 4, 4096),      # a single token: GEMVs
])
def test_swiglu_matches_oracle_composition(oracle, m, dim, hidden, bits, chunk):
    """Each of the three linears of the chunked SwiGLU against the oracle on
    the same inputs, at the per-linear bar (max|d| <= 1e-2 max|ref|,
    mean|d| <= 1e-3 max|ref|); the whole MLP against the oracle's own
    composition at max 1e-2 and mean 2e-3 (three chained linears, each
    rounding its weights to bf16 on the GEMM path)."""
    mlp = _swiglu(dim, hidden, bits, seed=m, chunk=chunk)
    x = sin_input(m, dim)
    xd = to_dev_u16(x)
    y = mlp.forward(xd.reshape(1, m, dim))
    torch.cuda.synchronize()
    assert y.shape == (1, m, dim)
    # the stages on the GPU, unchunked (chunking is checked bit-exactly below)
    g = mlp.gate.forward_fused(xd, activation="silu")
    h = mlp.up.forward_fused(xd, residual=g, residual_mul=True)
    pg, sg, og, _ = _host(mlp.gate)
    g_ref = oracle.linear_f32(x, pg, sg, og, bits, 64)
    g_ref = g_ref / (1.0 + np.exp(-g_ref.astype(np.float64)))
    h_ref = _oracle_mul(oracle, x, mlp.up, from_dev_bf16(g))
    pd, sd, od, _ = _host(mlp.down)
    y_ref = oracle.linear_f32(from_dev_bf16(h), pd, sd, od, bits, 64)
    got_y = from_dev_bf16(y.reshape(m, dim))
    for name, got, ref in (("gate", from_dev_bf16(g), g_ref), ("up*gate", from_dev_bf16(h), h_ref),
                           ("down", got_y, y_ref)):
        mx, mean = _rel(got, ref, oracle)
        assert mx <= 1e-2 and mean <= 1e-3, (name, mx, mean)
    # end to end against the oracle's composition from x alone
    g_o = oracle.f32_to_bf16(g_ref.astype(np.float32))
    h_o = oracle.f32_to_bf16(_oracle_mul(oracle, x, mlp.up, g_o))
    mx, mean = _rel(got_y, oracle.linear_f32(h_o, pd, sd, od, bits, 64), oracle)
    assert mx <= 1e-2 and mean <= 2e-3, (mx, mean)


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
