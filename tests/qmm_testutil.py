"""Helpers for the GPU parity tests: seeded layers, oracle comparisons."""
import numpy as np
import torch

from oracle import oracle as O


def random_layer(n, k, bits, group=64, seed=0, bias=True):
    """Random packed layer like the reference's `random_layer` (src/quant.rs:705-739):
    random words, scales U(-0.01,0.01), offsets U(-0.05,0.05), bias U(-0.5,0.5)."""
    rng = np.random.default_rng(seed)
    packed = rng.integers(0, 2**32, size=(n, k * bits // 32), dtype=np.uint64).astype(np.uint32)
    scales = O.f32_to_bf16(((rng.random((n, k // group)) - 0.5) * 0.02).astype(np.float32))
    offsets = O.f32_to_bf16(((rng.random((n, k // group)) - 0.5) * 0.1).astype(np.float32))
    b = O.f32_to_bf16(((rng.random(n) - 0.5) * 1.0).astype(np.float32)) if bias else None
    return packed, scales, offsets, b


def sin_input(m, k):
    """x[i] = sin(0.37 i), the reference test's input (src/quant.rs:759)."""
    return O.f32_to_bf16(np.sin(np.arange(m * k, dtype=np.float64) * 0.37).astype(np.float32).reshape(m, k))


def to_dev_u16(a):
    return torch.from_numpy(np.ascontiguousarray(a).astype(np.int16)).view(torch.bfloat16).cuda()


def to_dev_u32(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int32)).view(torch.uint32).cuda()


def from_dev_bf16(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def make_linear(packed, scales, offsets, bias, bits, group):
    from qwen_imager_b200 import Affine, Linear
    n = packed.shape[0]
    k = packed.shape[1] * 32 // bits
    a = Affine(packed=to_dev_u32(packed), scales=to_dev_u16(scales), offsets=to_dev_u16(offsets),
               bias=None if bias is None else to_dev_u16(bias), bits=bits, group=group, input=k)
    return Linear(affine=a)


def rel_errors(got_bf16, ref_f32):
    got = O.bf16_to_f32(got_bf16).astype(np.float64)
    ref = np.asarray(ref_f32, dtype=np.float64)
    scale = np.abs(ref).max()
    d = np.abs(got - ref)
    return d.max() / scale, d.mean() / scale


def bf16_ulp_diff(a_bf16, b_bf16):
    """Distance in bf16 units in the last place (same-sign ordered integers)."""
    def ordered(u):
        u = u.astype(np.int32)
        return np.where(u & 0x8000, -(u & 0x7FFF), u)
    return np.abs(ordered(a_bf16) - ordered(b_bf16))


def assert_one_rounding(got, ref_f32, oracle=O):
    """Within 1 bf16 ulp of the f32 reference, except where f32 accumulation
    order dominates (outputs near zero): there |d| <= 2^-12 max|ref|."""
    ref = oracle.f32_to_bf16(ref_f32)
    ulps = bf16_ulp_diff(got, ref)
    d = np.abs(oracle.bf16_to_f32(got).astype(np.float64) - np.asarray(ref_f32, dtype=np.float64))
    tol = np.abs(ref_f32).max() * 2.0**-12
    bad = (ulps > 1) & (d > tol)
    assert not bad.any(), (int(ulps.max()), float(d[bad].max() / np.abs(ref_f32).max()))
    assert (ulps > 0).mean() < 0.05


def _bits16(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _bits32(t):
    return t.detach().cpu().contiguous().view(torch.int32).numpy().view(np.uint32)


_ACT_CODES = {None: 0, "none": 0, "gelu_tanh": 1, "silu": 2}


_OWN = object()


def oracle_run_linear(lin, x, *, gate=None, residual=None, activation=None, out=None, bias=_OWN):
    """The oracle's fused linear on CPU tensors, with the same signature as the
    stack's CUDA linear: residual + gate * act(x . W^T + bias), rounded once
    (`bias` other than the default replaces the layer's own; None: none)."""
    a = lin.affine
    b = a.bias if bias is _OWN else bias
    m = x.numel() // a.input
    y = O.linear_f32(_bits16(x.reshape(m, a.input)), _bits32(a.packed), _bits16(a.scales),
                     _bits16(a.offsets), a.bits, a.group, None if b is None else _bits16(b.reshape(-1)))
    r = O.epilogue_bf16(y, None if gate is None else _bits16(gate.reshape(-1)),
                        None if residual is None else _bits16(residual.reshape(m, a.output)),
                        _ACT_CODES[activation])
    t = torch.from_numpy(r.view(np.int16)).view(torch.bfloat16).reshape(m, a.output)
    if out is None:
        return t
    out.copy_(t.reshape(out.shape))
    return out
