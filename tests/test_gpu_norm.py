"""Fused LayerNorm + adaLN modulation (qmm_layernorm_modulate) against an f32
torch reference of the same op (one bf16 rounding of the f32 result)."""
import pytest
import torch
import torch.nn.functional as F

from qwen_imager_b200 import _lib

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,hidden", [(1, 256), (37, 3072), (4352, 3072), (5, 4096), (300, 768)])
def test_layernorm_modulate_matches_f32_reference(rows, hidden):
    g = torch.Generator(device="cuda").manual_seed(rows + hidden)
    x = (torch.randn((rows, hidden), generator=g, device="cuda") * 3 + 0.5).to(torch.bfloat16)
    shift = torch.randn((hidden,), generator=g, device="cuda").to(torch.bfloat16)
    scale = (torch.randn((hidden,), generator=g, device="cuda") * 0.2).to(torch.bfloat16)
    out = torch.empty_like(x)
    lib = _lib.load()
    _lib.check(lib.qmm_layernorm_modulate(x.data_ptr(), rows, hidden, shift.data_ptr(), scale.data_ptr(), 1e-6,
                                          out.data_ptr(), torch.cuda.current_stream().cuda_stream))
    ref = F.layer_norm(x.float(), (hidden,), eps=1e-6) * (1 + scale.float()) + shift.float()
    d = (out.float() - ref).abs()
    # one bf16 rounding of the f32 value, up to f32 summation order
    assert (d <= ref.abs() * 2.0**-8 + 1e-5).all(), float(d.max())


def test_layernorm_modulate_in_place_and_errors():
    lib = _lib.load()
    x = torch.randn((64, 512), device="cuda").to(torch.bfloat16)
    shift = torch.zeros((512,), device="cuda", dtype=torch.bfloat16)
    scale = torch.zeros((512,), device="cuda", dtype=torch.bfloat16)
    ref = F.layer_norm(x.float(), (512,), eps=1e-6)
    st = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.qmm_layernorm_modulate(x.data_ptr(), 64, 512, shift.data_ptr(), scale.data_ptr(), 1e-6,
                                          x.data_ptr(), st))
    assert ((x.float() - ref).abs() <= ref.abs() * 2.0**-8 + 1e-5).all()
    assert lib.qmm_layernorm_modulate(x.data_ptr(), 64, 500, shift.data_ptr(), scale.data_ptr(), 1e-6,
                                      x.data_ptr(), st) == _lib.QMM_ERR_UNSUPPORTED


def _rln(lib, x, delta, bias, gate, shift, scale, out):
    rows, hidden = x.shape
    p = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    return lib.qmm_residual_layernorm_modulate(x.data_ptr(), rows, hidden, delta.data_ptr(), p(bias), p(gate),
                                               p(shift), p(scale), 1e-6, p(out),
                                               torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("rows,hidden", [(1, 256), (2112, 3072), (37, 3072), (300, 1024), (5, 4096)])
@pytest.mark.parametrize("with_bias,with_gate,with_norm", [(True, True, True), (True, False, True),
                                                           (False, False, True), (True, True, False)])
def test_residual_layernorm_modulate_matches_f32_reference(rows, hidden, with_bias, with_gate, with_norm):
    g = torch.Generator(device="cuda").manual_seed(rows * 7 + hidden)
    r = lambda *s, sd=1.0: (torch.randn(s, generator=g, device="cuda") * sd).to(torch.bfloat16)  # noqa: E731
    x, delta = r(rows, hidden, sd=2.0), r(rows, hidden, sd=0.5)
    bias = r(hidden, sd=0.1) if with_bias else None
    gate = r(hidden) if with_gate else None
    shift, scale = r(hidden), r(hidden, sd=0.2)
    out = torch.empty_like(x) if with_norm else None
    x0 = x.clone()
    lib = _lib.load()
    _lib.check(_rln(lib, x, delta, bias, gate, shift, scale, out))
    want = x0.float() + delta.float()
    if bias is not None:
        want = want + bias.float() * (gate.float() if gate is not None else 1.0)
    # x: one bf16 rounding of the f32 sum
    assert torch.equal(x, want.to(torch.bfloat16)), float((x.float() - want).abs().max())
    if with_norm:
        ref = F.layer_norm(x.float(), (hidden,), eps=1e-6) * (1 + scale.float()) + shift.float()
        d = (out.float() - ref).abs()
        assert (d <= ref.abs() * 2.0**-8 + 1e-5).all(), float(d.max())


def test_residual_layernorm_modulate_rejects_bad_arguments():
    lib = _lib.load()
    x = torch.zeros((8, 512), device="cuda", dtype=torch.bfloat16)
    d = torch.zeros_like(x)
    v = torch.zeros((512,), device="cuda", dtype=torch.bfloat16)
    assert _rln(lib, x, d, None, v, v, v, torch.empty_like(x)) == _lib.QMM_ERR_INVALID_ARGUMENT  # gate without bias
    assert _rln(lib, x, x, v, None, v, v, None) == _lib.QMM_ERR_INVALID_ARGUMENT  # delta aliases x
    assert _rln(lib, x, d, v, None, v, v, x) == _lib.QMM_ERR_INVALID_ARGUMENT  # out aliases x
    y = torch.zeros((8, 640), device="cuda", dtype=torch.bfloat16)
    assert _rln(lib, y, torch.zeros_like(y), None, None, None, None, None) == _lib.QMM_ERR_UNSUPPORTED
