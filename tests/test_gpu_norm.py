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
