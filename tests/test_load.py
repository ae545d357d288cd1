"""`Linear::load` semantics (src/quant.rs:43-77) on the golden fixture, on the
CPU: the reference test `dense_weights_load_unchanged_and_bad_packing_is_rejected`
(src/quant.rs:794-808) restated."""
import numpy as np
import pytest
import torch

from qwen_imager_b200 import Linear, VarBuilder, WeightError


def as_torch(golden):
    out = {}
    for k, v in golden.items():
        if v.dtype == np.uint16:
            out[k] = torch.from_numpy(v.astype(np.int16)).view(torch.bfloat16)
        else:
            out[k] = torch.from_numpy(v.view(np.int32)).view(torch.uint32)
    return out


def test_mlx_pack_loads_as_affine(golden):
    vb = VarBuilder.from_tensors(as_torch(golden), torch.bfloat16, "cpu")
    for bits in (4, 8):
        lin = Linear.load(vb.pp(f"q{bits}"), 192, 96, False)
        assert lin.is_quantized
        assert lin.affine.bits == bits and lin.affine.group == 64
        assert lin.dtype == torch.bfloat16
        assert lin.affine.packed.dtype == torch.uint32


def test_dense_weights_load_unchanged_and_bad_packing_is_rejected(golden):
    data = as_torch(golden)
    data["dense.weight"] = data["q4.dequantized"].clone()
    vb = VarBuilder.from_tensors(data, torch.bfloat16, "cpu")
    dense = Linear.load(vb.pp("dense"), 192, 96, False)
    assert not dense.is_quantized
    assert torch.equal(dense.dense()[0], data["q4.dequantized"])
    with pytest.raises(WeightError):
        Linear.load(vb.pp("q4"), 128, 96, False)
    data["q4.weight"] = data["q4.weight"][:, :20].contiguous()
    vb = VarBuilder.from_tensors(data, torch.bfloat16, "cpu")
    with pytest.raises(WeightError):
        Linear.load(vb.pp("q4"), 192, 96, False)


def test_missing_bias_is_an_error(golden):
    vb = VarBuilder.from_tensors(as_torch(golden), torch.bfloat16, "cpu")
    with pytest.raises(WeightError):
        Linear.load(vb.pp("q4"), 192, 96, True)


def test_safetensors_round_trip(tmp_path, golden):
    from safetensors.torch import save_file
    path = tmp_path / "pack.safetensors"
    save_file({k: v.contiguous() for k, v in as_torch(golden).items()}, str(path))
    vb = VarBuilder.from_safetensors(str(path), torch.bfloat16, "cpu")
    lin = Linear.load(vb.pp("q8"), 192, 96, False)
    assert lin.affine.bits == 8
    assert torch.equal(lin.affine.packed.view(torch.int32), as_torch(golden)["q8.weight"].view(torch.int32))


def test_cpu_forward_is_refused(golden):
    from qwen_imager_b200 import QmmError
    vb = VarBuilder.from_tensors(as_torch(golden), torch.bfloat16, "cpu")
    lin = Linear.load(vb.pp("q4"), 192, 96, False)
    x = as_torch(golden)["x"]
    with pytest.raises(QmmError):
        lin.forward(x)
