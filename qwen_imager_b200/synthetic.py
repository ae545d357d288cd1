"""Seeded synthetic layers and inputs for benchmarks.

No checkpoint or dataset is available offline, so benchmarks use random
weights quantized with the MLX affine scheme (per group of `group` inputs:
scale = (max - min) / (2^bits - 1), bias = min, stored bf16,
q = clamp(round((w - bias) / scale), 0, 2^bits - 1)), packed little-end-first
into uint32 words -- the layout `Linear::load` consumes (src/quant.rs:43-77).
Generation runs on the GPU with torch's seeded generators.
"""
from __future__ import annotations

from typing import Optional

import torch

from .quant import Affine, Linear


def quantize_affine(w: torch.Tensor, bits: int, group: int = 64):
    """Returns (packed uint32 [n, k*bits/32], scales bf16 [n, k/group], biases bf16 [n, k/group])."""
    n, k = w.shape
    levels = (1 << bits) - 1
    per_word = 32 // bits
    wg = w.float().reshape(n, k // group, group)
    lo = wg.amin(-1)
    hi = wg.amax(-1)
    scales = ((hi - lo) / levels).to(torch.bfloat16)
    biases = lo.to(torch.bfloat16)
    s = scales.float().unsqueeze(-1)
    b = biases.float().unsqueeze(-1)
    q = torch.where(s != 0, torch.round((wg - b) / torch.where(s != 0, s, torch.ones_like(s))),
                    torch.zeros_like(wg))
    q = q.clamp_(0, levels).to(torch.int64).reshape(n, k // per_word, per_word)
    del wg
    shifts = torch.arange(per_word, device=w.device, dtype=torch.int64) * bits
    words = (q << shifts).sum(-1)
    words = torch.where(words >= 2**31, words - 2**32, words).to(torch.int32)
    return words.view(torch.uint32).contiguous(), scales.contiguous(), biases.contiguous()


def gaussian(shape, std: float, generator: torch.Generator, device) -> torch.Tensor:
    return torch.randn(shape, generator=generator, device=device, dtype=torch.float32) * std


def quantized_linear(n: int, k: int, bits: int, *, seed: int, group: int = 64, std: float = 0.02,
                     bias_std: Optional[float] = None, device="cuda") -> Linear:
    """A layer with W ~ N(0, std^2) quantized by `quantize_affine`, optional bias ~ N(0, bias_std^2)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    w = gaussian((n, k), std, g, device)
    packed, scales, biases = quantize_affine(w, bits, group)
    del w
    bias = gaussian((n,), bias_std, g, device).to(torch.bfloat16) if bias_std else None
    return Linear(affine=Affine(packed=packed, scales=scales, offsets=biases, bias=bias, bits=bits,
                                group=group, input=k))


def random_codes_linear(n: int, k: int, bits: int, *, seed: int, group: int = 64, device="cuda") -> Linear:
    """Random codes, scales U(-0.01, 0.01), offsets U(-0.05, 0.05): the reference
    test's `random_layer` (src/quant.rs:705-739).  Cheap enough for the 20B-parameter
    DiT stack, where quantizing Gaussian weights would only cost time."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    words = k * bits // 32
    packed = torch.randint(-2**31, 2**31 - 1, (n, words), generator=g, device=device,
                           dtype=torch.int32).view(torch.uint32)
    scales = ((torch.rand((n, k // group), generator=g, device=device) - 0.5) * 0.02).to(torch.bfloat16)
    offsets = ((torch.rand((n, k // group), generator=g, device=device) - 0.5) * 0.1).to(torch.bfloat16)
    return Linear(affine=Affine(packed=packed, scales=scales, offsets=offsets, bias=None, bits=bits,
                                group=group, input=k))
