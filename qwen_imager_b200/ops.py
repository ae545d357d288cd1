"""Callers of the quantized linear beside the DiT block: the SwiGLU MLP.

Mirror of image-forger's `ops::SwiGlu` (src/ops.rs:183-208), the MLP of the
reference's own DiT blocks (src/dit.rs:32, 93) and text encoder
(src/text.rs:231-237): down(silu(gate(x)) * up(x)), in chunks of 4096 tokens
as the reference does to bound the [chunk, hidden] intermediates.

Here the elementwise part is fused into the linears' epilogues: the gate
projection's epilogue applies SiLU, and the up projection's epilogue
multiplies by that result (QMM_EPILOGUE_RESIDUAL_MUL), so each chunk is three
quantized GEMMs and no separate elementwise kernel.  The SiLU-activated gate
is rounded to bf16 once and the product once, where the reference rounds
gate, SiLU, up and product separately.
"""
from __future__ import annotations

from typing import Sequence

import torch

from .quant import Linear, linear
from .weights import VarBuilder

CHUNK = 4096  # tokens per chunk (src/ops.rs:199)


class SwiGlu:
    """gate, up: dim -> hidden; down: hidden -> dim; no biases (src/ops.rs:189-195)."""

    def __init__(self, gate: Linear, up: Linear, down: Linear, chunk: int = CHUNK):
        self.gate, self.up, self.down, self.chunk = gate, up, down, chunk

    @classmethod
    def new(cls, vb: VarBuilder, dim: int, hidden: int, names: Sequence[str]) -> "SwiGlu":
        return cls(linear(vb.pp(names[0]), dim, hidden, False), linear(vb.pp(names[1]), dim, hidden, False),
                   linear(vb.pp(names[2]), hidden, dim, False))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """x [..., tokens, dim] -> [..., tokens, dim]; chunked along the token
        dimension (dim -2), like the reference's narrow(1, start, 4096)."""
        if x.dim() < 2:
            raise ValueError(f"SwiGlu expects [..., tokens, dim], got {tuple(x.shape)}")
        tokens = x.shape[-2]
        outs = []
        for start in range(0, tokens, self.chunk):
            xx = x.narrow(-2, start, min(self.chunk, tokens - start))
            g = self.gate.forward_fused(xx, activation="silu")
            h = self.up.forward_fused(xx, residual=g, residual_mul=True)
            outs.append(self.down.forward(h))
        return outs[0] if len(outs) == 1 else torch.cat(outs, dim=-2)

    __call__ = forward
