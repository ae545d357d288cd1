"""Regenerates tests/golden/mlx_quantized.npz from the reference's own fixture.

The reference ships `tests/fixtures/quantized.safetensors`, written by MLX 0.32.3
(`mlx.core.quantize`, group size 64, 4 and 8 bits; see the reference's
tests/fixtures/README.md).  Its tensors are the golden vectors for the
quantized linear: packed codes, bf16 scales/biases, MLX's own dequantized
weights and MLX's quantized_matmul output.  This script copies them, unchanged,
into a numpy archive (bf16 as raw uint16 bits) so that the tests can run where
the reference tree is absent.

Usage: python tests/golden/make_golden.py <reference checkout>
"""
import os
import sys

import numpy as np
import torch
from safetensors.torch import load_file


def main() -> None:
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden.py <reference checkout (the directory holding tests/fixtures)>")
    ref = sys.argv[1]
    src = os.path.join(ref, "tests", "fixtures", "quantized.safetensors")
    tensors = load_file(src)
    out = {}
    for name, t in sorted(tensors.items()):
        if t.dtype == torch.bfloat16:
            out[name] = t.contiguous().view(torch.int16).numpy().view(np.uint16)
        elif t.dtype == torch.uint32:
            out[name] = t.contiguous().view(torch.int32).numpy().view(np.uint32)
        else:
            raise SystemExit(f"unexpected dtype {t.dtype} for {name}")
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "mlx_quantized.npz")
    np.savez_compressed(dst, **out)
    print(f"wrote {dst}: {', '.join(f'{k}{list(v.shape)}' for k, v in out.items())}")


if __name__ == "__main__":
    main()
