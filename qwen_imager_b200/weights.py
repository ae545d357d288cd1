"""Weight supply for the quantized linear: a small VarBuilder.

Mirrors the part of Candle's `VarBuilder` that image-forger's `Linear::load`
uses (src/quant.rs:43-77; weights reach it through `cached_builder`,
src/weights.rs:134-202): prefixes (`pp`), `contains_tensor`, typed `get` with a
shape check, and `get_unchecked_dtype`.  Packed uint32 codes are read
unconverted; floating tensors are converted to the builder's dtype, as
`stored_dtype` allows U32 through unchanged (src/weights.rs:171-191).

Tensors stay shared: the same device copy is returned for every `get` of the
same name (one device copy per name, src/weights.rs:171-191).
"""
from __future__ import annotations

import os
import threading
from typing import Dict, Iterable, Mapping, Optional, Sequence

import torch


class WeightError(ValueError):
    """A missing tensor or a shape mismatch (Candle's VarBuilder errors)."""


class VarBuilder:
    def __init__(self, tensors: Mapping[str, torch.Tensor], dtype: torch.dtype = torch.bfloat16,
                 device: torch.device | str = "cuda", prefix: str = "",
                 _cache: Optional[Dict] = None, _lock: Optional[threading.Lock] = None):
        self._tensors = tensors
        self._dtype = dtype
        self._device = torch.device(device)
        self._prefix = prefix
        self._cache = {} if _cache is None else _cache
        self._lock = threading.Lock() if _lock is None else _lock

    # -- construction ------------------------------------------------------
    @classmethod
    def from_tensors(cls, tensors: Mapping[str, torch.Tensor], dtype: torch.dtype = torch.bfloat16,
                     device: torch.device | str = "cuda") -> "VarBuilder":
        return cls(dict(tensors), dtype, device)

    @classmethod
    def from_safetensors(cls, paths: str | Sequence[str], dtype: torch.dtype = torch.bfloat16,
                         device: torch.device | str = "cuda") -> "VarBuilder":
        """Memory-maps one or more .safetensors files (MLX packs store `weight`
        as U32 next to bf16 `scales` and `biases`)."""
        from safetensors.torch import load_file

        if isinstance(paths, (str, os.PathLike)):
            paths = [paths]
        tensors: Dict[str, torch.Tensor] = {}
        for p in paths:
            tensors.update(load_file(str(p), device="cpu"))
        return cls(tensors, dtype, device)

    def pp(self, name: str) -> "VarBuilder":
        prefix = f"{self._prefix}.{name}" if self._prefix else name
        return VarBuilder(self._tensors, self._dtype, self._device, prefix, self._cache, self._lock)

    def to_dtype(self, dtype: torch.dtype) -> "VarBuilder":
        return VarBuilder(self._tensors, dtype, self._device, self._prefix, {}, self._lock)

    # -- queries -----------------------------------------------------------
    @property
    def dtype(self) -> torch.dtype:
        return self._dtype

    @property
    def device(self) -> torch.device:
        return self._device

    def prefix(self) -> str:
        return self._prefix

    def _path(self, name: str) -> str:
        return f"{self._prefix}.{name}" if self._prefix else name

    def contains_tensor(self, name: str) -> bool:
        return self._path(name) in self._tensors

    def names(self) -> Iterable[str]:
        return self._tensors.keys()

    def get_unchecked_dtype(self, name: str, dtype: torch.dtype) -> torch.Tensor:
        path = self._path(name)
        if path not in self._tensors:
            raise WeightError(f"cannot find tensor {path}")
        key = (path, dtype, str(self._device))
        with self._lock:
            t = self._cache.get(key)
            if t is None:
                src = self._tensors[path]
                if dtype == torch.uint32 or src.dtype == torch.uint32:
                    if src.dtype not in (torch.uint32, torch.int32):
                        raise WeightError(f"{path}: expected packed uint32 codes, got {src.dtype}")
                    t = src.contiguous().to(self._device)
                else:
                    t = src.to(device=self._device, dtype=dtype).contiguous()
                self._cache[key] = t
            return t

    def get(self, shape, name: str) -> torch.Tensor:
        t = self.get_unchecked_dtype(name, self._dtype)
        shape = (shape,) if isinstance(shape, int) else tuple(shape)
        if tuple(t.shape) != shape:
            raise WeightError(f"shape mismatch for {self._path(name)}, expected {shape}, got {tuple(t.shape)}")
        return t
