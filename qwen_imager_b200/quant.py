"""Linear layers stored dense or as MLX affine-quantized weights.

Host-side mirror of image-forger's `quant::Linear` (src/quant.rs:26-124) over
the libqmm C ABI.  MLX packs `bits`-wide unsigned codes little-end-first into
uint32 words along the input dimension; each group of `group` inputs has a
bf16 scale and offset (`biases`): w = scale * q + offset.  The layer's own
additive bias is `bias`.

Same names, argument meanings and failure behaviour as the reference:
  Linear.load(vb, input, output, bias)   src/quant.rs:43-77
  Linear.dense()                         src/quant.rs:80-85
  Linear.device / Linear.dtype           src/quant.rs:87-100
  Linear.forward(x)                      src/quant.rs:115-124, 139-161
  linear(vb, input, output, bias)        src/ops.rs:8-10
Quantized layers stay packed on the GPU; forward runs the fused CUDA kernels
(GEMV for m <= 16, tcgen05 GEMM otherwise) with the bias fused into the
epilogue.  Layouts the kernels do not cover (2-bit GEMMs, odd group sizes)
dequantize on the GPU and run a dense GEMM, as the reference falls back to
`self.dense()?.forward(x)` (src/quant.rs:121).  There is no CPU path: a CPU
tensor is an error.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib
from ._lib import QmmEpilogue, QmmError, QmmWeight
from .weights import VarBuilder, WeightError

ACTIVATIONS = {None: _lib.QMM_ACT_NONE, "none": _lib.QMM_ACT_NONE,
               "gelu_tanh": _lib.QMM_ACT_GELU_TANH, "silu": _lib.QMM_ACT_SILU}

# Default of the epilogue-bias argument: the layer's own bias.
OWN_BIAS = object()


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


_workspaces = {}


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Split-K scratch for the current stream of `device`, grown on demand.
    Kernels on one stream run in order, so one buffer per stream suffices."""
    key = (device.index, torch.cuda.current_stream(device).cuda_stream)
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _workspaces[key] = buf
    return buf


def _require_cuda(t: torch.Tensor, what: str) -> None:
    if t.device.type != "cuda":
        raise QmmError(_lib.QMM_ERR_CUDA, f"{what} is on {t.device}; the quantized linear runs on CUDA only")


@dataclass
class Affine:
    """Packed weights of one layer (src/quant.rs:31-39)."""

    packed: torch.Tensor   # uint32 [output, input * bits / 32]
    scales: torch.Tensor   # bf16 [output, groups]
    offsets: torch.Tensor  # bf16 [output, groups]  (MLX "biases")
    bias: Optional[torch.Tensor]  # bf16 [output]
    bits: int
    group: int
    input: int

    @property
    def output(self) -> int:
        return int(self.packed.shape[0])

    def c_weight(self) -> QmmWeight:
        return QmmWeight(self.packed.data_ptr(), self.scales.data_ptr(), self.offsets.data_ptr(),
                         self.output, self.input, self.bits, self.group)

    def dequantize(self, dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
        """Dense [output, input] weights (src/quant.rs:163-178), bit-exact."""
        if dtype not in (torch.bfloat16, torch.float32):
            raise QmmError(_lib.QMM_ERR_INVALID_ARGUMENT, f"dequantize does not support {dtype}")
        _require_cuda(self.packed, "packed weight")
        out = torch.empty((self.output, self.input), dtype=dtype, device=self.packed.device)
        w = self.c_weight()
        code = _lib.QMM_DTYPE_F32 if dtype == torch.float32 else _lib.QMM_DTYPE_BF16
        _lib.check(_lib.load().qmm_dequantize(ctypes.byref(w), out.data_ptr(), code,
                                              _stream_handle(out.device)))
        return out

    def fused_eligible(self, x: torch.Tensor) -> bool:
        """Counterpart of `Affine::fused` (src/quant.rs:129-137) for this library."""
        return (x.device.type == "cuda" and x.dtype == self.scales.dtype == torch.bfloat16
                and x.numel() > 0)

    def run(self, x2d: torch.Tensor, *, gate: Optional[torch.Tensor] = None,
            residual: Optional[torch.Tensor] = None, activation: Optional[str] = None,
            out: Optional[torch.Tensor] = None, path: int = _lib.QMM_PATH_AUTO,
            splits: Optional[int] = None, bias=OWN_BIAS, residual_mul: bool = False) -> torch.Tensor:
        """y [m, output] = residual + gate * act(x2d . W^T + bias)
        (residual * (...) with residual_mul).

        The GEMM (m > 16 under QMM_PATH_AUTO, or QMM_PATH_GEMM) splits K when
        the output tiles alone would leave most SMs idle; `splits` forces a
        split count (1 = none).  The f32 workspace comes from a per-device,
        per-stream cache.  `bias` replaces the layer's own bias in the
        epilogue (None: no bias), e.g. for a row-parallel shard whose bias is
        added once after the reduction."""
        bias = self.bias if bias is OWN_BIAS else bias
        m = int(x2d.shape[0])
        n = self.output
        if out is None:
            out = torch.empty((m, n), dtype=torch.bfloat16, device=x2d.device)
        if residual is not None:
            residual = residual.reshape(m, n)
            if not residual.is_contiguous() or residual.dtype != torch.bfloat16:
                residual = residual.to(torch.bfloat16).contiguous()
        if gate is not None:
            gate = gate.reshape(n).to(torch.bfloat16).contiguous()
        if bias is not None:
            bias = bias.reshape(n).to(torch.bfloat16).contiguous()
        act_code = ACTIVATIONS[activation] | (_lib.QMM_EPILOGUE_RESIDUAL_MUL if residual_mul else 0)
        ep = QmmEpilogue(_ptr(bias), _ptr(gate), _ptr(residual), act_code)
        w = self.c_weight()
        lib = _lib.load()
        gemm = path == _lib.QMM_PATH_GEMM or (path == _lib.QMM_PATH_AUTO and m > 16)
        if path == _lib.QMM_PATH_GEMM_F16:
            gemm, splits = False, 1  # one launch of the fp16-operand GEMM (no split-K)
        if gemm and m > 0:
            sp = lib.qmm_gemm_splits(ctypes.byref(w), m) if splits is None else int(splits)
            if sp > 1:
                nbytes = int(lib.qmm_splitk_workspace_bytes(ctypes.byref(w), m, sp))
                ws = _workspace(x2d.device, nbytes)
                status = lib.qmm_linear_splitk(ctypes.byref(w), x2d.data_ptr(), m, ctypes.byref(ep),
                                               out.data_ptr(), sp, ws.data_ptr(), nbytes,
                                               _stream_handle(x2d.device))
                if status == _lib.QMM_ERR_UNSUPPORTED and path == _lib.QMM_PATH_AUTO:
                    return self._dense_fallback(x2d, gate, residual, activation, out, bias, residual_mul)
                _lib.check(status)
                return out
        status = lib.qmm_linear_ex(ctypes.byref(w), x2d.data_ptr(), m, ctypes.byref(ep),
                                   out.data_ptr(), path, _stream_handle(x2d.device))
        if status == _lib.QMM_ERR_UNSUPPORTED and path == _lib.QMM_PATH_AUTO:
            return self._dense_fallback(x2d, gate, residual, activation, out, bias, residual_mul)
        _lib.check(status)
        return out

    def _dense_fallback(self, x2d, gate, residual, activation, out, bias, residual_mul=False):
        # Dequantize on the GPU, dense GEMM, then the epilogue: the reference's
        # `self.dense()?.forward(x)` for layouts the fused kernel skips.
        t = torch.nn.functional.linear(x2d.float(), self.dequantize(torch.float32),
                                       None if bias is None else bias.float())
        if activation == "gelu_tanh":
            t = torch.nn.functional.gelu(t, approximate="tanh")
        elif activation == "silu":
            t = torch.nn.functional.silu(t)
        if gate is not None:
            t = t * gate.float()
        if residual is not None:
            t = residual.float() * t if residual_mul else residual.float() + t
        out.copy_(t.to(out.dtype))
        return out


class Linear:
    """Dense or MLX-quantized linear layer (src/quant.rs:26-29)."""

    def __init__(self, dense_weight: Optional[torch.Tensor] = None,
                 dense_bias: Optional[torch.Tensor] = None, affine: Optional[Affine] = None):
        self._weight = dense_weight
        self._bias = dense_bias
        self.affine = affine

    # -- construction -------------------------------------------------------
    @classmethod
    def load(cls, vb: VarBuilder, input: int, output: int, bias: bool) -> "Linear":
        """Loads `weight` (and `bias`), quantized when the checkpoint has `scales`."""
        if not vb.contains_tensor("scales"):
            w = vb.get((output, input), "weight")
            b = vb.get(output, "bias") if bias else None
            return cls(dense_weight=w, dense_bias=b)
        scales = vb.get_unchecked_dtype("scales", vb.dtype)
        if scales.dim() != 2:
            raise WeightError(f"{vb.prefix()}: scales {tuple(scales.shape)} is not a matrix")
        rows, groups = scales.shape
        if rows != output or groups == 0 or input % groups != 0:
            raise WeightError(f"{vb.prefix()}: scales {tuple(scales.shape)} do not match a "
                              f"{input}->{output} linear")
        packed = vb.get_unchecked_dtype("weight", torch.uint32)
        if packed.dim() != 2:
            raise WeightError(f"{vb.prefix()}: packed weight {tuple(packed.shape)} is not a matrix")
        try:
            bits, group = _lib.infer_layout(input, output, tuple(scales.shape), tuple(packed.shape))
        except QmmError as exc:
            raise WeightError(f"{vb.prefix()}: packed weight {tuple(packed.shape)} is not 2-, 4- "
                              f"or 8-bit for {input} inputs") from exc
        return cls(affine=Affine(
            packed=packed,
            scales=_as_bf16(scales, vb, "scales"),
            offsets=_as_bf16(vb.get((output, groups), "biases"), vb, "biases"),
            bias=vb.get(output, "bias") if bias else None,
            bits=bits,
            group=group,
            input=input,
        ))

    # -- properties ---------------------------------------------------------
    @property
    def is_quantized(self) -> bool:
        return self.affine is not None

    @property
    def device(self) -> torch.device:
        return self.affine.scales.device if self.affine else self._weight.device

    @property
    def dtype(self) -> torch.dtype:
        """Floating-point dtype of the layer's weights and outputs."""
        return self.affine.scales.dtype if self.affine else self._weight.dtype

    def dense(self):
        """(weight, bias) of the equivalent dense layer; quantized layers allocate."""
        if self.affine is None:
            return self._weight, self._bias
        return self.affine.dequantize(self.affine.scales.dtype), self.affine.bias

    # -- forward ------------------------------------------------------------
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.forward_fused(x)

    __call__ = forward

    def forward_fused(self, x: torch.Tensor, *, gate: Optional[torch.Tensor] = None,
                      residual: Optional[torch.Tensor] = None,
                      activation: Optional[str] = None, path: int = _lib.QMM_PATH_AUTO,
                      out: Optional[torch.Tensor] = None, splits: Optional[int] = None,
                      bias=OWN_BIAS, residual_mul: bool = False, operands: str = "bf16") -> torch.Tensor:
        """residual + gate * act(x . W^T + bias) with any leading dims on x.

        gate: [output] per-feature multiplier; residual: same shape as the output;
        bias: replaces the layer's own bias (None: no bias); residual_mul: the
        residual multiplies instead, residual * (gate * act(x . W^T + bias)).

        bf16 inputs run the fused kernels.  operands="fp16" (or an fp16 x) runs
        the GEMM with fp16 operands (QMM_PATH_GEMM_F16): x converted to fp16,
        the weights dequantized to fp16, closer to the reference's f32 weights;
        the result stays bf16.  f32 inputs take the reference's non-fused route
        (src/quant.rs:121): the weight dequantized to f32 (bit-exact) and a
        dense f32 GEMM, with an f32 result.
        """
        if operands not in ("bf16", "fp16"):
            raise QmmError(_lib.QMM_ERR_INVALID_ARGUMENT, f"operands must be bf16 or fp16, not {operands!r}")
        if activation not in ACTIVATIONS:
            raise QmmError(_lib.QMM_ERR_INVALID_ARGUMENT, f"unknown activation {activation!r}")
        *lead, k = x.shape
        if self.affine is None:
            _require_cuda(x, "input")
            t = torch.nn.functional.linear(x, self._weight, self._bias if bias is OWN_BIAS else bias)
            return _epilogue_torch(t, gate, residual, activation, residual_mul)
        a = self.affine
        if k != a.input:
            raise QmmError(_lib.QMM_ERR_BAD_SHAPE, f"quantized linear expects {a.input} inputs, got {k}")
        _require_cuda(x, "input")
        m = x.numel() // k if k else 0
        if x.dtype == torch.float32:
            b = a.bias if bias is OWN_BIAS else bias
            t = torch.nn.functional.linear(x.reshape(m, k), a.dequantize(torch.float32),
                                           None if b is None else b.float())
            t = _epilogue_torch(t, gate, None if residual is None else residual.reshape(m, a.output),
                                activation, residual_mul)
            if out is not None:
                out.view(m, a.output).copy_(t)
                return out
            return t.reshape(*lead, a.output)
        if x.dtype == torch.float16 or operands == "fp16":
            if x.dtype not in (torch.bfloat16, torch.float16):
                raise QmmError(_lib.QMM_ERR_INVALID_ARGUMENT, f"fp16 operands from a {x.dtype} input")
            x = x.to(torch.float16)
            path = _lib.QMM_PATH_GEMM_F16
            splits = 1
        elif x.dtype != torch.bfloat16:
            raise QmmError(_lib.QMM_ERR_INVALID_ARGUMENT,
                           f"quantized linear computes in bf16 (or f32 through dequantization); got {x.dtype}")
        x2d = x.reshape(m, k)
        if not x2d.is_contiguous() or x2d.data_ptr() % 16:
            x2d = x2d.contiguous()
        if out is not None:
            out = out.view(m, a.output)
        y = a.run(x2d, gate=gate, residual=residual, activation=activation, out=out, path=path, splits=splits,
                  bias=bias, residual_mul=residual_mul)
        return y.reshape(*lead, a.output)


def _epilogue_torch(t, gate, residual, activation, residual_mul):
    """The fused epilogue's arithmetic with torch ops, in t's dtype."""
    if activation == "gelu_tanh":
        t = torch.nn.functional.gelu(t, approximate="tanh")
    elif activation == "silu":
        t = torch.nn.functional.silu(t)
    if gate is not None:
        t = t * gate.to(t.dtype)
    if residual is not None:
        r = residual.to(t.dtype)
        t = r * t if residual_mul else r + t
    return t


def _as_bf16(t: torch.Tensor, vb: VarBuilder, name: str) -> torch.Tensor:
    """Scales and offsets as the kernels read them (bf16).  MLX stores them in
    bf16, so a builder in another float dtype (e.g. f32, as the reference's
    f32 tests load them) converts back exactly; values that bf16 cannot hold
    are an error rather than a silent rounding."""
    if t.dtype == torch.bfloat16:
        return t
    b = t.to(torch.bfloat16)
    if not torch.equal(b.to(t.dtype), t):
        raise WeightError(f"{vb.prefix()}: {name} in {t.dtype} are not exact in bf16, which the kernels read")
    return b


def linear(vb: VarBuilder, input: int, output: int, bias: bool) -> Linear:
    """Dense or MLX-quantized, depending on the checkpoint's tensors (src/ops.rs:8-10)."""
    return Linear.load(vb, input, output, bias)


def device_error(device: Optional[torch.device] = None) -> int:
    """Reads and clears the library's device-side timeout word (0 = none)."""
    dev = torch.device("cuda") if device is None else device
    code = ctypes.c_uint32()
    status = _lib.load().qmm_device_error(_stream_handle(dev), ctypes.byref(code))
    if status not in (_lib.QMM_OK, _lib.QMM_ERR_TIMEOUT):
        _lib.check(status)
    return int(code.value)
