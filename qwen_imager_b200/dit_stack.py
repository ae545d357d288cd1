"""Tensor-parallel dual-stream MMDiT linear stack over the quantized linear.

The caller of the quantized linear in image-forger is the DiT block
(src/dit.rs:36-94): per block, a modulation linear on the timestep embedding
(src/dit.rs:279, m = 1), q/k/v projections of the modulated, normalised
hidden state (src/dit.rs:51-62), attention, the output projection with a
gated residual (src/dit.rs:88-91) and a gated feed-forward residual
(src/dit.rs:92-93, src/ops.rs:196-207).  This module runs that linear
skeleton in the dual-stream, hidden-3072 form of the 60-block benchmark stack
(image and text streams with their own weights, joint attention over both):

  mod   = Linear(3072 -> 18432)(silu(temb))          per stream, m = 1
  shift1, scale1, gate1, shift2, scale2, gate2 = mod.chunk(6)
  n     = layer_norm(x) * (1 + scale1) + shift1
  q,k,v = Linear(3072 -> 9216)(n)                     24 heads x 128
  a     = attention(q, k, v) over the image and text tokens together
  x     = x + gate1 * Linear(3072 -> 3072)(a)
  n     = layer_norm(x) * (1 + scale2) + shift2
  x     = x + gate2 * Linear(12288 -> 3072)(gelu_tanh(Linear(3072 -> 12288)(n)))

Tensor parallelism over `world` ranks (one process per GPU):
  * q/k/v and FFN-up are column-parallel: each rank holds 24/world heads
    (its q, k and v columns, contiguous) and 12288/world FFN features;
  * out and FFN-down are row-parallel: each rank holds a K slice, whole
    scale groups, and computes a partial product;
  * the partials meet in one NCCL all-reduce (sum, bf16) of the joint
    [m_img + m_txt, 3072] hidden state per row-parallel layer.  Because
    x + g * (sum_r P_r + b) = sum_r (g * P_r) + (x + g * b), every rank applies
    the gate in its epilogue and only rank 0 adds the bias and the residual,
    so the reduced buffer is the next hidden state with no extra pass;
  * the modulation GEMV, the norms and the attention of a rank's heads need
    no exchange (the GEMV is replicated: 32 MB per rank at 4-bit).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Callable, List, Optional

import torch
import torch.nn.functional as F

from . import _lib
from .quant import Affine, Linear, _stream_handle

# ----------------------------------------------------------------- shapes


@dataclass(frozen=True)
class StackConfig:
    """Shape of the dual-stream stack (hidden 3072, 24 heads of 128)."""

    img_tokens: int
    txt_tokens: int
    bits: int
    blocks: int = 60
    hidden: int = 3072
    heads: int = 24
    head_dim: int = 128
    ffn: int = 12288
    group: int = 64

    @property
    def tokens(self) -> int:
        return self.img_tokens + self.txt_tokens

    @property
    def mod_features(self) -> int:
        return 6 * self.hidden

    def check_world(self, world: int) -> None:
        if self.heads % world or self.ffn % world or self.hidden % world:
            raise ValueError(f"{world} ranks do not divide {self.heads} heads / {self.ffn} features")
        # Inputs of the row-parallel shards: out-proj and FFN-down.
        for k in (self.heads * self.head_dim // world, self.ffn // world):
            if k % self.group or (k * self.bits) % 32:
                raise ValueError(f"a {k}-input shard does not hold whole {self.group}-groups")

    def linear_flops_per_block(self) -> float:
        h, f, m = self.hidden, self.ffn, self.tokens
        per_token = 2.0 * h * (3 * h) + 2.0 * h * h + 2.0 * h * f + 2.0 * f * h
        return per_token * m + 2 * 2.0 * h * self.mod_features

    def attention_flops_per_block(self) -> float:
        # QK^T and PV over the joint sequence, all heads.
        return 4.0 * self.tokens * self.tokens * self.heads * self.head_dim


STACKS = {
    # 1024x1024 image: 4096 image tokens + 256 text tokens, 4-bit weights.
    "dit_1024_4bit": StackConfig(img_tokens=4096, txt_tokens=256, bits=4),
    # 2048x2048 image: 16384 image tokens + 512 text tokens, 8-bit weights.
    "dit_2048_8bit": StackConfig(img_tokens=16384, txt_tokens=512, bits=8),
}

# ----------------------------------------------------------------- sharding


def _slice_affine(a: Affine, rows: Optional[torch.Tensor] = None, k0: int = 0, k1: Optional[int] = None,
                  keep_bias: bool = True) -> Affine:
    k1 = a.input if k1 is None else k1
    per_word = 32 // a.bits
    if k0 % a.group or k1 % a.group or k0 % per_word or k1 % per_word:
        raise ValueError(f"input slice [{k0}, {k1}) splits a {a.group}-group or a packed word")
    packed = a.packed[:, k0 // per_word:k1 // per_word]
    scales = a.scales[:, k0 // a.group:k1 // a.group]
    offsets = a.offsets[:, k0 // a.group:k1 // a.group]
    bias = a.bias if keep_bias else None
    if rows is not None:
        # (index_select has no uint32 kernel on CUDA: gather the words as int32)
        packed = packed.view(torch.int32)[rows].view(torch.uint32)
        scales, offsets = scales[rows], offsets[rows]
        bias = None if bias is None else bias[rows]
    return Affine(packed=packed.contiguous(), scales=scales.contiguous(), offsets=offsets.contiguous(),
                  bias=None if bias is None else bias.contiguous(), bits=a.bits, group=a.group,
                  input=k1 - k0)


def shard_output(a: Affine, rank: int, world: int, segments: int = 1) -> Affine:
    """Column-parallel shard: the output features are `segments` equal blocks
    (q, k, v for a fused QKV); rank r keeps the r-th of `world` slices of
    every block, concatenated in block order."""
    n = a.output
    if n % segments or (n // segments) % world:
        raise ValueError(f"{n} outputs in {segments} segments do not split over {world} ranks")
    seg = n // segments
    part = seg // world
    rows = torch.cat([torch.arange(s * seg + rank * part, s * seg + (rank + 1) * part)
                      for s in range(segments)]).to(a.packed.device)
    return _slice_affine(a, rows=rows)


def shard_input(a: Affine, rank: int, world: int) -> Affine:
    """Row-parallel shard: rank r keeps inputs [r*K/world, (r+1)*K/world) as
    whole packed words and whole scale groups; the layer bias stays on rank 0
    so the sum over ranks adds it once."""
    if a.input % world:
        raise ValueError(f"{a.input} inputs do not split over {world} ranks")
    kw = a.input // world
    return _slice_affine(a, k0=rank * kw, k1=(rank + 1) * kw, keep_bias=(rank == 0))


# ----------------------------------------------------------------- weights


def stack_affine(n: int, k: int, bits: int, *, generator: torch.Generator, group: int = 64,
                 bias: bool = True, device="cuda") -> Affine:
    """Random codes with scales and offsets of a quantized N(0, 0.02) weight
    (scale ~ 6 * 0.02 / (2^bits - 1), offset ~ -scale * (2^bits - 1) / 2), so
    activations keep their size through 60 blocks."""
    levels = (1 << bits) - 1
    words = k * bits // 32
    packed = torch.randint(-2**31, 2**31 - 1, (n, words), generator=generator, device=device,
                           dtype=torch.int32).view(torch.uint32)
    s = (torch.rand((n, k // group), generator=generator, device=device) + 0.5) * (0.12 / levels)
    o = -s * (levels / 2.0) + (torch.rand((n, k // group), generator=generator, device=device) - 0.5) * 0.01
    b = (torch.randn((n,), generator=generator, device=device) * 0.01).to(torch.bfloat16) if bias else None
    return Affine(packed=packed, scales=s.to(torch.bfloat16), offsets=o.to(torch.bfloat16), bias=b,
                  bits=bits, group=group, input=k)


@dataclass
class StreamWeights:
    """One stream's linears in one block, already sharded for this rank."""

    mod: Linear   # 3072 -> 18432, replicated
    qkv: Linear   # 3072 -> 3 * heads/world * 128, column-parallel by heads
    out: Linear   # heads/world * 128 -> 3072, row-parallel
    up: Linear    # 3072 -> 12288/world, column-parallel
    down: Linear  # 12288/world -> 3072, row-parallel


def stream_weights_full(cfg: StackConfig, generator: torch.Generator, device) -> dict:
    """Unsharded affine weights of one stream of one block."""
    h, d = cfg.hidden, cfg.heads * cfg.head_dim
    return {
        "mod": stack_affine(cfg.mod_features, h, cfg.bits, generator=generator, group=cfg.group, device=device),
        "qkv": stack_affine(3 * d, h, cfg.bits, generator=generator, group=cfg.group, device=device),
        "out": stack_affine(h, d, cfg.bits, generator=generator, group=cfg.group, device=device),
        "up": stack_affine(cfg.ffn, h, cfg.bits, generator=generator, group=cfg.group, device=device),
        "down": stack_affine(h, cfg.ffn, cfg.bits, generator=generator, group=cfg.group, device=device),
    }


def shard_stream(full: dict, rank: int, world: int) -> StreamWeights:
    return StreamWeights(
        mod=Linear(affine=full["mod"]),
        qkv=Linear(affine=shard_output(full["qkv"], rank, world, segments=3)),
        out=Linear(affine=shard_input(full["out"], rank, world)),
        up=Linear(affine=shard_output(full["up"], rank, world)),
        down=Linear(affine=shard_input(full["down"], rank, world)),
    )


def stream_weights_shard(cfg: StackConfig, rank: int, world: int, generator: torch.Generator,
                         device) -> StreamWeights:
    """This rank's shard generated directly (the benchmark's 20B-parameter
    stack never exists unsharded): same shapes and statistics as sharding
    `stream_weights_full`, different random draws."""
    h, dl, fl = cfg.hidden, cfg.heads * cfg.head_dim // world, cfg.ffn // world
    g, b = cfg.group, cfg.bits
    down = stack_affine(h, fl, b, generator=generator, group=g, bias=(rank == 0), device=device)
    out = stack_affine(h, dl, b, generator=generator, group=g, bias=(rank == 0), device=device)
    return StreamWeights(
        mod=Linear(affine=stack_affine(cfg.mod_features, h, b, generator=generator, group=g, device=device)),
        qkv=Linear(affine=stack_affine(3 * dl, h, b, generator=generator, group=g, device=device)),
        out=Linear(affine=out),
        up=Linear(affine=stack_affine(fl, h, b, generator=generator, group=g, device=device)),
        down=Linear(affine=down),
    )


# ----------------------------------------------------------------- forward

RunLinear = Callable[..., torch.Tensor]


def cuda_linear(lin: Linear, x: torch.Tensor, *, gate=None, residual=None, activation=None, out=None):
    return lin.forward_fused(x, gate=gate, residual=residual, activation=activation, out=out)


@dataclass
class Timers:
    """CUDA-event spans per category on the current stream (None: untimed)."""

    spans: dict = field(default_factory=dict)
    enabled: bool = False

    def span(self, name: str):
        return _Span(self, name)

    def totals_ms(self) -> dict:
        return {k: sum(a.elapsed_time(b) for a, b in v) for k, v in self.spans.items()}


class _Span:
    def __init__(self, timers: Timers, name: str):
        self.t, self.name = timers, name

    def __enter__(self):
        if self.t.enabled:
            self.a = torch.cuda.Event(enable_timing=True)
            self.a.record()
        return self

    def __exit__(self, *exc):
        if self.t.enabled:
            b = torch.cuda.Event(enable_timing=True)
            b.record()
            self.t.spans.setdefault(self.name, []).append((self.a, b))


class TensorParallel:
    """Rank, world and the all-reduce of a tensor-parallel group.

    overlap_chunks > 1 (opt-in; measured slower than one all-reduce per layer
    on 8 B200 at the benchmark shapes, where four smaller collectives and
    smaller GEMMs on fewer SMs cost more than the overlap hides): the
    row-parallel linears run in that many token chunks
    and each chunk's all-reduce is issued asynchronously as soon as the chunk's
    GEMMs are enqueued, so it runs on NVLink while the next chunk computes;
    the GEMMs then use `comm_sms` fewer SMs (qmm_set_sm_budget) so that the
    collective's kernels have SMs to run on."""

    def __init__(self, rank: int = 0, world: int = 1, group=None, overlap_chunks: int = 1, comm_sms: int = 16):
        self.rank, self.world, self.group = rank, world, group
        self.overlap_chunks = overlap_chunks if world > 1 else 1
        self.comm_sms = comm_sms

    @classmethod
    def from_env(cls):
        import torch.distributed as dist
        if dist.is_available() and dist.is_initialized():
            return cls(dist.get_rank(), dist.get_world_size())
        return cls()

    def all_reduce(self, t: torch.Tensor) -> None:
        if self.world > 1:
            import torch.distributed as dist
            dist.all_reduce(t, group=self.group)

    def all_reduce_async(self, t: torch.Tensor):
        """Enqueues the all-reduce after the current stream's work; the
        returned handle's wait() makes the current stream wait for it."""
        import torch.distributed as dist
        return dist.all_reduce(t, group=self.group, async_op=True)


class DitStack:
    """The 60-block dual-stream linear stack on one rank of a TP group."""

    def __init__(self, cfg: StackConfig, blocks: List[List[StreamWeights]], tp: TensorParallel,
                 run_linear: RunLinear = cuda_linear, attention: Optional[Callable] = None):
        cfg.check_world(tp.world)
        self.cfg, self.blocks, self.tp = cfg, blocks, tp
        self.run_linear = run_linear
        self.attention = attention or _sdpa
        self._bufs = None

    @classmethod
    def random(cls, cfg: StackConfig, tp: TensorParallel, seed: int = 0, device="cuda", blocks=None):
        g = torch.Generator(device=device)
        g.manual_seed(seed * 7919 + tp.rank)
        nb = cfg.blocks if blocks is None else blocks
        weights = [[stream_weights_shard(cfg, tp.rank, tp.world, g, device) for _ in range(2)]
                   for _ in range(nb)]
        return cls(cfg, weights, tp)

    @classmethod
    def from_full(cls, cfg: StackConfig, full_blocks: List[List[dict]], tp: TensorParallel, **kw):
        """Shards unsharded per-block, per-stream weights for this rank."""
        return cls(cfg, [[shard_stream(f, tp.rank, tp.world) for f in blk] for blk in full_blocks], tp, **kw)

    def _buffers(self, x: torch.Tensor):
        cfg, w = self.cfg, self.tp.world
        key = (x.shape[0], x.device, x.dtype)
        if self._bufs is None or self._bufs[0] != key:
            m = x.shape[0]
            dl = cfg.heads * cfg.head_dim // w
            self._bufs = (key, torch.empty((m, 3 * dl), dtype=x.dtype, device=x.device),
                          torch.empty((m, dl), dtype=x.dtype, device=x.device),
                          torch.empty((m, cfg.ffn // w), dtype=x.dtype, device=x.device),
                          torch.empty((2, cfg.mod_features), dtype=x.dtype, device=x.device),
                          torch.empty((m, cfg.hidden), dtype=x.dtype, device=x.device))
        return self._bufs[1:]

    def forward(self, x: torch.Tensor, temb: torch.Tensor, timers: Optional[Timers] = None) -> torch.Tensor:
        """x: bf16 [img_tokens + txt_tokens, hidden] (image rows first), updated
        in place and returned; temb: bf16 [hidden] timestep embedding."""
        cfg, tp = self.cfg, self.tp
        timers = timers or Timers()
        mi = cfg.img_tokens
        if x.shape != (cfg.tokens, cfg.hidden):
            raise ValueError(f"hidden state {tuple(x.shape)} is not [{cfg.tokens}, {cfg.hidden}]")
        qkv, attn, hid, mod, nbuf = self._buffers(x)
        rows = (slice(0, mi), slice(mi, cfg.tokens))
        dl = cfg.heads * cfg.head_dim // tp.world
        t_act = F.silu(temb.float()).to(x.dtype).reshape(1, cfg.hidden)
        last = tp.rank == 0
        # Row-parallel linears and their all-reduce overlap on several ranks:
        # one timing category for both.
        rowpar = "linear" if tp.world == 1 else "rowpar_linear+all_reduce"
        for blk in self.blocks:
            with timers.span("linear"):
                for s in range(2):
                    self.run_linear(blk[s].mod, t_act, out=mod[s:s + 1])
            chunks = [mod[s].view(6, cfg.hidden) for s in range(2)]
            with timers.span("other"):
                n = [_modulate(x[rows[s]], chunks[s][0], chunks[s][1], nbuf[rows[s]]) for s in range(2)]
            with timers.span("linear"):
                for s in range(2):
                    self.run_linear(blk[s].qkv, n[s], out=qkv[rows[s]])
            with timers.span("attention"):
                self.attention(qkv, attn, dl // cfg.head_dim, cfg.head_dim)
            with timers.span(rowpar):
                self._row_parallel([blk[0].out, blk[1].out], attn, [chunks[0][2], chunks[1][2]], x, last)
            with timers.span("other"):
                n = [_modulate(x[rows[s]], chunks[s][3], chunks[s][4], nbuf[rows[s]]) for s in range(2)]
            with timers.span("linear"):
                for s in range(2):
                    self.run_linear(blk[s].up, n[s], activation="gelu_tanh", out=hid[rows[s]])
            with timers.span(rowpar):
                self._row_parallel([blk[0].down, blk[1].down], hid, [chunks[0][5], chunks[1][5]], x, last)
        return x

    def _row_parallel(self, lins, inp, gates, x, last):
        """x[rows of stream s] = gate_s * lin_s(inp[rows]) (+ x, rank 0), then
        the sum over ranks; in token chunks with the all-reduce of each chunk
        overlapping the next chunk's GEMMs when the group has several ranks."""
        cfg, tp = self.cfg, self.tp
        bounds = (0, cfg.img_tokens, cfg.tokens)
        chunks = tp.overlap_chunks
        if chunks <= 1:
            for s in range(2):
                r = slice(bounds[s], bounds[s + 1])
                self.run_linear(lins[s], inp[r], gate=gates[s], residual=x[r] if last else None, out=x[r])
            tp.all_reduce(x)
            return
        # Chunk edges on 192-token tiles of the joint token range.
        step = -(-cfg.tokens // chunks)
        step = -(-step // 192) * 192
        edges = list(range(0, cfg.tokens, step)) + [cfg.tokens]
        on_gpu = x.device.type == "cuda"
        lib = _lib.load() if on_gpu else None
        prev = lib.qmm_set_sm_budget(max(1, _sm_count(x.device) - tp.comm_sms)) if on_gpu else 0
        try:
            works = []
            for a, b in zip(edges[:-1], edges[1:]):
                for s in range(2):
                    lo, hi = max(a, bounds[s]), min(b, bounds[s + 1])
                    if lo < hi:
                        r = slice(lo, hi)
                        self.run_linear(lins[s], inp[r], gate=gates[s], residual=x[r] if last else None, out=x[r])
                works.append(tp.all_reduce_async(x[a:b]))
            for wk in works:
                wk.wait()
        finally:
            if on_gpu:
                lib.qmm_set_sm_budget(prev)


_SM_COUNTS = {}


def _sm_count(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _SM_COUNTS:
        _SM_COUNTS[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return _SM_COUNTS[idx]


def _modulate(x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """LayerNorm (eps 1e-6, no affine) * (1 + scale) + shift into `out`: one
    fused CUDA kernel (qmm_layernorm_modulate) on the GPU; torch ops for the
    CPU tensors of the host-logic tests."""
    if x.device.type == "cuda":
        rows, hidden = x.shape
        _lib.check(_lib.load().qmm_layernorm_modulate(x.data_ptr(), rows, hidden, shift.data_ptr(), scale.data_ptr(),
                                                      1e-6, out.data_ptr(), _stream_handle(x.device)))
        return out
    n = F.layer_norm(x.float(), (x.shape[-1],), eps=1e-6)
    out.copy_(torch.addcmul(shift.float(), n, scale.float() + 1))
    return out


def _sdpa(qkv: torch.Tensor, out: torch.Tensor, heads: int, head_dim: int) -> None:
    """Joint attention of this rank's heads; qkv [m, 3 * heads * head_dim]
    holds q, k, v of every head contiguously; out [m, heads * head_dim]."""
    m = qkv.shape[0]
    q, k, v = (qkv.view(m, 3, heads, head_dim)[:, i].transpose(0, 1).unsqueeze(0) for i in range(3))
    a = F.scaled_dot_product_attention(q, k, v, scale=1.0 / math.sqrt(head_dim))
    out.view(m, heads, head_dim).copy_(a.squeeze(0).transpose(0, 1))
