"""Tensor-parallel dual-stream MMDiT linear stack over the quantized linear.

The caller of the quantized linear in image-forger is the DiT block
(src/dit.rs:36-94): q/k/v projections of the modulated, normalised hidden
state (src/dit.rs:51-62), attention, the output projection with a gated
residual (src/dit.rs:88-91) and a gated feed-forward residual
(src/dit.rs:92-93, src/ops.rs:196-207); the modulation linear runs once per
denoising step on the timestep embedding, before the block loop
(src/dit.rs:277-279, m = 1).  This module runs that linear skeleton in the
dual-stream, hidden-3072 form of the 60-block benchmark stack (image and text
streams with their own weights, joint attention over both):

  mod   = Linear(3072 -> 18432)(silu(temb))          per block and stream, m = 1
  shift1, scale1, gate1, shift2, scale2, gate2 = mod.chunk(6)
  n     = layer_norm(x) * (1 + scale1) + shift1
  q,k,v = Linear(3072 -> 9216)(n)                     24 heads x 128
  a     = attention(q, k, v) over the image and text tokens together
  x     = x + gate1 * Linear(3072 -> 3072)(a)
  n     = layer_norm(x) * (1 + scale2) + shift2
  x     = x + gate2 * Linear(12288 -> 3072)(gelu_tanh(Linear(3072 -> 12288)(n)))

Every modulation depends only on the timestep, so all 2 x 60 modulation
linears run first, column-parallel (each rank computes 1/world of every
modulation's features) and one all-gather assembles them.

Tensor parallelism over `world` ranks (one process per GPU), sequence-parallel
form (the default on several ranks):
  * q/k/v and FFN-up are column-parallel: each rank holds 24/world heads
    (its q, k and v columns, contiguous) and 12288/world FFN features, and
    reads the whole normalised input;
  * out and FFN-down are row-parallel: each rank holds a K slice, whole
    scale groups, and writes its gated partial product g * P_r of every
    token (the gate is per feature, so g * sum_r P_r = sum_r g * P_r);
  * a reduce-scatter (NCCL, bf16 sum) leaves each rank the summed partials of
    its 1/world of the tokens; the hidden state itself is held that way,
    sharded by tokens.  One fused kernel per rank adds the reduced partials
    and g * bias to its rows and applies the next LayerNorm + modulation
    (qmm_residual_layernorm_modulate), and an all-gather rebuilds the whole
    normalised input of the next column-parallel linear.  The bytes on the
    wire equal one all-reduce per row-parallel layer; the residual and norm
    work is divided by world and no rank does more than another.
The replicated form (sequence_parallel=False) keeps the whole hidden state on
every rank and all-reduces it after each row-parallel layer, rank 0 folding
the residual and bias into its GEMM epilogue; one rank always runs that form,
with the residual fused into the GEMM epilogue.
"""
from __future__ import annotations

import ctypes
import math
import os
from dataclasses import dataclass, field
from typing import Callable, List, Optional

import torch
import torch.nn.functional as F

from . import _lib
from .quant import OWN_BIAS, Affine, Linear, _stream_handle

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


def shard_input(a: Affine, rank: int, world: int, keep_bias: Optional[bool] = None) -> Affine:
    """Row-parallel shard: rank r keeps inputs [r*K/world, (r+1)*K/world) as
    whole packed words and whole scale groups.  By default the layer bias
    stays on rank 0 so the sum over ranks adds it once; keep_bias=False drops
    it on every rank (the caller adds it after the reduction)."""
    if a.input % world:
        raise ValueError(f"{a.input} inputs do not split over {world} ranks")
    kw = a.input // world
    keep = (rank == 0) if keep_bias is None else keep_bias
    return _slice_affine(a, k0=rank * kw, k1=(rank + 1) * kw, keep_bias=keep)


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

    mod: Linear   # 3072 -> 18432 / world, column-parallel (rows [r F/w, (r+1) F/w) of the modulation)
    qkv: Linear   # 3072 -> 3 * heads/world * 128, column-parallel by heads
    out: Linear   # heads/world * 128 -> 3072, row-parallel (no bias of its own)
    up: Linear    # 3072 -> 12288/world, column-parallel
    down: Linear  # 12288/world -> 3072, row-parallel (no bias of its own)
    out_bias: Optional[torch.Tensor] = None   # bf16 [3072], the same on every rank
    down_bias: Optional[torch.Tensor] = None  # bf16 [3072], the same on every rank


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
        mod=Linear(affine=shard_output(full["mod"], rank, world)),
        qkv=Linear(affine=shard_output(full["qkv"], rank, world, segments=3)),
        out=Linear(affine=shard_input(full["out"], rank, world, keep_bias=False)),
        up=Linear(affine=shard_output(full["up"], rank, world)),
        down=Linear(affine=shard_input(full["down"], rank, world, keep_bias=False)),
        out_bias=full["out"].bias,
        down_bias=full["down"].bias,
    )


def stream_weights_shard(cfg: StackConfig, rank: int, world: int, generator: torch.Generator, device,
                         shared: torch.Generator) -> StreamWeights:
    """This rank's shard generated directly (the benchmark's 20B-parameter
    stack never exists unsharded): same shapes and statistics as sharding
    `stream_weights_full`, different random draws.  The row-parallel layers'
    biases come from `shared`, a generator seeded alike on every rank, since
    every rank adds them to its own tokens."""
    h, dl, fl = cfg.hidden, cfg.heads * cfg.head_dim // world, cfg.ffn // world
    g, b = cfg.group, cfg.bits
    down = stack_affine(h, fl, b, generator=generator, group=g, bias=False, device=device)
    out = stack_affine(h, dl, b, generator=generator, group=g, bias=False, device=device)
    return StreamWeights(
        mod=Linear(affine=stack_affine(cfg.mod_features // world, h, b, generator=generator, group=g,
                                       device=device)),
        qkv=Linear(affine=stack_affine(3 * dl, h, b, generator=generator, group=g, device=device)),
        out=Linear(affine=out),
        up=Linear(affine=stack_affine(fl, h, b, generator=generator, group=g, device=device)),
        down=Linear(affine=down),
        out_bias=(torch.randn((h,), generator=shared, device=device) * 0.01).to(torch.bfloat16),
        down_bias=(torch.randn((h,), generator=shared, device=device) * 0.01).to(torch.bfloat16),
    )


# ----------------------------------------------------------------- forward

RunLinear = Callable[..., torch.Tensor]


def cuda_linear(lin: Linear, x: torch.Tensor, *, gate=None, residual=None, activation=None, out=None,
                bias=OWN_BIAS):
    return lin.forward_fused(x, gate=gate, residual=residual, activation=activation, out=out, bias=bias)


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
    """Rank, world and the collectives of a tensor-parallel group.

    sequence_parallel (default): row-parallel outputs are reduce-scattered and
    the hidden state is held sharded by tokens (see the module docstring);
    otherwise they are all-reduced and every rank holds the whole hidden
    state.

    overlap_chunks > 1 (replicated form only; opt-in, measured slower than one
    all-reduce per layer on 2 B200 at the benchmark shapes, where four smaller
    collectives and smaller GEMMs on fewer SMs cost more than the overlap
    hides): the row-parallel linears run in that many token chunks and each
    chunk's all-reduce is issued asynchronously as soon as the chunk's GEMMs
    are enqueued, so it runs on NVLink while the next chunk computes; the
    GEMMs then use `comm_sms` fewer SMs (qmm_set_sm_budget) so that the
    collective's kernels have SMs to run on."""

    def __init__(self, rank: int = 0, world: int = 1, group=None, overlap_chunks: int = 1, comm_sms: int = 16,
                 sequence_parallel: bool = True, sp_chunks: int = 1, peer: bool = False):
        self.rank, self.world, self.group = rank, world, group
        self.overlap_chunks = overlap_chunks if world > 1 else 1
        self.comm_sms = comm_sms
        self.sequence_parallel = sequence_parallel and world > 1
        self.sp_chunks = sp_chunks if self.sequence_parallel else 1
        # Sequence-parallel collectives over peer memory (qmm_tp_*), fused
        # with the residual update and norm, instead of NCCL.
        self.peer = peer and self.sequence_parallel
        if self.peer and self.sp_chunks != 1:
            raise ValueError("the peer-memory collectives run the stack in one token chunk")

    @classmethod
    def from_env(cls, **kw):
        import torch.distributed as dist
        if dist.is_available() and dist.is_initialized():
            return cls(dist.get_rank(), dist.get_world_size(), **kw)
        return cls(**kw)

    def _native(self, t: torch.Tensor) -> bool:
        """NCCL's tensor collectives for CUDA tensors; gloo (the CPU tests) lacks
        reduce-scatter and gathers into a list."""
        return t.device.type == "cuda"

    def all_reduce(self, t: torch.Tensor) -> None:
        if self.world > 1:
            import torch.distributed as dist
            dist.all_reduce(t, group=self.group)

    def all_reduce_async(self, t: torch.Tensor):
        """Enqueues the all-reduce after the current stream's work; the
        returned handle's wait() makes the current stream wait for it."""
        import torch.distributed as dist
        return dist.all_reduce(t, group=self.group, async_op=True)

    def reduce_scatter(self, out: torch.Tensor, inp: torch.Tensor, async_op: bool = False):
        """out [M / world, ...] = rows [rank M / world, (rank + 1) M / world) of
        the sum over ranks of inp [M, ...].  async_op: enqueued after the
        current stream's work; the returned handle's wait() makes the current
        stream wait for it (None when it already ran)."""
        if self.world == 1:
            out.copy_(inp)
            return None
        import torch.distributed as dist
        if self._native(inp):
            return dist.reduce_scatter_tensor(out, inp, group=self.group, async_op=async_op)
        t = inp.clone()
        dist.all_reduce(t, group=self.group)
        out.copy_(t.chunk(self.world)[self.rank])
        return None

    def all_gather(self, out: torch.Tensor, inp: torch.Tensor, async_op: bool = False):
        """out [world * L, ...] = the ranks' inp [L, ...] in rank order
        (async_op as for reduce_scatter)."""
        if self.world == 1:
            out.copy_(inp)
            return None
        import torch.distributed as dist
        if self._native(inp):
            return dist.all_gather_into_tensor(out, inp, group=self.group, async_op=async_op)
        dist.all_gather(list(out.chunk(self.world)), inp.contiguous(), group=self.group)
        return None


class PeerBuffers:
    """The symmetric buffers of the peer-memory collectives (include/qmm.h,
    qmm_tp_*): every rank's `part` (gated row-parallel partials), `gathered`
    (normalised input of the column-parallel linears) and counters, mapped
    into every rank's address space by torch's symmetric memory (allocation
    and address exchange only; the data moves in this library's kernels)."""

    def __init__(self, tokens: int, hidden: int, tp: "TensorParallel", device):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm

        # The kernels use plain peer loads and stores: ask torch not to bind
        # the buffers to an NVLink multicast object.
        os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
        group = tp.group or dist.group.WORLD
        name = group.group_name
        symm.enable_symm_mem_for_group(name)
        self.part = symm.empty((tokens, hidden), dtype=torch.bfloat16, device=device)
        self.gathered = symm.empty((tokens, hidden), dtype=torch.bfloat16, device=device)
        self.counters = symm.empty((4,), dtype=torch.int64, device=device)
        self.counters.zero_()
        handles = [symm.rendezvous(t, name) for t in (self.part, self.gathered, self.counters)]
        torch.cuda.synchronize(device)
        dist.barrier(group)  # every rank's counters are zero before anyone signals
        self.peers = _lib.QmmTpPeers()
        self.peers.world, self.peers.rank = tp.world, tp.rank
        for j in range(tp.world):
            self.peers.part[j] = handles[0].buffer_ptrs[j]
            self.peers.gathered[j] = handles[1].buffer_ptrs[j]
            self.peers.counters[j] = handles[2].buffer_ptrs[j]
        self._handles = handles
        self.epoch = 0  # qmm_tp_reduce_norm_gather calls so far (the same on every rank)

    def exchange(self, x_local: torch.Tensor, split: int, vectors, reduce: bool, normalize: bool) -> None:
        """One layer: this rank's partial is complete; reduce, update x_local,
        normalise and gather; wait until every rank is done.  `vectors` holds
        (bias, gate, shift, scale) per stream (entries may be None)."""
        lib = _lib.load()
        st = _stream_handle(x_local.device)
        self.epoch += 1
        norm = _lib.QmmTpNorm()
        for s in range(2):
            bias, gate, shift, scale = vectors[s]
            if bias is None:
                gate = None
            norm.bias[s] = None if bias is None else bias.data_ptr()
            norm.gate[s] = None if gate is None else gate.data_ptr()
            norm.shift[s] = None if shift is None else shift.data_ptr()
            norm.scale[s] = None if scale is None else scale.data_ptr()
        norm.split = split
        norm.eps = 1e-6
        rows, hidden = x_local.shape
        _lib.check(lib.qmm_tp_signal_ready(ctypes.byref(self.peers), st))
        _lib.check(lib.qmm_tp_reduce_norm_gather(ctypes.byref(self.peers), self.epoch, rows, hidden,
                                                  x_local.data_ptr(), ctypes.byref(norm), int(reduce),
                                                  int(normalize), st))
        _lib.check(lib.qmm_tp_wait_gathered(ctypes.byref(self.peers), self.epoch, st))


class DitStack:
    """The 60-block dual-stream linear stack on one rank of a TP group."""

    def __init__(self, cfg: StackConfig, blocks: List[List[StreamWeights]], tp: TensorParallel,
                 run_linear: RunLinear = cuda_linear, attention: Optional[Callable] = None):
        cfg.check_world(tp.world)
        if tp.sequence_parallel and cfg.tokens % (tp.world * tp.sp_chunks):
            raise ValueError(f"{cfg.tokens} tokens do not split into {tp.sp_chunks} chunks over {tp.world} ranks")
        self.cfg, self.blocks, self.tp = cfg, blocks, tp
        self.run_linear = run_linear
        self.attention = attention or _sdpa
        self._bufs = None
        self._peer = None

    @classmethod
    def random(cls, cfg: StackConfig, tp: TensorParallel, seed: int = 0, device="cuda", blocks=None):
        g = torch.Generator(device=device)
        g.manual_seed(seed * 7919 + tp.rank)
        shared = torch.Generator(device=device)
        shared.manual_seed(seed * 7919 + 104729)
        nb = cfg.blocks if blocks is None else blocks
        weights = [[stream_weights_shard(cfg, tp.rank, tp.world, g, device, shared) for _ in range(2)]
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
            m, h = x.shape[0], cfg.hidden
            dl = cfg.heads * cfg.head_dim // w
            nb = len(self.blocks)
            local = m // w if self.tp.sequence_parallel else m
            e = lambda *shape: torch.empty(shape, dtype=x.dtype, device=x.device)  # noqa: E731
            self._bufs = (key, dict(
                qkv=e(m, 3 * dl), attn=e(m, dl), hid=e(m, cfg.ffn // w),
                mod_local=e(2 * nb, cfg.mod_features // w), mod_all=e(w * 2 * nb, cfg.mod_features // w),
                mods=e(2 * nb, cfg.mod_features),
                nfull=e(m, h),            # normalised input of the column-parallel linears
                part=e(m, h),             # gated row-parallel partials (sequence-parallel form)
                xl=e(local, h), nl=e(local, h), red=e(local, h)))
        return self._bufs[1]

    def modulations(self, temb: torch.Tensor, timers: Optional["Timers"] = None) -> torch.Tensor:
        """All modulations of the step, bf16 [blocks, 2 streams, 6, hidden]:
        each rank runs its column shard of the 2 x blocks modulation linears
        (silu(temb) at m = 1, the streaming GEMV) and an all-gather assembles
        the features."""
        cfg, tp = self.cfg, self.tp
        timers = timers or Timers()
        if self._bufs is None:
            raise RuntimeError("modulations() runs inside forward(), which sizes the buffers")
        bufs = self._bufs[1]
        nb = len(self.blocks)
        t_act = F.silu(temb.float()).to(torch.bfloat16).reshape(1, cfg.hidden)
        loc = bufs["mod_local"]
        with timers.span("linear"):
            for b, blk in enumerate(self.blocks):
                for s in range(2):
                    self.run_linear(blk[s].mod, t_act, out=loc[2 * b + s:2 * b + s + 1])
        if tp.world == 1:
            return loc.view(nb, 2, 6, cfg.hidden)
        with timers.span("comm"):
            tp.all_gather(bufs["mod_all"], loc)
        mods = bufs["mods"]
        fl = cfg.mod_features // tp.world
        mods.view(2 * nb, tp.world, fl).copy_(bufs["mod_all"].view(tp.world, 2 * nb, fl).transpose(0, 1))
        return mods.view(nb, 2, 6, cfg.hidden)

    def forward(self, x: torch.Tensor, temb: torch.Tensor, timers: Optional["Timers"] = None) -> torch.Tensor:
        """x: bf16 [img_tokens + txt_tokens, hidden] (image rows first), updated
        in place and returned; temb: bf16 [hidden] timestep embedding.  Every
        rank passes the same x and temb and gets the whole new hidden state."""
        cfg = self.cfg
        timers = timers or Timers()
        if x.shape != (cfg.tokens, cfg.hidden):
            raise ValueError(f"hidden state {tuple(x.shape)} is not [{cfg.tokens}, {cfg.hidden}]")
        self._buffers(x)
        # The stack's weights are only read once loaded: the streaming GEMVs
        # may fetch them before the kernel ahead of them completes.
        lib = _lib.load() if x.device.type == "cuda" else None
        prev = lib.qmm_set_weights_immutable(1) if lib else 0
        try:
            mods = self.modulations(temb, timers)
            if self.tp.peer and x.device.type == "cuda":
                return self._forward_peer(x, mods, timers)
            if self.tp.sequence_parallel:
                return self._forward_sequence_parallel(x, mods, timers)
            return self._forward_replicated(x, mods, timers)
        finally:
            if lib:
                lib.qmm_set_weights_immutable(prev)

    def _stream_rows(self, lo: int, hi: int):
        """(slice of [lo, hi) relative to lo, stream) for the stream segments of token rows [lo, hi)."""
        bounds = (0, self.cfg.img_tokens, self.cfg.tokens)
        out = []
        for s in range(2):
            a, b = max(lo, bounds[s]), min(hi, bounds[s + 1])
            if a < b:
                out.append((slice(a - lo, b - lo), s))
        return out

    def _forward_sequence_parallel(self, x, mods, timers):
        """Sequence-parallel form in tp.sp_chunks token chunks.  Chunk c holds
        tokens [c M/C, (c+1) M/C) and this rank owns the rank-th 1/world of
        each chunk.  With one chunk every collective runs in turn with the
        computation; with several, each chunk's reduce-scatter and all-gather
        run on the collective stream while the next chunk's linears run (the
        steps between two attentions are per token, so the chunks only meet
        at attention), and the GEMMs leave tp.comm_sms SMs to the
        collectives."""
        cfg, tp = self.cfg, self.tp
        bufs = self._bufs[1]
        qkv, attn, hid, part = bufs["qkv"], bufs["attn"], bufs["hid"], bufs["part"]
        nfull, xl, nl, red = bufs["nfull"], bufs["xl"], bufs["nl"], bufs["red"]
        nc = tp.sp_chunks
        span = cfg.tokens // nc             # tokens per chunk
        piece = span // tp.world            # this rank's tokens of a chunk
        chunk = [slice(c * span, (c + 1) * span) for c in range(nc)]
        own = [slice(c * piece, (c + 1) * piece) for c in range(nc)]  # the chunk's piece in xl / nl / red
        first = [c * span + tp.rank * piece for c in range(nc)]        # its first token
        # (rows of xl, stream) of each piece, and (token rows, stream) of each chunk
        segs = [[(slice(c * piece + r.start, c * piece + r.stop), s)
                 for r, s in self._stream_rows(first[c], first[c] + piece)] for c in range(nc)]
        rows = [[(slice(c * span + r.start, c * span + r.stop), s)
                 for r, s in self._stream_rows(c * span, (c + 1) * span)] for c in range(nc)]
        dl = cfg.heads * cfg.head_dim // tp.world
        overlap = nc > 1
        for c in range(nc):
            xl[own[c]].copy_(x[first[c]:first[c] + piece])

        def waitall(works):
            with timers.span("comm"):
                for w in works:
                    if w is not None:
                        w.wait()

        with timers.span("other"):
            for c in range(nc):
                for r, s in segs[c]:
                    _modulate(xl[r], mods[0, s, 0], mods[0, s, 1], nl[r])
        with timers.span("comm"):
            for c in range(nc):
                tp.all_gather(nfull[chunk[c]], nl[own[c]])
        ag = [None] * nc
        budget = None
        if overlap and x.device.type == "cuda":
            budget = _lib.load().qmm_set_sm_budget(max(1, _sm_count(x.device) - tp.comm_sms))
        try:
            nb = len(self.blocks)
            for b, blk in enumerate(self.blocks):
                m = mods[b]
                for c in range(nc):
                    waitall([ag[c]])
                    with timers.span("linear"):
                        for r, s in rows[c]:
                            self.run_linear(blk[s].qkv, nfull[r], out=qkv[r])
                with timers.span("attention"):
                    self.attention(qkv, attn, dl // cfg.head_dim, cfg.head_dim)
                rs = []
                for c in range(nc):
                    with timers.span("linear"):
                        for r, s in rows[c]:
                            self.run_linear(blk[s].out, attn[r], gate=m[s, 2], bias=None, out=part[r])
                    with timers.span("comm"):
                        rs.append(tp.reduce_scatter(red[own[c]], part[chunk[c]], async_op=overlap))
                ag = []
                for c in range(nc):
                    waitall([rs[c]])
                    with timers.span("other"):
                        for r, s in segs[c]:
                            _residual_modulate(xl[r], red[r], blk[s].out_bias, m[s, 2], m[s, 3], m[s, 4], nl[r])
                    with timers.span("comm"):
                        ag.append(tp.all_gather(nfull[chunk[c]], nl[own[c]], async_op=overlap))
                rs = []
                for c in range(nc):
                    waitall([ag[c]])
                    with timers.span("linear"):
                        for r, s in rows[c]:
                            self.run_linear(blk[s].up, nfull[r], activation="gelu_tanh", out=hid[r])
                        for r, s in rows[c]:
                            self.run_linear(blk[s].down, hid[r], gate=m[s, 5], bias=None, out=part[r])
                    with timers.span("comm"):
                        rs.append(tp.reduce_scatter(red[own[c]], part[chunk[c]], async_op=overlap))
                last = b + 1 == nb
                ag = [None] * nc
                for c in range(nc):
                    waitall([rs[c]])
                    with timers.span("other"):
                        for r, s in segs[c]:
                            if last:
                                _residual_modulate(xl[r], red[r], blk[s].down_bias, m[s, 5], None, None, None)
                            else:
                                _residual_modulate(xl[r], red[r], blk[s].down_bias, m[s, 5], mods[b + 1, s, 0],
                                                   mods[b + 1, s, 1], nl[r])
                    if not last:
                        with timers.span("comm"):
                            ag[c] = tp.all_gather(nfull[chunk[c]], nl[own[c]], async_op=overlap)
        finally:
            if budget is not None:
                _lib.load().qmm_set_sm_budget(budget)
        with timers.span("comm"):
            for c in range(nc):
                tp.all_gather(x[chunk[c]], xl[own[c]])
        return x

    def _forward_peer(self, x, mods, timers):
        """Sequence-parallel form with the collectives over peer memory: per
        row-parallel layer one qmm_tp_* exchange sums the ranks' partials of
        this rank's tokens in f32, updates the residual, normalises for the
        next linear and stores the result into every rank's gathered input."""
        cfg, tp = self.cfg, self.tp
        bufs = self._bufs[1]
        if self._peer is None:
            self._peer = PeerBuffers(cfg.tokens, cfg.hidden, tp, x.device)
        pb = self._peer
        part, nfull = pb.part, pb.gathered
        qkv, attn, hid, xl = bufs["qkv"], bufs["attn"], bufs["hid"], bufs["xl"]
        local = cfg.tokens // tp.world
        lo = tp.rank * local
        split = min(max(cfg.img_tokens - lo, 0), local)
        rows = (slice(0, cfg.img_tokens), slice(cfg.img_tokens, cfg.tokens))
        dl = cfg.heads * cfg.head_dim // tp.world
        xl.copy_(x[lo:lo + local])
        with timers.span("comm"):
            pb.exchange(xl, split, [(None, None, mods[0, s, 0], mods[0, s, 1]) for s in range(2)],
                        reduce=False, normalize=True)
        nb = len(self.blocks)
        for b, blk in enumerate(self.blocks):
            m = mods[b]
            with timers.span("linear"):
                for s in range(2):
                    self.run_linear(blk[s].qkv, nfull[rows[s]], out=qkv[rows[s]])
            with timers.span("attention"):
                self.attention(qkv, attn, dl // cfg.head_dim, cfg.head_dim)
            with timers.span("linear"):
                for s in range(2):
                    self.run_linear(blk[s].out, attn[rows[s]], gate=m[s, 2], bias=None, out=part[rows[s]])
            with timers.span("comm"):
                pb.exchange(xl, split, [(blk[s].out_bias, m[s, 2], m[s, 3], m[s, 4]) for s in range(2)],
                            reduce=True, normalize=True)
            with timers.span("linear"):
                for s in range(2):
                    self.run_linear(blk[s].up, nfull[rows[s]], activation="gelu_tanh", out=hid[rows[s]])
                for s in range(2):
                    self.run_linear(blk[s].down, hid[rows[s]], gate=m[s, 5], bias=None, out=part[rows[s]])
            last = b + 1 == nb
            with timers.span("comm"):
                if last:
                    vec = [(blk[s].down_bias, m[s, 5], None, None) for s in range(2)]
                else:
                    vec = [(blk[s].down_bias, m[s, 5], mods[b + 1, s, 0], mods[b + 1, s, 1]) for s in range(2)]
                pb.exchange(xl, split, vec, reduce=True, normalize=not last)
        with timers.span("comm"):
            tp.all_gather(x, xl)
        return x

    def _forward_replicated(self, x, mods, timers):
        cfg, tp = self.cfg, self.tp
        bufs = self._bufs[1]
        qkv, attn, hid, nbuf = bufs["qkv"], bufs["attn"], bufs["hid"], bufs["nfull"]
        mi = cfg.img_tokens
        rows = (slice(0, mi), slice(mi, cfg.tokens))
        dl = cfg.heads * cfg.head_dim // tp.world
        first = tp.rank == 0
        # On several ranks the row-parallel linears and their all-reduce are
        # one timing category (they overlap when chunked).
        rowpar = "linear" if tp.world == 1 else "rowpar_linear+all_reduce"
        for b, blk in enumerate(self.blocks):
            chunks = mods[b]
            with timers.span("other"):
                n = [_modulate(x[rows[s]], chunks[s][0], chunks[s][1], nbuf[rows[s]]) for s in range(2)]
            with timers.span("linear"):
                for s in range(2):
                    self.run_linear(blk[s].qkv, n[s], out=qkv[rows[s]])
            with timers.span("attention"):
                self.attention(qkv, attn, dl // cfg.head_dim, cfg.head_dim)
            with timers.span(rowpar):
                self._row_parallel([blk[0].out, blk[1].out], [blk[0].out_bias, blk[1].out_bias], attn,
                                   [chunks[0][2], chunks[1][2]], x, first)
            with timers.span("other"):
                n = [_modulate(x[rows[s]], chunks[s][3], chunks[s][4], nbuf[rows[s]]) for s in range(2)]
            with timers.span("linear"):
                for s in range(2):
                    self.run_linear(blk[s].up, n[s], activation="gelu_tanh", out=hid[rows[s]])
            with timers.span(rowpar):
                self._row_parallel([blk[0].down, blk[1].down], [blk[0].down_bias, blk[1].down_bias], hid,
                                   [chunks[0][5], chunks[1][5]], x, first)
        return x

    def _row_parallel(self, lins, biases, inp, gates, x, first):
        """x[rows of stream s] = gate_s * (lin_s(inp[rows]) + bias_s) + x on rank
        0, gate_s * lin_s(inp[rows]) elsewhere, then the sum over ranks; in
        token chunks with the all-reduce of each chunk overlapping the next
        chunk's GEMMs when overlap_chunks > 1."""
        cfg, tp = self.cfg, self.tp
        bounds = (0, cfg.img_tokens, cfg.tokens)
        chunks = tp.overlap_chunks

        def run(s, r):
            self.run_linear(lins[s], inp[r], gate=gates[s], residual=x[r] if first else None, out=x[r],
                            bias=biases[s] if first else None)

        if chunks <= 1:
            for s in range(2):
                run(s, slice(bounds[s], bounds[s + 1]))
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
                        run(s, slice(lo, hi))
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


def _residual_modulate(x: torch.Tensor, delta: torch.Tensor, bias: Optional[torch.Tensor],
                       gate: Optional[torch.Tensor], shift: Optional[torch.Tensor], scale: Optional[torch.Tensor],
                       out: Optional[torch.Tensor]) -> None:
    """x = x + delta + gate * bias (one rounding), then, when `out` is given,
    out = LayerNorm(x) * (1 + scale) + shift: one fused CUDA kernel
    (qmm_residual_layernorm_modulate) on the GPU; torch ops on CPU tensors."""
    if bias is None:
        gate = None
    if x.device.type == "cuda":
        rows, hidden = x.shape
        _lib.check(_lib.load().qmm_residual_layernorm_modulate(
            x.data_ptr(), rows, hidden, delta.data_ptr(), None if bias is None else bias.data_ptr(),
            None if gate is None else gate.data_ptr(), None if out is None else shift.data_ptr(),
            None if out is None else scale.data_ptr(), 1e-6, None if out is None else out.data_ptr(),
            _stream_handle(x.device)))
        return
    t = x.float() + delta.float()
    if bias is not None:
        t = t + (bias.float() * gate.float() if gate is not None else bias.float())
    x.copy_(t.to(x.dtype))
    if out is not None:
        n = F.layer_norm(x.float(), (x.shape[-1],), eps=1e-6)
        out.copy_(torch.addcmul(shift.float(), n, scale.float() + 1))


def _sdpa(qkv: torch.Tensor, out: torch.Tensor, heads: int, head_dim: int) -> None:
    """Joint attention of this rank's heads; qkv [m, 3 * heads * head_dim]
    holds q, k, v of every head contiguously; out [m, heads * head_dim]."""
    m = qkv.shape[0]
    q, k, v = (qkv.view(m, 3, heads, head_dim)[:, i].transpose(0, 1).unsqueeze(0) for i in range(3))
    a = F.scaled_dot_product_attention(q, k, v, scale=1.0 / math.sqrt(head_dim))
    out.view(m, heads, head_dim).copy_(a.squeeze(0).transpose(0, 1))
