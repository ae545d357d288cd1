"""Benchmark of the MLX affine quantized linear on B200 (one JSON line).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload dit_2048_8bit|dit_1024_4bit|ffn_up|linear_4bit|ffn_down|adaln_gemv]

Default workload (`dit_2048_8bit`): one denoising step of the 60-block
dual-stream DiT linear stack at 2048x2048 (16384 image + 512 text tokens,
hidden 3072, 8-bit group-64 weights; qwen_imager_b200/dit_stack.py), in ms,
tensor-parallel over the N ranks (strong scaling: the image is fixed, every
rank holds 1/N of the weights).  On several ranks the stack runs in
sequence-parallel form: after each row-parallel layer an NCCL reduce-scatter
of the gated partials, one fused residual + LayerNorm + modulation kernel on
the rank's tokens, and an NCCL all-gather before the next column-parallel
layer.  The line carries a breakdown (quantized linears, attention,
collectives, the rest), every distinct linear's per-launch time and
roofline, an end-to-end time through host memory, and on N > 1 an untimed
check of a small stack sharded over the N ranks against one rank
(`tp_parity`).  Weights are random codes with N(0, 0.02)-sized scales; the
hidden state is random.

The kernel workloads (ffn_up, linear_4bit, ffn_down, adaln_gemv) time single
quantized linears of the benchmark configurations in TFLOP/s; every linear
rotates over at least three weight/input sets whose bytes together are at
least twice the 126 MB L2, so every launch streams its operands from HBM.
With N > 1 every rank runs its own batch (weak scaling, no collective).

--impl reference times the reference's CPU path for the same workload on the
host cores (the oracle's restatement of src/quant.rs:105-113: per-call f32
dequantization of the whole weight plus an f32 GEMM over all tokens), rank 0
only; for the stack, one block timed piece by piece, x60.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    # name: (description, [(m, k, n, bits, extras)], seed)
    "ffn_up": ("FFN up 8-bit [4352x3072]x[12288x3072]^T + adaLN GEMV 4-bit [1x3072]x[18432x3072]^T",
               [(4352, 3072, 12288, 8, {}), (1, 3072, 18432, 4, {"silu_input": True})], 1),
    "linear_4bit": ("4-bit linear [4096x3072]x[3072x3072]^T + bias",
                    [(4096, 3072, 3072, 4, {"bias": True})], 0),
    "ffn_down": ("FFN down 4-bit [4352x12288]x[3072x12288]^T + fused residual, GELU-tanh input",
                 [(4352, 12288, 3072, 4, {"residual": True, "gelu_input": True})], 2),
    "adaln_gemv": ("adaLN GEMV 4-bit [1x3072]x[18432x3072]^T", [(1, 3072, 18432, 4, {"silu_input": True})], 1),
    "adaln_gemv_8bit": ("adaLN GEMV 8-bit [1x3072]x[18432x3072]^T (the 2048x2048 stack's modulation)",
                        [(1, 3072, 18432, 8, {"silu_input": True})], 5),
    # The 2048x2048 stack's image-stream FFN-up GEMM on one rank (for profiles).
    "stack_img_up": ("image-stream FFN up 8-bit [16384x3072]x[12288x3072]^T + GELU-tanh",
                     [(16384, 3072, 12288, 8, {"activation": "gelu_tanh"})], 6),
    # Its image-stream out-projection as one of 8 row-parallel shards (K = 3072 / 8).
    "stack_out_shard8": ("image-stream out-projection shard of 8 ranks, 8-bit [16384x384]x[3072x384]^T",
                         [(16384, 384, 3072, 8, {})], 7),
}
STACK_WORKLOADS = {
    "dit_1024_4bit": "60-block dual-stream DiT linear stack, 1024x1024 (4096 image + 256 text tokens), 4-bit",
    "dit_2048_8bit": "60-block dual-stream DiT linear stack, 2048x2048 (16384 image + 512 text tokens), 8-bit",
}
ROTATE = 3              # fewest sets a linear rotates over
L2_BYTES = 126 * 2**20  # each linear's rotation covers at least twice this
METRIC = "qmm TFLOP/s (quantized DiT linears, bf16 tensor cores)"
STACK_METRIC = "DiT-stack step ms (60 blocks: quantized linears + joint attention + TP collectives)"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=None, help="default 300 (kernels), 10 (dit stacks)")
    p.add_argument("--warmup", type=int, default=None, help="default 5 (kernels), 3 (dit stacks)")
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=sorted(WORKLOADS) + sorted(STACK_WORKLOADS), default="dit_2048_8bit")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    p.add_argument("--no-configs", action="store_true",
                   help="dit_* on one GPU: skip timing the single-linear configurations beside the stack")
    p.add_argument("--no-parity", action="store_true", help="dit_*: skip the untimed TP-vs-one-rank check (N > 1)")
    p.add_argument("--replicated", action="store_true",
                   help="dit_*: all-reduce the whole hidden state on every rank instead of the sequence-parallel form")
    p.add_argument("--overlap-chunks", type=int, default=1,
                   help="dit_* --replicated: token chunks whose all-reduce overlaps the next chunk's GEMMs (1 = none)")
    p.add_argument("--sp-chunks", type=int, default=1,
                   help="dit_* on N > 1: token chunks whose reduce-scatter / all-gather overlap the other chunks' "
                        "linears (1 = none)")
    p.add_argument("--comm", choices=["peer", "nccl"], default="peer",
                   help="dit_* on N > 1, one token chunk, sequence-parallel: the per-layer reduce + norm + gather "
                        "over peer memory (qmm_tp_*, the default) or as NCCL reduce-scatter / all-gather")
    p.add_argument("--comm-sms", type=int, default=16,
                   help="dit_* with --sp-chunks > 1: SMs the GEMMs leave to the collectives")
    a = p.parse_args()
    stack = a.workload in STACK_WORKLOADS
    if a.steps is None:
        a.steps = 10 if stack else 300
    if a.warmup is None:
        a.warmup = 3 if stack else 5
    # The peer-memory exchange serves the one-chunk sequence-parallel form.
    a.peer = a.comm == "peer" and not a.replicated and a.sp_chunks == 1
    return a


def step_flops(layers):
    return sum(2.0 * m * n * k for (m, k, n, _b, _e) in layers)


def measured_peaks():
    """(bf16 burst TFLOP/s, bf16 sustained TFLOP/s, HBM GB/s, source)."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), d["hbm_gbs"], "measured"
    except Exception:
        return 1590.0, 1400.0, 6650.0, "fallback"


def profile_traffic(workload):
    """dram bytes per launch of the dominant kernel from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", f"traffic_{workload}.txt")
    try:
        with open(path) as f:
            for line in f:
                if line.startswith("dram_bytes_per_launch:"):
                    return float(line.split(":", 1)[1])
    except OSError:
        pass
    return None


class ClockSampler:
    """Samples SM clocks and clock-event reasons through NVML during the timed region."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, index):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self.power_w, self.limit_w = [], None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            try:
                self.limit_w = pynvml.nvmlDeviceGetEnforcedPowerLimit(self.h) / 1000.0
            except Exception:
                self.limit_w = None
        except Exception:
            self.nv = None

    def _run(self):
        nv = self.nv
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                try:
                    self.power_w.append(nv.nvmlDeviceGetPowerUsage(self.h) / 1000.0)
                except Exception:
                    pass
                mask = get_reasons(self.h)
                for bit, name in self.REASONS.items():
                    if mask & bit and bit != 0x1:
                        self.reasons.add(name)
            except Exception:
                pass
            self._stop.wait(0.005)

    def __enter__(self):
        if self.nv:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._thread:
            self._thread.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"]}
        out = {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
               "reasons": sorted(self.reasons), "samples": len(self.samples)}
        if self.power_w:
            # Power draw against the enforced limit shows power capping even
            # when the sampled reason mask misses it.
            out["power_w_max"] = round(max(self.power_w), 1)
            out["power_w_median"] = round(statistics.median(self.power_w), 1)
            out["power_limit_w"] = self.limit_w
        return out


# --------------------------------------------------------------------- our arm
def layer_bytes(m, k, n, bits, ex):
    """Bytes one launch reads and writes: codes, scales and offsets, x, y (and residual)."""
    return n * k * bits // 8 + 2 * n * (k // 64) * 2 + 2 * m * k + 2 * m * n * (2 if ex.get("residual") else 1)


def rotation(layer):
    """Number of input sets a linear rotates over: its sets exceed twice the L2."""
    return max(ROTATE, -(-2 * L2_BYTES // layer_bytes(*layer)))


def build_sets(layers, seed, device):
    """sets[li][r]: the r-th (Linear, x, residual, y) of layer li."""
    import torch

    from qwen_imager_b200.synthetic import gaussian, quantized_linear

    sets = []
    for li, (m, k, n, bits, ex) in enumerate(layers):
        entry = []
        for r in range(rotation(layers[li])):
            s = seed * 1000 + r * 10 + li
            lin = quantized_linear(n, k, bits, seed=s, bias_std=0.01 if ex.get("bias") else None, device=device)
            g = torch.Generator(device=device)
            g.manual_seed(s + 500)
            x = gaussian((m, k), 1.0, g, device)
            if ex.get("silu_input"):
                x = torch.nn.functional.silu(x)
            if ex.get("gelu_input"):
                x = torch.nn.functional.gelu(x, approximate="tanh")
            x = x.to(torch.bfloat16)
            res = gaussian((m, n), 1.0, g, device).to(torch.bfloat16) if ex.get("residual") else None
            y = torch.empty((m, n), dtype=torch.bfloat16, device=device)
            entry.append((lin, x, res, y))
        sets.append(entry)
    return sets


def run_ours(args, rank, world, device):
    import torch

    from qwen_imager_b200 import _lib, device_error

    desc, layers, seed = WORKLOADS[args.workload]
    sets = build_sets(layers, seed + 17 * rank, device)
    dist = world > 1
    if dist:
        import torch.distributed as tdist

    def step(i, only=None):
        for li, rot in enumerate(sets):
            if only is None or only == li:
                lin, x, res, y = rot[i % len(rot)]
                lin.forward_fused(x, residual=res, out=y, activation=layers[li][4].get("activation"))

    # Weights are written once, before the step: the streaming GEMV may fetch
    # them before the kernel ahead of it completes.
    _lib.load().qmm_set_weights_immutable(1)
    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize()
    if device_error(device):
        raise RuntimeError("device-side wait expired during warm-up")

    # The K timed steps are captured once as one CUDA graph (the steady state
    # of a serving loop: no per-call host work, no gaps between launches),
    # and each layer's K launches as another graph for its per-launch time.
    cap = torch.cuda.Stream(device)
    c0 = _lib.launch_count()
    with torch.cuda.stream(cap):
        steps_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(steps_graph, stream=cap):
            for i in range(args.steps):
                step(i)
        launches = _lib.launch_count() - c0
        layer_graphs = []
        for li in range(len(layers)):
            gl = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gl, stream=cap):
                for i in range(args.steps):
                    step(i, only=li)
            layer_graphs.append(gl)
    torch.cuda.synchronize()
    steps_graph.replay()  # untimed: first replay uploads the graph
    torch.cuda.synchronize()

    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(torch.cuda.current_device())
    if dist:
        tdist.barrier()
    torch.cuda.synchronize()
    with sampler:
        t0.record()
        steps_graph.replay()
        t1.record()
        torch.cuda.synchronize()
    elapsed = t0.elapsed_time(t1)
    # Per-layer launch time: the layer's K launches, same rotation, same stream.
    kernel_ms = []
    layer_sampler = ClockSampler(torch.cuda.current_device())
    with layer_sampler:
        for gl in layer_graphs:
            gl.replay()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            gl.replay()
            b.record()
            torch.cuda.synchronize()
            kernel_ms.append(a.elapsed_time(b) / args.steps)
    if dist:
        tdist.barrier()
        t = torch.tensor([elapsed], device=device, dtype=torch.float64)
        tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
        elapsed = float(t.item())
    ms_per_step = elapsed / args.steps
    flops = step_flops(layers)
    value = world * flops / (ms_per_step * 1e-3) / 1e12

    # End to end through the public API with host buffers: per step, copy the
    # step's inputs from pinned host memory, run, read the outputs back.
    e2e = None
    if not args.no_e2e:
        host = []
        for (lin, x, res, y) in (rot[0] for rot in sets):
            hx = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
            hx.copy_(x)
            hr = None
            if res is not None:
                hr = torch.empty(res.shape, dtype=res.dtype, pin_memory=True)
                hr.copy_(res)
            hy = torch.empty(y.shape, dtype=y.dtype, pin_memory=True)
            host.append((hx, hr, hy))
        h2d = sum(hx.numel() * 2 + (hr.numel() * 2 if hr is not None else 0) for hx, hr, _ in host)
        d2h = sum(hy.numel() * 2 for _, _, hy in host)

        def e2e_step(i):
            for li, (rot, (hx, hr, hy)) in enumerate(zip(sets, host)):
                lin, x, res, y = rot[i % len(rot)]
                x.copy_(hx, non_blocking=True)
                if hr is not None:
                    res.copy_(hr, non_blocking=True)
                lin.forward_fused(x, residual=res, out=y, activation=layers[li][4].get("activation"))
                hy.copy_(y, non_blocking=True)

        for i in range(2):
            e2e_step(i)
        torch.cuda.synchronize()
        if dist:
            tdist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        n_e2e = max(3, min(args.steps, 20))
        for i in range(n_e2e):
            e2e_step(i)
        b.record()
        torch.cuda.synchronize()
        e_ms = a.elapsed_time(b) / n_e2e
        if dist:
            t = torch.tensor([e_ms], device=device, dtype=torch.float64)
            tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
            e_ms = float(t.item())
        e2e = {"value": round(world * flops / (e_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
               "ms_per_step": round(e_ms, 4), "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h)}

    if device_error(device):
        raise RuntimeError("device-side wait expired during the timed region")

    # Roofline of the dominant kernel (largest FLOP count).
    dom = max(range(len(layers)), key=lambda li: 2.0 * layers[li][0] * layers[li][1] * layers[li][2])
    m, k, n, bits, _ = layers[dom]
    burst_tf, sustained_tf, hbm_gbs, peak_kind = measured_peaks()
    # Burst or sustained denominator from the layer's own timed region: its
    # length and the clock record taken while it ran.
    peak_tf, tf_source = choose_peak(kernel_ms[dom] * args.steps * 1e-3, layer_sampler.summary())
    if m <= 16:
        alg_bytes = n * k * bits / 8 + n * (k // 64) * 4 + m * k * 2 + m * n * 2
        achieved = alg_bytes / (kernel_ms[dom] * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_gbs, "unit": "GB/s",
                "frac": round(achieved / hbm_gbs, 4)}
    else:
        achieved = 2.0 * m * n * k / (kernel_ms[dom] * 1e-3) / 1e12
        roof = {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak_tf, "unit": "TFLOP/s",
                "frac": round(achieved / peak_tf, 4)}
    if m <= 16:
        roof["peak_source"] = f"{peak_kind} HBM copy (MEASURED_PEAKS.json hbm_gbs)"
    else:
        roof["peak_source"] = tf_source
    roof["layer_clocks"] = layer_sampler.summary()
    roof["traffic"] = profile_traffic(args.workload)
    roof["kernel_ms"] = round(kernel_ms[dom], 5)
    per_layer = []
    for li, (m, k, n, bits, _) in enumerate(layers):
        entry = {"m": m, "k": k, "n": n, "bits": bits, "kernel_us": round(kernel_ms[li] * 1e3, 2)}
        if m <= 16:
            b = n * k * bits / 8 + n * (k // 64) * 4 + m * k * 2 + m * n * 2
            entry["GB/s"] = round(b / (kernel_ms[li] * 1e-3) / 1e9, 1)
            entry["hbm_frac"] = round(entry["GB/s"] / hbm_gbs, 4)
        else:
            entry["TFLOP/s"] = round(2.0 * m * n * k / (kernel_ms[li] * 1e-3) / 1e12, 1)
        per_layer.append(entry)
    del steps_graph, layer_graphs
    return {
        "value": round(value, 3), "ms_per_step": round(ms_per_step, 5), "e2e": e2e, "roofline": roof,
        "gpu_launches": int(launches), "layers": per_layer, "clocks": sampler.summary(),
    }


# --------------------------------------------------------------- DiT stack arm
def _layer_shapes(cfg, world):
    """(name, stream, m, k, n, epilogue) of every distinct linear launch of one
    block on one rank (column shards /world, row shards K/world)."""
    h, f, d = cfg.hidden, cfg.ffn, cfg.heads * cfg.head_dim
    out = []
    for s, m in ((0, cfg.img_tokens), (1, cfg.txt_tokens)):
        tag = ("img", "txt")[s]
        out += [(f"{tag}_qkv", s, m, h, 3 * d // world, "none"),
                (f"{tag}_out", s, m, d // world, h, "gate" if world > 1 else "gate+bias+residual"),
                (f"{tag}_up", s, m, h, f // world, "gelu_tanh"),
                (f"{tag}_down", s, m, f // world, h, "gate" if world > 1 else "gate+bias+residual")]
    out.append(("modulation", 0, 1, h, cfg.mod_features // world, "none"))
    return out


def time_stack_layers(stack, cfg, world, steps, device):
    """Per-launch device time of each distinct linear of the stack on this
    rank: for each, a CUDA graph of `steps` launches that walks over the
    blocks' weights (each launch reads another block's weights from HBM),
    timed with CUDA events on the capture stream."""
    import torch

    from qwen_imager_b200.quant import OWN_BIAS

    bufs = stack._bufs[1]
    h = cfg.hidden
    srcs = {"qkv": bufs["nfull"], "out": bufs["attn"], "up": bufs["nfull"], "down": bufs["hid"]}
    rows = (slice(0, cfg.img_tokens), slice(cfg.img_tokens, cfg.tokens))
    gate = torch.ones((h,), dtype=torch.bfloat16, device=device)
    bias = torch.zeros((h,), dtype=torch.bfloat16, device=device)
    y = torch.empty((cfg.tokens, max(3 * cfg.heads * cfg.head_dim // world, cfg.ffn // world, h)),
                    dtype=torch.bfloat16, device=device)
    res = torch.zeros((cfg.tokens, h), dtype=torch.bfloat16, device=device)
    t_act = torch.zeros((1, h), dtype=torch.bfloat16, device=device)
    mod_out = torch.empty((1, cfg.mod_features // world), dtype=torch.bfloat16, device=device)
    results = []
    cap = torch.cuda.Stream(device)
    for name, s, m, k, n, ep in _layer_shapes(cfg, world):
        kind = name.split("_")[-1]

        def launch(i, name=name, s=s, m=m, n=n, ep=ep, kind=kind):
            blk = stack.blocks[i % len(stack.blocks)][s]
            if name == "modulation":
                blk.mod.forward_fused(t_act, out=mod_out)
                return
            lin = getattr(blk, kind)
            x = srcs[kind][rows[s]]
            out = y.view(-1)[: m * n].view(m, n)
            kw = {}
            if ep == "gelu_tanh":
                kw["activation"] = "gelu_tanh"
            elif ep.startswith("gate"):
                kw["gate"] = gate
                kw["bias"] = bias if "bias" in ep else None
                if "residual" in ep:
                    kw["residual"] = res[rows[s]]
            lin.forward_fused(x, out=out, **kw)

        for i in range(2):
            launch(i)
        torch.cuda.synchronize()
        with torch.cuda.stream(cap):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cap):
                for i in range(steps):
                    launch(i)
        torch.cuda.synchronize()
        g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(cap):
            a.record(cap)
            g.replay()
            b.record(cap)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / steps
        del g
        flops = 2.0 * m * n * k
        entry = {"layer": name, "m": m, "k": k, "n": n, "bits": cfg.bits, "epilogue": ep,
                 "launches_per_step": len(stack.blocks) * (1 if name != "modulation" else 2),
                 "kernel_us": round(ms * 1e3, 2)}
        if m <= 16:
            byts = n * k * cfg.bits / 8 + n * (k // cfg.group) * 4 + m * k * 2 + m * n * 2
            entry["GB/s"] = round(byts / (ms * 1e-3) / 1e9, 1)
            entry["alg_bytes"] = int(byts)
        else:
            entry["TFLOP/s"] = round(flops / (ms * 1e-3) / 1e12, 1)
            entry["alg_flops"] = flops
        results.append(entry)
    return results


# The single-linear configurations also timed inside the stack line at N = 1
# (each on its own 20-launch graph, rotating over weight sets larger than L2).
CONFIG_LINES = (("config1 linear_4bit", "linear_4bit"), ("config2 ffn_up", "ffn_up"),
                ("config3 ffn_down", "ffn_down"), ("adaln_gemv_8bit", "adaln_gemv_8bit"))


def time_configs(device, steps=20):
    """Per-launch device time of the single-linear configurations (GEMMs and
    the modulation GEMV) with their rooflines against the burst peaks: the
    region of each is a few milliseconds."""
    import torch

    burst_tf, _, hbm_gbs, _ = measured_peaks()
    out = []
    cap = torch.cuda.Stream(device)
    for label, name in CONFIG_LINES:
        _, layers, seed = WORKLOADS[name]
        sets = build_sets(layers, seed, device)
        for li, (m, k, n, bits, ex) in enumerate(layers):
            rot = sets[li]

            def launch(i, rot=rot, ex=ex):
                lin, x, res, y = rot[i % len(rot)]
                lin.forward_fused(x, residual=res, out=y, activation=ex.get("activation"))

            for i in range(3):
                launch(i)
            torch.cuda.synchronize()
            with torch.cuda.stream(cap):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=cap):
                    for i in range(steps):
                        launch(i)
            torch.cuda.synchronize()
            g.replay()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            g.replay()
            b.record()
            torch.cuda.synchronize()
            us = a.elapsed_time(b) / steps * 1e3
            e = {"config": label, "m": m, "k": k, "n": n, "bits": bits, "kernel_us": round(us, 2)}
            if m <= 16:
                gbs = (n * k * bits / 8 + n * (k // 64) * 4 + m * k * 2 + m * n * 2) / (us * 1e-6) / 1e9
                e.update({"GB/s": round(gbs, 1), "hbm_frac": round(gbs / hbm_gbs, 4)})
            else:
                tf = 2.0 * m * n * k / (us * 1e-6) / 1e12
                e.update({"TFLOP/s": round(tf, 1), "frac_of_burst": round(tf / burst_tf, 4)})
            out.append(e)
            del g
        del sets
        torch.cuda.empty_cache()
    return out


PEER_COPY_GBS = 770.0  # measured peer-copy bandwidth per direction per B200 on this NVSwitch fabric


def time_exchange(stack, cfg, world, rank, device, reps=20):
    """Device time of the peer-memory exchange alone: 3 untimed exchanges, a
    barrier, one more untimed exchange enqueued right before the start event
    (it ends on every rank only when every rank has finished it, so the ranks'
    timed regions start together on the device, whatever the host skew after
    the barrier), then `reps` exchanges back to back, max over ranks.  Per
    exchange each GPU's NVLink carries, in each direction, the partials it
    serves to the other ranks plus the normalised rows it stores into them:
    2 * (world - 1) * (tokens / world) * hidden * 2 bytes, the roofline's
    numerator."""
    import torch
    import torch.distributed as tdist

    pb = stack._peer
    xl = stack._bufs[1]["xl"]
    local = cfg.tokens // world
    lo = rank * local
    split = min(max(cfg.img_tokens - lo, 0), local)
    z = torch.zeros((cfg.hidden,), dtype=torch.bfloat16, device=device)
    vec = [(z, z, z, z), (z, z, z, z)]
    for _ in range(3):
        pb.exchange(xl, split, vec, reduce=True, normalize=True)
    torch.cuda.synchronize()
    tdist.barrier()
    pb.exchange(xl, split, vec, reduce=True, normalize=True)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        pb.exchange(xl, split, vec, reduce=True, normalize=True)
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / reps], device=device, dtype=torch.float64)
    tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
    us = float(t.item()) * 1e3
    remote = 2 * (world - 1) * local * cfg.hidden * 2
    gbs = remote / (us * 1e-6) / 1e9
    return {"us_per_exchange": round(us, 2), "nvlink_bytes_per_direction": int(remote),
            "achieved_gbs_per_direction": round(gbs, 1), "peak_gbs_per_direction": PEER_COPY_GBS,
            "frac": round(gbs / PEER_COPY_GBS, 4),
            "what": "qmm_tp_signal_ready + qmm_tp_reduce_norm_gather + qmm_tp_wait_gathered on zeroed "
                    f"vectors, {reps} back to back after an aligning exchange, max over ranks; bytes = partials "
                    "served + rows stored per GPU per direction; peak = measured peer copy per direction"}


def choose_peak(region_s, clocks):
    """Burst or sustained bf16 denominator for a kernel timed in a region of
    `region_s` seconds with clock record `clocks`: sustained only when the
    region lasts seconds and the record shows the power cap (or clocks held
    well below the maximum); burst otherwise."""
    burst, sustained, _hbm, kind = measured_peaks()
    capped = "sw_power_cap" in (clocks.get("reasons") or [])
    low = bool(clocks.get("sm_mhz") and clocks.get("sm_max_mhz") and clocks["sm_mhz"] < 0.9 * clocks["sm_max_mhz"])
    if region_s >= 1.0 and (capped or low):
        return sustained, f"{kind} sustained cuBLAS bf16 (MEASURED_PEAKS.json bf16_tflops_sustained): " \
                          f"the timed region lasted {region_s:.1f} s under the power cap; burst {burst}"
    return burst, f"{kind} burst cuBLAS bf16 (MEASURED_PEAKS.json bf16_tflops): the timed region lasted " \
                  f"{region_s * 1e3:.0f} ms{' (power cap seen)' if capped else ''}; sustained {sustained}"


TP_PARITY_CFG = dict(img_tokens=448, txt_tokens=64, blocks=2, hidden=1024, heads=8, head_dim=128, ffn=2048)


def tp_parity(bits, rank, world, device, sp_chunks=1, peer=False):
    """Untimed check on every rank: a small stack sharded over the N ranks
    (sequence-parallel form, NCCL) against the same weights on this rank
    alone; max|d| / max|ref| <= 1e-2 and mean|d| / max|ref| <= 1e-3."""
    import torch
    import torch.distributed as tdist

    from qwen_imager_b200.dit_stack import DitStack, StackConfig, TensorParallel, stream_weights_full
    from qwen_imager_b200.quant import Affine

    cfg = StackConfig(bits=bits, **TP_PARITY_CFG)
    g = torch.Generator().manual_seed(77)
    full = [[stream_weights_full(cfg, g, "cpu") for _ in range(2)] for _ in range(cfg.blocks)]

    def to_dev(a):
        return Affine(packed=a.packed.to(device), scales=a.scales.to(device), offsets=a.offsets.to(device),
                      bias=None if a.bias is None else a.bias.to(device), bits=a.bits, group=a.group, input=a.input)

    full = [[{k: to_dev(v) for k, v in f.items()} for f in blk] for blk in full]
    x = torch.randn((cfg.tokens, cfg.hidden), generator=g).to(torch.bfloat16).to(device)
    temb = torch.randn((cfg.hidden,), generator=g).to(torch.bfloat16).to(device)
    ref = DitStack.from_full(cfg, full, TensorParallel()).forward(x.clone(), temb).float()
    got = DitStack.from_full(cfg, full, TensorParallel(rank, world, sp_chunks=sp_chunks, peer=peer)).forward(
        x.clone(), temb).float()
    torch.cuda.synchronize()
    d = (got - ref).abs()
    scale = ref.abs().max()
    errs = torch.tensor([float(d.max() / scale), float(d.mean() / scale), float(d.mean() / ref.abs().mean())],
                        dtype=torch.float64, device=device)
    tdist.all_reduce(errs, op=tdist.ReduceOp.MAX)
    mx, mean, mm = (float(v) for v in errs.tolist())
    form = ("sequence-parallel, peer-memory exchange (qmm_tp_*: f32 sum of the partials)" if peer else
            f"sequence-parallel (reduce-scatter + all-gather, NCCL bf16), {sp_chunks} token chunk(s)")
    return {"world": world, "form": form,
            "max_rel": round(mx, 6), "mean_rel": round(mean, 7), "mean_abs_over_mean_abs": round(mm, 6),
            "bar": {"max_rel": 1e-2, "mean_rel": 1e-3}, "pass": bool(mx <= 1e-2 and mean <= 1e-3),
            "normalised_by": "max|ref| (the reference test's metric); worst rank",
            "config": f"{cfg.blocks} blocks, {cfg.img_tokens}+{cfg.txt_tokens} tokens, hidden {cfg.hidden}, "
                      f"{cfg.heads} heads x {cfg.head_dim}, ffn {cfg.ffn}, {bits}-bit; TP{world} vs 1 rank"}


def run_stack(args, rank, world, device):
    import torch

    from qwen_imager_b200 import _lib, device_error
    from qwen_imager_b200.dit_stack import STACKS, DitStack, TensorParallel, Timers

    cfg = STACKS[args.workload]
    tp = TensorParallel(rank, world, overlap_chunks=args.overlap_chunks, comm_sms=args.comm_sms,
                        sequence_parallel=not args.replicated, sp_chunks=args.sp_chunks, peer=args.peer)
    stack = DitStack.random(cfg, tp, seed=1, device=device)
    g = torch.Generator(device=device)
    g.manual_seed(1234)  # the same hidden state and timestep on every rank
    x0 = torch.randn((cfg.tokens, cfg.hidden), generator=g, device=device).to(torch.bfloat16)
    temb = torch.randn((cfg.hidden,), generator=g, device=device).to(torch.bfloat16)
    x = torch.empty_like(x0)
    dist = world > 1
    if dist:
        import torch.distributed as tdist

    def step(timers=None):
        x.copy_(x0)
        stack.forward(x, temb, timers)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    if device_error(device):
        raise RuntimeError("device-side wait expired during warm-up")
    if not torch.isfinite(x.float()).all():
        raise RuntimeError("non-finite hidden state after one step")
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(torch.cuda.current_device())
    if dist:
        tdist.barrier()
    torch.cuda.synchronize()
    launches0 = _lib.launch_count()
    with sampler:
        t0.record()
        for _ in range(args.steps):
            step()
        t1.record()
        torch.cuda.synchronize()
    launches = _lib.launch_count() - launches0
    elapsed = t0.elapsed_time(t1)
    if dist:
        t = torch.tensor([elapsed], device=device, dtype=torch.float64)
        tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
        elapsed = float(t.item())
    ms = elapsed / args.steps
    clocks = sampler.summary()

    # One more step with CUDA events around every op category, inside an NVTX
    # range ("dit_step") so that a profiler can capture exactly one step.
    timers = Timers(enabled=True)
    if dist:
        tdist.barrier()
    torch.cuda.nvtx.range_push("dit_step")
    step(timers)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    parts = {k: round(v, 3) for k, v in timers.totals_ms().items()}
    lin_flops = cfg.blocks * cfg.linear_flops_per_block()
    att_flops = cfg.blocks * cfg.attention_flops_per_block()

    # Per-launch time of every distinct linear on this rank; the roofline is
    # that of the GEMM with the largest share of the step.
    layer_sampler = ClockSampler(torch.cuda.current_device())
    lt0 = time.perf_counter()
    with layer_sampler:
        layers = time_stack_layers(stack, cfg, world, max(args.steps, 8), device)
    layer_region = time.perf_counter() - lt0
    gemms = [e for e in layers if e["m"] > 16]
    dom = max(gemms, key=lambda e: e["kernel_us"] * e["launches_per_step"])
    peak, peak_source = choose_peak(layer_region / max(1, len(layers)), layer_sampler.summary())
    achieved = dom["alg_flops"] / (dom["kernel_us"] * 1e-6) / 1e12
    roof = {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
            "frac": round(achieved / peak, 4),
            # the committed capture is of the one-rank shape; the shards of N > 1 are other shapes
            "traffic": profile_traffic(args.workload) if world == 1 else None,
            "kernel": f"{dom['layer']} GEMM {dom['m']}x{dom['k']}x{dom['n']} {cfg.bits}-bit ({dom['epilogue']}), "
                      f"rank 0",
            "kernel_ms": round(dom["kernel_us"] * 1e-3, 5), "peak_source": peak_source,
            "layer_clocks": layer_sampler.summary()}
    for e in layers:
        if "TFLOP/s" in e:
            e["frac_of_peak"] = round(e["TFLOP/s"] / peak, 4)
        else:
            e["hbm_frac"] = round(e["GB/s"] / measured_peaks()[2], 4)

    e2e = None
    if not args.no_e2e:
        hx = torch.empty(x0.shape, dtype=x0.dtype, pin_memory=True)
        hx.copy_(x0)
        ht = torch.empty(temb.shape, dtype=temb.dtype, pin_memory=True)
        ht.copy_(temb)
        hy = torch.empty(x0.shape, dtype=x0.dtype, pin_memory=True)
        tt = torch.empty_like(temb)

        def e2e_step():
            x.copy_(hx, non_blocking=True)
            tt.copy_(ht, non_blocking=True)
            stack.forward(x, tt)
            hy.copy_(x, non_blocking=True)

        e2e_step()
        torch.cuda.synchronize()
        if dist:
            tdist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n_e2e = max(2, min(args.steps, 5))
        a.record()
        for _ in range(n_e2e):
            e2e_step()
        b.record()
        torch.cuda.synchronize()
        e_ms = a.elapsed_time(b) / n_e2e
        if dist:
            t = torch.tensor([e_ms], device=device, dtype=torch.float64)
            tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
            e_ms = float(t.item())
        e2e = {"value": round(e_ms, 3), "unit": "ms", "h2d_bytes_per_step": int(hx.numel() * 2 + ht.numel() * 2),
               "d2h_bytes_per_step": int(hy.numel() * 2),
               "what": "the public DitStack.forward with the hidden state and timestep copied in from pinned host "
                       "memory and the new hidden state read back, every step (bytes per rank)"}
    exchange = time_exchange(stack, cfg, world, rank, device) if (dist and tp.peer) else None
    if device_error(device):
        raise RuntimeError("device-side wait expired during the timed region")
    parity = (tp_parity(cfg.bits, rank, world, device, args.sp_chunks, args.peer)
              if (dist and not args.no_parity) else None)
    breakdown = {"ms_" + k: v for k, v in parts.items()}
    lin_ms = parts.get("linear", 0.0) + parts.get("rowpar_linear+all_reduce", 0.0)
    breakdown.update({
        "linear_tflops_per_rank": round(lin_flops / world / (lin_ms * 1e-3) / 1e12, 1) if lin_ms else None,
        "attention_tflops_per_rank": round(att_flops / world / (parts.get("attention", float("nan")) * 1e-3) / 1e12, 1),
        "linear_tflop_per_step": round(lin_flops / 1e12, 2), "attention_tflop_per_step": round(att_flops / 1e12, 2),
        "collectives_per_step": ((2 * cfg.blocks + 2 if tp.peer else
                                  4 * cfg.blocks + 1 if tp.sequence_parallel else 2 * cfg.blocks)
                                 + (1 if dist else 0)),
    })
    configs = time_configs(device) if (world == 1 and not args.no_configs) else None
    return {"value": round(ms, 3), "ms_per_step": round(ms, 3), "e2e": e2e, "roofline": roof,
            "gpu_launches": int(launches), "breakdown": breakdown, "clocks": clocks, "layers": layers,
            "configs": configs, "exchange": exchange, "tp_parity": parity, "form": "sequence-parallel" if tp.sequence_parallel else
            ("replicated" if dist else "one rank")}


STACK_PIECES = ("modulation", "img_qkv", "img_out", "img_up", "img_down", "txt_linears", "attention", "norms")


def cpu_stack_reference(workload, steps, warmup=0):
    """The reference CPU path for the stack, timed on whole pieces of one
    block: every linear runs as the reference's CPU path does
    (src/quant.rs:105-113: the weight dequantized to f32 in full on every
    call, an f32 GEMM over all its tokens, f32 bias, bf16 output), plus the
    block's f32 joint attention over all tokens and its norms.  Each bench
    step times one piece (rotating); every piece is timed at least once; the
    block time is the sum of the pieces' medians and the step time that x 60
    (the blocks are identical in cost).  Returns (step ms, cores, sample
    description, mean seconds per bench step)."""
    import numpy as np
    import torch

    from oracle import oracle as O
    from qwen_imager_b200.dit_stack import STACKS

    O.build()
    cfg = STACKS[workload]
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    O.lib().oracle_set_threads(threads)
    rng = np.random.default_rng(7)
    h, f, d = cfg.hidden, cfg.ffn, cfg.heads * cfg.head_dim
    shapes = {"mod": (cfg.mod_features, h), "qkv": (3 * d, h), "out": (h, d), "up": (f, h), "down": (h, f)}
    weights = {}
    for name, (n, k) in shapes.items():
        w = rng.standard_normal((n, k), dtype=np.float32) * 0.02
        weights[name] = O.quantize_affine(w, cfg.bits, cfg.group)
    bias = O.f32_to_bf16((rng.standard_normal(h) * 0.01).astype(np.float32))

    def linear(name, m):
        k = shapes[name][1]
        x = O.f32_to_bf16(rng.standard_normal((m, k), dtype=np.float32))
        packed, scales, offsets = weights[name]
        t0 = time.perf_counter()
        wf = O.dequantize_f32(packed, scales, offsets, cfg.bits, cfg.group)
        y = torch.from_numpy(O.bf16_to_f32(x)) @ torch.from_numpy(wf).T
        if name in ("out", "down"):
            y += torch.from_numpy(O.bf16_to_f32(bias))
        O.f32_to_bf16(y.numpy())
        return time.perf_counter() - t0

    def piece(name):
        if name == "modulation":
            return linear("mod", 1) + linear("mod", 1)
        if name.startswith("img_"):
            return linear(name[4:], cfg.img_tokens)
        if name == "txt_linears":
            return sum(linear(n, cfg.txt_tokens) for n in ("qkv", "out", "up", "down"))
        if name == "attention":
            q, k, v = (torch.randn((1, cfg.heads, cfg.tokens, cfg.head_dim)) for _ in range(3))
            t0 = time.perf_counter()
            torch.nn.functional.scaled_dot_product_attention(q, k, v)
            return time.perf_counter() - t0
        # norms: per stream two LayerNorm + modulation passes and two gated residual adds (f32)
        xs = torch.randn((cfg.tokens, h))
        sh, sc, gt = (torch.randn(h) for _ in range(3))
        t0 = time.perf_counter()
        for _ in range(2):
            n = torch.nn.functional.layer_norm(xs, (h,), eps=1e-6) * (1 + sc) + sh
            xs = xs + gt * n
        return time.perf_counter() - t0

    times = {p: [] for p in STACK_PIECES}
    spent = []
    for i in range(warmup + steps):
        p = STACK_PIECES[i % len(STACK_PIECES)]
        t = piece(p)
        spent.append(t)
        if i >= warmup:
            times[p].append(t)
    for p in STACK_PIECES:  # pieces the rotation did not reach
        if not times[p]:
            times[p].append(piece(p))
    block_s = sum(statistics.median(v) for v in times.values())
    sample = (f"one block of the stack timed piece by piece ({', '.join(STACK_PIECES)}; each bench step times "
              f"one piece in rotation, every piece at least once), every linear over all its tokens with its "
              f"weight dequantized to f32 in full per call; block time = sum of piece medians = "
              f"{block_s:.2f} s, x{cfg.blocks} blocks")
    return block_s * cfg.blocks * 1e3, threads, sample, statistics.mean(spent)


# --------------------------------------------------------------------- CPU arm
def cpu_reference(layers, seed, steps, warmup, budget_s=120.0):
    """Times the reference CPU path (the oracle's restatement of
    src/quant.rs:105-113) for one step of the workload: every weight
    dequantized to f32 in full per call, an f32 GEMM over all token rows, f32
    bias, bf16 output.  Steps beyond what fits in `budget_s` seconds are not
    run (the number timed is in the sample description)."""
    import numpy as np
    import torch

    from oracle import oracle as O

    O.build()
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    O.lib().oracle_set_threads(threads)
    rng = np.random.default_rng(seed)
    data = []
    for (m, k, n, bits, ex) in layers:
        w = (rng.standard_normal((n, k), dtype=np.float32) * 0.02)
        packed, scales, biases = O.quantize_affine(w, bits, 64)
        x = O.f32_to_bf16(rng.standard_normal((m, k), dtype=np.float32))
        b = O.f32_to_bf16((rng.standard_normal(n) * 0.01).astype(np.float32)) if ex.get("bias") else None
        data.append((packed, scales, biases, bits, x, b))

    def one_step():
        t0 = time.perf_counter()
        for (packed, scales, biases, bits, x, b) in data:
            wf = O.dequantize_f32(packed, scales, biases, bits, 64)
            y = torch.from_numpy(O.bf16_to_f32(x)) @ torch.from_numpy(wf).T
            if b is not None:
                y += torch.from_numpy(O.bf16_to_f32(b))
            O.f32_to_bf16(y.numpy())
        return time.perf_counter() - t0

    first = one_step()
    fit = max(1, int(budget_s / max(first, 1e-6)))
    n_warm = min(max(warmup - 1, 0), fit // 4)
    n_steps = max(1, min(steps, fit - n_warm))
    for _ in range(n_warm):
        one_step()
    times = [one_step() for _ in range(n_steps)]
    t = statistics.median(times)
    sample = (f"per step: every weight dequantized to f32 in full (as the reference does per call), f32 GEMM over "
              f"all {max(l[0] for l in layers)} token rows, bf16 output; median of {n_steps} steps"
              + (f" (of {steps} asked; the rest did not fit {budget_s:.0f} s)" if n_steps < steps else ""))
    return step_flops(layers) / t / 1e12, t, threads, sample


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.workload in STACK_WORKLOADS:
        return main_stack(args, world, rank, local)
    desc, layers, seed = WORKLOADS[args.workload]
    config = {"workload": f"{args.workload}: {desc}", "global_batch": world,
              "tokens_per_rank": max(l[0] for l in layers), "group": 64,
              "parallelism": f"dp{world} (independent token batches)",
              "l2": "per linear " + "/".join(str(rotation(l)) for l in layers)
                    + " rotating weight/input sets, together at least 2x the 126 MB L2 (no flush)",
              "launch": "the K timed steps replayed as one CUDA graph; e2e through the eager public API",
              "weights": "immutable after load (qmm_set_weights_immutable(1): the GEMVs stream weights before "
                         "their dependency wait)"}

    if args.impl == "reference":
        if rank != 0:
            return
        value, t, cores, sample = cpu_reference(layers, seed, args.steps, args.warmup)
        out = {"metric": METRIC, "value": round(value, 5), "unit": "TFLOP/s", "impl": "reference",
               "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
               "ms_per_step": round(t * 1e3, 3), "higher_is_better": True, "scaling": "weak",
               "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config,
               "cpu_baseline": {"value": round(value, 5), "unit": "TFLOP/s", "cores": cores, "kind": "port",
                                "sample": sample},
               "e2e": {"value": round(value, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                       "d2h_bytes_per_step": 0}}
        print(json.dumps(out), flush=True)
        return

    import torch

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as tdist
        tdist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=120))
    try:
        res = run_ours(args, rank, world, device)
    finally:
        if world > 1:
            import torch.distributed as tdist
            tdist.barrier()
    out = {"metric": METRIC, "value": res["value"], "unit": "TFLOP/s", "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["ms_per_step"],
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
           "data": "synthetic (seeded random weights, MLX affine quantized; random activations)",
           "config": config, "e2e": res["e2e"], "roofline": res["roofline"],
           "gpu_launches": res["gpu_launches"], "clocks": res["clocks"], "layers": res["layers"]}
    if rank == 0 and world == 1 and not args.no_cpu:
        try:
            value, t, cores, sample = cpu_reference(layers, seed, 3, 1, budget_s=30.0)
            out["cpu_baseline"] = {"value": round(value, 5), "unit": "TFLOP/s", "cores": cores,
                                   "kind": "port", "sample": sample}
        except Exception as exc:  # the CPU leg must not hide the GPU result
            out["cpu_baseline"] = {"value": None, "error": str(exc)[:200]}
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        import torch.distributed as tdist
        tdist.destroy_process_group()


def main_stack(args, world, rank, local):
    from qwen_imager_b200.dit_stack import STACKS
    cfg = STACKS[args.workload]
    if args.replicated:
        form = "replicated hidden state, NCCL all-reduce after each row-parallel layer"
    elif args.peer:
        form = ("sequence-parallel over peer memory: after each row-parallel layer one qmm_tp_* exchange sums "
                "the ranks' partials of the local tokens in f32, applies residual + LayerNorm + modulation and "
                "writes the result into every rank's input buffer")
    else:
        form = ("sequence-parallel: NCCL reduce-scatter after each row-parallel layer, fused residual + LayerNorm + "
                "modulation on the local tokens, NCCL all-gather before each column-parallel layer")
    config = {"workload": f"{args.workload}: {STACK_WORKLOADS[args.workload]}", "global_batch": 1,
              "tokens": cfg.tokens, "hidden": cfg.hidden, "blocks": cfg.blocks, "bits": cfg.bits, "group": cfg.group,
              "parallelism": f"tp{world} (column-parallel QKV/up/modulation, row-parallel out/down; {form})"
                             if world > 1 else "tp1",
              "overlap_chunks": args.overlap_chunks, "sp_chunks": args.sp_chunks, "peer_collectives": args.peer and world > 1,
              "l2": "weights of every step (GBs) far exceed L2 (no flush); per-layer timings walk over the blocks' "
                    "weights (inputs + weights of each launch > 126 MB)"}
    common = {"metric": STACK_METRIC, "unit": "ms", "steps": args.steps, "warmup": args.warmup,
              "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "config": config}
    if args.impl == "reference":
        if rank != 0:
            return
        ms, cores, sample, per_step_s = cpu_stack_reference(args.workload, args.steps, args.warmup)
        out = dict(common, value=round(ms, 1), impl="reference", n_gpus=args.gpus,
                   ms_per_step=round(per_step_s * 1e3, 1), dtype="f32", data="synthetic",
                   cpu_baseline={"value": round(ms, 1), "unit": "ms", "cores": cores, "kind": "port",
                                 "sample": sample + "; ms_per_step is the mean wall time of one bench step "
                                                    "(one piece), value the whole denoising step"},
                   e2e={"value": round(ms, 1), "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0})
        print(json.dumps(out), flush=True)
        return
    import torch

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as tdist
        if args.sp_chunks > 1:
            # Collectives that overlap the GEMMs run on the SMs the GEMMs leave.
            os.environ.setdefault("NCCL_MAX_CTAS", str(args.comm_sms))
        tdist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=180))
    try:
        res = run_stack(args, rank, world, device)
        out = dict(common, value=res["value"], n_gpus=world, ms_per_step=res["ms_per_step"], dtype="bf16",
                   data="synthetic (random 4/8-bit codes with N(0,0.02)-sized scales; random hidden state)",
                   e2e=res["e2e"], roofline=res["roofline"], gpu_launches=res["gpu_launches"],
                   clocks=res["clocks"], breakdown=res["breakdown"], layers=res["layers"],
                   tp_parity=res["tp_parity"])
        if res["configs"] is not None:
            out["configs"] = res["configs"]
        if res["exchange"] is not None:
            out["exchange"] = res["exchange"]
        if rank == 0 and world == 1 and not args.no_cpu:
            try:
                ms, cores, sample, _ = cpu_stack_reference(args.workload, len(STACK_PIECES))
                out["cpu_baseline"] = {"value": round(ms, 1), "unit": "ms", "cores": cores, "kind": "port",
                                       "sample": sample}
            except Exception as exc:
                out["cpu_baseline"] = {"value": None, "error": str(exc)[:200]}
        if rank == 0:
            print(json.dumps(out), flush=True)
    finally:
        if world > 1:
            import torch.distributed as tdist
            tdist.barrier()
            tdist.destroy_process_group()


if __name__ == "__main__":
    main()
