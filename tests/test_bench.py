"""bench.py's contract, checked on the CPU.

- Every linear of every kernel workload rotates over enough input sets that each launch reads its
  operands from HBM: at least three sets, together at least twice the 126 MB L2.
- The reference arm (the CPU path, run here on a small workload) prints one JSON line with the keys the
  driver reads: `impl`, `cpu_baseline` and an `e2e` with no host-device bytes.
"""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


@pytest.mark.parametrize("workload", sorted(bench.WORKLOADS))
def test_every_linear_rotates_past_l2(workload):
    _desc, layers, _seed = bench.WORKLOADS[workload]
    for layer in layers:
        sets = bench.rotation(layer)
        assert sets >= bench.ROTATE
        assert sets * bench.layer_bytes(*layer) >= 2 * bench.L2_BYTES, (workload, layer, sets)


def test_layer_bytes_of_the_adaln_gemv():
    # codes 28.31 MB + scales and offsets 3.54 MB + x 6 KB + y 37 KB
    assert bench.layer_bytes(1, 3072, 18432, 4, {}) == 31893504


def test_reference_arm_prints_the_contract_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "1", "--workload", "adaln_gemv"],
                         capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    line = [ln for ln in out.stdout.splitlines() if ln.startswith("{")][-1]
    d = json.loads(line)
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["steps"] == 1 and d["value"] > 0
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] in ("port", "reference") and cb["cores"] >= 1
    assert cb["sample"]
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["unit"] == d["unit"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert "workload" in d["config"]


def test_default_workload_is_the_tensor_parallel_stack():
    old = sys.argv
    try:
        sys.argv = ["bench.py"]
        a = bench.parse()
    finally:
        sys.argv = old
    assert a.workload == "dit_2048_8bit" and a.gpus == 1 and a.steps == 10 and a.warmup == 3
    assert not a.replicated


def test_stack_layer_shapes_cover_every_linear_of_a_block():
    from qwen_imager_b200.dit_stack import STACKS
    cfg = STACKS["dit_2048_8bit"]
    for world in (1, 2, 4, 8):
        shapes = bench._layer_shapes(cfg, world)
        flops = sum(2.0 * m * k * n * (2 if name == "modulation" else 1) for name, _s, m, k, n, _e in shapes)
        # the block's linear FLOPs divided over the ranks
        assert abs(flops * world - cfg.linear_flops_per_block()) < 1e-6 * flops * world, world


def test_peak_choice_follows_the_timed_region():
    burst, sustained, _, _ = bench.measured_peaks()
    assert bench.choose_peak(0.02, {"reasons": ["sw_power_cap"], "sm_mhz": 1900, "sm_max_mhz": 1965})[0] == burst
    assert bench.choose_peak(5.0, {"reasons": [], "sm_mhz": 1965, "sm_max_mhz": 1965})[0] == burst
    assert bench.choose_peak(5.0, {"reasons": ["sw_power_cap"], "sm_mhz": 1400, "sm_max_mhz": 1965})[0] == sustained


def test_stack_reference_arm_times_every_piece_of_a_block():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "2",
                          "--warmup", "1", "--workload", "dit_1024_4bit"],
                         capture_output=True, text=True, timeout=900, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    d = json.loads([ln for ln in out.stdout.splitlines() if ln.startswith("{")][-1])
    assert d["impl"] == "reference" and d["unit"] == "ms" and d["higher_is_better"] is False
    assert d["steps"] == 2 and d["value"] > 0 and d["cpu_baseline"]["value"] == d["value"]
    for piece in bench.STACK_PIECES:
        assert piece in d["cpu_baseline"]["sample"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0
