"""Failure detection on the host, with `gloo` ranks on the CPU: a rank that
never joins the group, and a rank that leaves (or stalls) between steps of
the tensor-parallel stack.  The surviving rank gets an error within the
process group's short timeout instead of waiting for good."""
import os
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp

from qwen_imager_b200.dit_stack import DitStack, StackConfig, TensorParallel, stream_weights_full
from qmm_testutil import oracle_run_linear

SMALL = StackConfig(img_tokens=96, txt_tokens=32, bits=4, blocks=1, hidden=512, heads=4, head_dim=128, ffn=1024)
TIMEOUT_S = 3


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _record(path, rank, what):
    with open(f"{path}.{rank}", "w") as f:
        f.write(what)


def _absent_peer(rank, world, port, path):
    import datetime

    import torch.distributed as dist
    if rank == 1:
        _record(path, rank, "left")
        return  # never joins
    t0 = time.monotonic()
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=TIMEOUT_S))
        _record(path, rank, "joined")
        dist.destroy_process_group()
    except Exception as exc:  # noqa: BLE001 - the error is the result
        _record(path, rank, f"error {time.monotonic() - t0:.1f} {type(exc).__name__}: {exc}")


def test_rank_that_never_joins_surfaces_a_timeout(tmp_path):
    path = str(tmp_path / "r")
    t0 = time.monotonic()
    mp.start_processes(_absent_peer, args=(2, _port(), path), nprocs=2, start_method="spawn")
    assert time.monotonic() - t0 < 60
    assert open(f"{path}.1").read() == "left"
    got = open(f"{path}.0").read()
    assert got.startswith("error"), got


def _stack_inputs():
    g = torch.Generator().manual_seed(5)
    full = [[stream_weights_full(SMALL, g, "cpu") for _ in range(2)] for _ in range(SMALL.blocks)]
    x = torch.randn((SMALL.tokens, SMALL.hidden), generator=g).to(torch.bfloat16)
    temb = torch.randn((SMALL.hidden,), generator=g).to(torch.bfloat16)
    return full, x, temb


def _peer_leaves_between_steps(rank, world, port, path, mode):
    import datetime

    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=TIMEOUT_S))
    full, x, temb = _stack_inputs()
    stack = DitStack.from_full(SMALL, full, TensorParallel(rank, world), run_linear=oracle_run_linear)
    stack.forward(x.clone(), temb)  # step 1: every rank
    if rank == 1:
        # Leaves between steps, with no collective of its in flight.
        _record(path, rank, "left")
        if mode == "stall":
            time.sleep(4 * TIMEOUT_S)
        os._exit(0)
    t0 = time.monotonic()
    try:
        stack.forward(x.clone(), temb)  # step 2: its first collective has no partner
        _record(path, rank, "finished")
    except Exception as exc:  # noqa: BLE001 - the error is the result
        _record(path, rank, f"error {time.monotonic() - t0:.1f} {type(exc).__name__}")
    os._exit(0)


@pytest.mark.parametrize("mode", ["exit", "stall"])
def test_stack_rank_leaving_between_steps_fails_the_next_collective(tmp_path, mode):
    path = str(tmp_path / "r")
    t0 = time.monotonic()
    ctx = mp.start_processes(_peer_leaves_between_steps, args=(2, _port(), path, mode), nprocs=2,
                             start_method="spawn", join=False)
    while not ctx.join(timeout=60):
        assert time.monotonic() - t0 < 120, "ranks did not end"
    got = open(f"{path}.0").read()
    assert open(f"{path}.1").read() == "left"
    assert got.startswith("error"), got
    assert float(got.split()[1]) < 10 * TIMEOUT_S, got
