"""The tensor-parallel DiT linear stack on B200: CUDA linears against the
oracle's linears on CPU, and (with 2, 4 or 8 GPUs) tensor parallelism against
one rank: NCCL collectives (sequence-parallel, chunked, replicated) and the
library's peer-memory collectives (qmm_tp_*)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from qwen_imager_b200.dit_stack import DitStack, StackConfig, TensorParallel, stream_weights_full
from qwen_imager_b200.quant import Affine
from qmm_testutil import _bits16, oracle_run_linear, rel_errors

pytestmark = pytest.mark.gpu

SMALL = StackConfig(img_tokens=320, txt_tokens=64, bits=4, blocks=2, hidden=512, heads=4, head_dim=128,
                    ffn=1024)
# 8 heads, so that 2, 4 and 8 ranks each hold whole heads.
SMALL_TP = StackConfig(img_tokens=320, txt_tokens=64, bits=4, blocks=2, hidden=512, heads=8, head_dim=128,
                       ffn=1024)
SMALL8 = StackConfig(img_tokens=200, txt_tokens=56, bits=8, blocks=2, hidden=512, heads=4, head_dim=128,
                     ffn=1024)


def _to(a: Affine, device) -> Affine:
    return Affine(packed=a.packed.to(device), scales=a.scales.to(device), offsets=a.offsets.to(device),
                  bias=None if a.bias is None else a.bias.to(device), bits=a.bits, group=a.group, input=a.input)


def _weights(cfg, seed, device):
    g = torch.Generator().manual_seed(seed)
    full = [[stream_weights_full(cfg, g, "cpu") for _ in range(2)] for _ in range(cfg.blocks)]
    return [[{k: _to(v, device) for k, v in f.items()} for f in blk] for blk in full]


def _inputs(cfg, seed):
    g = torch.Generator().manual_seed(seed + 1)
    return (torch.randn((cfg.tokens, cfg.hidden), generator=g).to(torch.bfloat16),
            torch.randn((cfg.hidden,), generator=g).to(torch.bfloat16))


@pytest.mark.parametrize("cfg", [SMALL, SMALL8], ids=["4bit", "8bit"])
def test_stack_cuda_matches_oracle_stack(cfg):
    seed = 21
    x, temb = _inputs(cfg, seed)
    ref = DitStack.from_full(cfg, _weights(cfg, seed, "cpu"), TensorParallel(),
                             run_linear=oracle_run_linear).forward(x.clone(), temb)
    got = DitStack.from_full(cfg, _weights(cfg, seed, "cuda"), TensorParallel()).forward(x.cuda(), temb.cuda())
    mx, mean = rel_errors(_bits16(got), ref.float().numpy())
    assert mx <= 1e-2 and mean <= 1e-3, (mx, mean)


def _nccl_rank(rank, world, port, seed, path, sp, chunks=1, peer=False):
    import datetime

    import torch.distributed as dist
    if peer == "lanes":  # the exchange's per-lane-store variant, read when the library first launches it
        os.environ["QMM_TP_BULK_STORE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        x, temb = _inputs(SMALL_TP, seed)
        dev = torch.device("cuda", rank)
        stack = DitStack.from_full(SMALL_TP, _weights(SMALL_TP, seed, dev),
                                   TensorParallel(rank, world, sequence_parallel=sp, sp_chunks=chunks,
                                                  peer=bool(peer)))
        y = stack.forward(x.to(dev), temb.to(dev))
        torch.cuda.synchronize()
        torch.save(y.cpu(), f"{path}.{rank}")
        dist.barrier()
    finally:
        dist.destroy_process_group()


# Sequence-parallel TP-N meets the one-rank bar; the replicated form sums the
# whole hidden state in bf16 (see tests/test_dit_stack.py) and gets twice it.
@pytest.mark.parametrize("world,sp,chunks,peer", [(2, True, 1, False), (4, True, 1, False), (8, True, 1, False),
                                                   (2, False, 1, False), (2, True, 2, False), (8, True, 2, False),
                                                   (2, True, 1, True), (4, True, 1, True), (8, True, 1, True),
                                                   (2, True, 1, "lanes"), (8, True, 1, "lanes")],
                         ids=["sp2", "sp4", "sp8", "replicated2", "sp2-chunked", "sp8-chunked",
                              "sp2-peer", "sp4-peer", "sp8-peer", "sp2-peer-lanes", "sp8-peer-lanes"])
def test_stack_nccl_matches_one_rank(tmp_path, world, sp, chunks, peer):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    seed = 23
    x, temb = _inputs(SMALL_TP, seed)
    ref = DitStack.from_full(SMALL_TP, _weights(SMALL_TP, seed, "cuda"), TensorParallel()).forward(x.cuda(),
                                                                                                   temb.cuda())
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    path = str(tmp_path / "y")
    mp.start_processes(_nccl_rank, args=(world, port, seed, path, sp, chunks, peer), nprocs=world,
                       start_method="spawn")
    bar = 1e-2 if sp else 2e-2
    for r in range(world):
        mx, mean = rel_errors(_bits16(torch.load(f"{path}.{r}")), ref.float().cpu().numpy())
        assert mx <= bar and mean <= 1e-3, (r, mx, mean)
