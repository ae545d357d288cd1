"""Host-side logic of the tensor-parallel DiT linear stack, on CPU.

Sharding is checked bit-exactly against the oracle's dequantization, the
row-parallel partial sums against the unsharded product, and a two-rank
`gloo` run of the whole block loop (oracle linears on CPU) against one rank.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from qwen_imager_b200.dit_stack import (DitStack, StackConfig, TensorParallel, shard_input, shard_output,
                                        stack_affine, stream_weights_full)
from qmm_testutil import _bits16, _bits32, oracle_run_linear, rel_errors

# TP-N against one rank, normalised by max|ref| like the reference test
# (src/quant.rs:768-775).  The sequence-parallel form meets the one-rank bar;
# the replicated form rounds each rank's partial with the residual folded in
# (rank 0) and sums the whole hidden state in bf16, two extra roundings at
# the hidden state's full magnitude per row-parallel layer, so its bar on the
# largest element is twice that.
TP_MAX_REL = 1e-2
TP_MAX_REL_REPLICATED = 2e-2
SMALL = StackConfig(img_tokens=96, txt_tokens=32, bits=4, blocks=2, hidden=512, heads=4, head_dim=128,
                    ffn=1024)


def _deq(oracle, a):
    return oracle.dequantize_f32(_bits32(a.packed), _bits16(a.scales), _bits16(a.offsets), a.bits, a.group)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_column_shards_are_row_slices(oracle, bits, world):
    g = torch.Generator().manual_seed(3)
    a = stack_affine(3 * 8 * 64, 256, bits, generator=g, device="cpu")
    full = _deq(oracle, a)
    seg = full.shape[0] // 3
    for r in range(world):
        s = shard_output(a, r, world, segments=3)
        part = seg // world
        want = np.concatenate([full[i * seg + r * part:i * seg + (r + 1) * part] for i in range(3)])
        assert np.array_equal(_deq(oracle, s), want)
        assert torch.equal(s.bias, torch.cat([a.bias[i * seg + r * part:i * seg + (r + 1) * part]
                                              for i in range(3)]))


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_row_shards_are_column_slices_and_sum(oracle, bits, world):
    g = torch.Generator().manual_seed(5)
    k = 64 * world * 2
    a = stack_affine(96, k, bits, generator=g, device="cpu")
    full = _deq(oracle, a)
    kw = k // world
    x = oracle.f32_to_bf16(np.random.default_rng(1).standard_normal((7, k)).astype(np.float32))
    total = np.zeros((7, 96))
    for r in range(world):
        s = shard_input(a, r, world)
        assert s.input == kw
        assert (s.bias is not None) == (r == 0)
        assert np.array_equal(_deq(oracle, s), full[:, r * kw:(r + 1) * kw])
        total += oracle.linear_f32(x[:, r * kw:(r + 1) * kw], _bits32(s.packed), _bits16(s.scales),
                                   _bits16(s.offsets), bits, 64, None if s.bias is None else _bits16(s.bias))
    ref = oracle.linear_f32(x, _bits32(a.packed), _bits16(a.scales), _bits16(a.offsets), bits, 64,
                            _bits16(a.bias))
    assert np.abs(total - ref).max() <= 1e-5 * np.abs(ref).max()


def test_shards_reject_split_groups():
    g = torch.Generator().manual_seed(0)
    a = stack_affine(64, 192, 4, generator=g, device="cpu")
    with pytest.raises(ValueError):
        shard_input(a, 0, 2)  # 96-input shards split a 64-group
    with pytest.raises(ValueError):
        shard_output(a, 0, 3, segments=2)


@pytest.mark.parametrize("world", [5, 16])
def test_stack_rejects_world_sizes_that_split_heads_or_groups(world):
    with pytest.raises(ValueError):
        StackConfig(img_tokens=4096, txt_tokens=256, bits=4).check_world(world)


def test_stack_configs_shard_at_1_2_4_8():
    from qwen_imager_b200.dit_stack import STACKS
    for cfg in STACKS.values():
        for w in (1, 2, 4, 8):
            cfg.check_world(w)


def _full_weights(cfg, seed):
    g = torch.Generator().manual_seed(seed)
    return [[stream_weights_full(cfg, g, "cpu") for _ in range(2)] for _ in range(cfg.blocks)]


def _inputs(cfg, seed):
    g = torch.Generator().manual_seed(seed + 1)
    x = torch.randn((cfg.tokens, cfg.hidden), generator=g).to(torch.bfloat16)
    temb = torch.randn((cfg.hidden,), generator=g).to(torch.bfloat16)
    return x, temb


def _run_stack(cfg, rank, world, seed, sp=True, chunks=1):
    x, temb = _inputs(cfg, seed)
    stack = DitStack.from_full(cfg, _full_weights(cfg, seed),
                               TensorParallel(rank, world, sequence_parallel=sp, sp_chunks=chunks),
                               run_linear=oracle_run_linear)
    return stack.forward(x, temb)


def _gloo_rank(rank, world, port, seed, path, sp=True, chunks=1):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        y = _run_stack(SMALL, rank, world, seed, sp, chunks)
        torch.save(y, f"{path}.{rank}")
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,sp", [(2, True), (4, True), (2, False)], ids=["sp2", "sp4", "replicated2"])
def test_gloo_stack_matches_one_rank(tmp_path, world, sp):
    seed = 11
    ref = _run_stack(SMALL, 0, 1, seed)
    path = str(tmp_path / "y")
    mp.start_processes(_gloo_rank, args=(world, _free_port(), seed, path, sp), nprocs=world, start_method="spawn")
    bar = TP_MAX_REL if sp else TP_MAX_REL_REPLICATED
    for r in range(world):
        y = torch.load(f"{path}.{r}")
        mx, mean = rel_errors(_bits16(y), ref.float().numpy())
        assert mx <= bar and mean <= 1e-3, (r, mx, mean)
    for r in range(1, world):  # every rank ends with the same whole hidden state
        assert torch.equal(torch.load(f"{path}.0"), torch.load(f"{path}.{r}"))


def test_chunked_sequence_parallel_equals_unchunked(tmp_path):
    # Two token chunks pipeline the collectives against the linears; with two
    # ranks every sum is one addition in either form, so the result is
    # bit-identical (with more ranks the reduction order of the collective
    # may differ with the message size; see the next test).
    seed, world = 13, 2
    outs = {}
    for chunks in (1, 2):
        path = str(tmp_path / f"c{chunks}")
        mp.start_processes(_gloo_rank, args=(world, _free_port(), seed, path, True, chunks), nprocs=world,
                           start_method="spawn")
        outs[chunks] = [torch.load(f"{path}.{r}") for r in range(world)]
    for r in range(world):
        assert torch.equal(outs[1][r], outs[2][r]), r


def test_chunked_sequence_parallel_four_ranks_matches_one_rank(tmp_path):
    seed, world = 13, 4
    ref = _run_stack(SMALL, 0, 1, seed)
    path = str(tmp_path / "y")
    mp.start_processes(_gloo_rank, args=(world, _free_port(), seed, path, True, 2), nprocs=world,
                       start_method="spawn")
    for r in range(world):
        mx, mean = rel_errors(_bits16(torch.load(f"{path}.{r}")), ref.float().numpy())
        assert mx <= TP_MAX_REL and mean <= 1e-3, (r, mx, mean)


def test_sequence_parallel_needs_tokens_divisible_by_ranks():
    cfg = StackConfig(img_tokens=97, txt_tokens=32, bits=4, blocks=1, hidden=512, heads=4, head_dim=128, ffn=1024)
    with pytest.raises(ValueError):
        DitStack.from_full(cfg, _full_weights(cfg, 1), TensorParallel(0, 2), run_linear=oracle_run_linear)
    # the replicated form has no such constraint
    DitStack.from_full(cfg, _full_weights(cfg, 1), TensorParallel(0, 2, sequence_parallel=False),
                       run_linear=oracle_run_linear)


def test_modulation_shards_reassemble_the_whole_modulation(oracle):
    # Column shards of the modulation linear, gathered in rank order, are the
    # unsharded linear's outputs (the all-gather of DitStack.modulations).
    g = torch.Generator().manual_seed(9)
    a = stack_affine(6 * 256, 256, 8, generator=g, device="cpu")
    x = oracle.f32_to_bf16(np.random.default_rng(2).standard_normal((1, 256)).astype(np.float32))
    full = oracle.linear_f32(x, _bits32(a.packed), _bits16(a.scales), _bits16(a.offsets), 8, 64, _bits16(a.bias))
    world = 4
    parts = []
    for r in range(world):
        s = shard_output(a, r, world)
        parts.append(oracle.linear_f32(x, _bits32(s.packed), _bits16(s.scales), _bits16(s.offsets), 8, 64,
                                       _bits16(s.bias)))
    assert np.array_equal(np.concatenate(parts, axis=1), full)
