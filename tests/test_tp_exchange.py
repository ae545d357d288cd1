"""The peer-memory exchange of the tensor-parallel stack (include/qmm.h,
qmm_tp_*): argument checks on the CPU (every refusal comes before any CUDA
call), and on one B200 the exchange of a one-rank group against a plain f32
computation of the same steps: x <- bf16(x + sum of partials + gate * bias)
and gathered <- bf16(LayerNorm(x) * (1 + scale) + shift), per stream
(src/dit.rs:50,88-93 is the reference's residual update and norm).  With one
rank the exchange's waits are met by the kernels before it on the stream, so
no kernel waits on another that runs beside it."""
import ctypes

import numpy as np
import pytest
import torch

from qwen_imager_b200 import _lib, device_error


def _peers(world=1, rank=0, part=0x1000, gathered=0x2000, counters=0x3000):
    p = _lib.QmmTpPeers()
    p.world, p.rank = world, rank
    for j in range(max(0, min(world, _lib.QMM_TP_MAX_RANKS))):
        p.part[j], p.gathered[j], p.counters[j] = part, gathered, counters
    return p


def test_peer_set_is_checked_before_any_launch():
    lib = _lib.load()
    assert lib.qmm_tp_signal_ready(None, None) == _lib.QMM_ERR_INVALID_ARGUMENT
    assert lib.qmm_tp_wait_gathered(None, 1, None) == _lib.QMM_ERR_INVALID_ARGUMENT
    for world, rank in ((0, 0), (_lib.QMM_TP_MAX_RANKS + 1, 0), (2, 2), (2, -1)):
        p = _peers(world=world, rank=rank)
        assert lib.qmm_tp_signal_ready(ctypes.byref(p), None) == _lib.QMM_ERR_INVALID_ARGUMENT, (world, rank)
    p = _peers(world=2)
    p.gathered[1] = None  # rank 1's buffers are missing
    assert lib.qmm_tp_signal_ready(ctypes.byref(p), None) == _lib.QMM_ERR_INVALID_ARGUMENT
    p = _peers(counters=0x3008)  # not 16-byte aligned
    assert lib.qmm_tp_signal_ready(ctypes.byref(p), None) == _lib.QMM_ERR_MISALIGNED


# ------------------------------------------------------------------ one B200
def _bf16(t):
    return t.to(torch.bfloat16)


def _reference(x, part, vecs, split, eps):
    """f32 restatement of the exchange for one rank: returns (x', gathered)."""
    rows = x.shape[0]
    xn = torch.empty_like(x)
    g = torch.empty_like(x)
    for s, sl in enumerate((slice(0, split), slice(split, rows))):
        bias, gate, shift, scale = vecs[s]
        t = x[sl].float() + part[sl].float() + gate.float() * bias.float()
        xb = _bf16(t)
        xn[sl] = xb
        v = xb.float()
        mean = v.mean(dim=1, keepdim=True)
        var = ((v - mean) ** 2).mean(dim=1, keepdim=True)
        g[sl] = _bf16((v - mean) * torch.rsqrt(var + eps) * (1.0 + scale.float()) + shift.float())
    return xn, g


@pytest.mark.gpu
@pytest.mark.parametrize("rows,hidden,split", [(300, 3072, 150), (148 * 3 + 5, 1024, 0), (64, 4096, 64),
                                               (37, 256, 20)])
def test_one_rank_exchange_matches_f32_steps(rows, hidden, split):
    lib = _lib.load()
    dev = torch.device("cuda")
    g = torch.Generator(device=dev)
    g.manual_seed(rows + hidden)
    x = _bf16(torch.randn((rows, hidden), generator=g, device=dev))
    part = _bf16(torch.randn((rows, hidden), generator=g, device=dev))
    gathered = torch.zeros((rows, hidden), dtype=torch.bfloat16, device=dev)
    counters = torch.zeros((4,), dtype=torch.int64, device=dev)
    vecs = [tuple(_bf16(0.3 * torch.randn((hidden,), generator=g, device=dev)) for _ in range(4)) for _ in range(2)]
    eps = 1e-6
    peers = _peers(part=part.data_ptr(), gathered=gathered.data_ptr(), counters=counters.data_ptr())
    norm = _lib.QmmTpNorm()
    for s in range(2):
        norm.bias[s], norm.gate[s], norm.shift[s], norm.scale[s] = (t.data_ptr() for t in vecs[s])
    norm.split, norm.eps = split, eps
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for epoch in (1, 2):  # the second exchange checks the counters' epochs; x is updated twice
        want_x, want_g = _reference(x, part, vecs, split, eps)
        assert lib.qmm_tp_signal_ready(ctypes.byref(peers), st) == _lib.QMM_OK
        assert lib.qmm_tp_reduce_norm_gather(ctypes.byref(peers), epoch, rows, hidden, ctypes.c_void_p(x.data_ptr()),
                                             ctypes.byref(norm), 1, 1, st) == _lib.QMM_OK
        assert lib.qmm_tp_wait_gathered(ctypes.byref(peers), epoch, st) == _lib.QMM_OK
        torch.cuda.synchronize()
        assert device_error() == 0
        # One rounding of the f32 sum: equal to the f32 steps, or one bf16 ulp off where the
        # kernel's fused multiply-add rounds the gate * bias product differently.
        d = (x.float() - want_x.float()).abs()
        ulp = torch.clamp(want_x.float().abs(), min=2.0 ** -126) * 2.0 ** -7
        assert bool((d <= ulp).all()), (epoch, float((d / ulp).max()))
        dg = (gathered.float() - want_g.float()).abs()
        assert float(dg.max()) <= 2.0 ** -6 * max(1.0, float(want_g.float().abs().max())), (epoch, float(dg.max()))
        assert float(dg.mean()) <= 1e-3 * float(want_g.float().abs().mean()), epoch
    np.testing.assert_array_equal(counters[:2].cpu().numpy(), [2, 2])  # ready, done after two epochs


@pytest.mark.gpu
def test_a_rank_that_never_signals_is_reported_as_a_timeout():
    """A two-rank group emulated in one process whose rank 1 never runs: rank
    0's exchange waits for rank 1's ready signal (a counter nothing else will
    raise), gives up after its bounded wait (4 s), skips its work and reports
    QMM_ERR_TIMEOUT through qmm_device_error; the context stays usable, and a
    one-rank exchange launched after it is correct."""
    lib = _lib.load()
    dev = torch.device("cuda")
    rows, hidden = 64, 256
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    x = _bf16(torch.randn((rows, hidden), generator=g, device=dev))
    x0 = x.clone()
    part = [torch.zeros((2 * rows, hidden), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    gathered = [torch.zeros((2 * rows, hidden), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    counters = [torch.zeros((4,), dtype=torch.int64, device=dev) for _ in range(2)]
    peers = _peers(world=2, rank=0)
    for j in range(2):
        peers.part[j], peers.gathered[j], peers.counters[j] = (part[j].data_ptr(), gathered[j].data_ptr(),
                                                               counters[j].data_ptr())
    ones = torch.ones((hidden,), dtype=torch.bfloat16, device=dev)
    norm = _lib.QmmTpNorm()
    for s in range(2):
        norm.bias[s], norm.gate[s], norm.shift[s], norm.scale[s] = (ones.data_ptr(),) * 4
    norm.split, norm.eps = rows // 2, 1e-6
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert device_error() == 0
    import time
    t0 = time.monotonic()
    assert lib.qmm_tp_signal_ready(ctypes.byref(peers), st) == _lib.QMM_OK
    assert lib.qmm_tp_reduce_norm_gather(ctypes.byref(peers), 1, rows, hidden, ctypes.c_void_p(x.data_ptr()),
                                         ctypes.byref(norm), 1, 1, st) == _lib.QMM_OK
    assert lib.qmm_tp_wait_gathered(ctypes.byref(peers), 1, st) == _lib.QMM_OK
    torch.cuda.synchronize()
    took = time.monotonic() - t0
    code = ctypes.c_uint32()
    assert lib.qmm_device_error(st, ctypes.byref(code)) == _lib.QMM_ERR_TIMEOUT
    assert code.value != 0
    assert 3.0 < took < 60.0, took
    assert torch.equal(x, x0)  # the exchange skipped its work
    assert not bool(gathered[0].any()) and not bool(gathered[1].any())
    assert device_error() == 0  # reading the code cleared it
    test_one_rank_exchange_matches_f32_steps(37, 256, 20)
