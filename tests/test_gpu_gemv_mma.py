"""The tensor-core GEMV (4- and 8-bit, m <= 16, n % 8 == 0, group a multiple
of 64) against the oracle's f32 path (src/quant.rs:105-113): within one bf16
rounding of the oracle for every output, across token counts, row-block
tails, K sizes, group sizes and the fused epilogue; the programmatic
dependent launch with and without the weights-immutable prefetch."""
import numpy as np
import pytest

from qmm_testutil import assert_one_rounding, make_linear, random_layer, sin_input, to_dev_u16
from test_gpu_linear import run
from qwen_imager_b200 import _lib

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("m", list(range(1, 17)))
def test_gemv_mma_token_counts(oracle, m, bits):
    k, n = 1024, 200  # 200 rows: six 32-row blocks and an 8-row tail
    packed, scales, offsets, bias = random_layer(n, k, bits, 64, seed=300 + m + bits)
    lin = make_linear(packed, scales, offsets, bias, bits, 64)
    x = sin_input(m, k)
    got = run(lin, x, path=_lib.QMM_PATH_GEMV)
    assert_one_rounding(got, oracle.linear_f32(x, packed, scales, offsets, bits, 64, bias), oracle)


@pytest.mark.parametrize("k,n,group", [(64, 8, 64), (128, 24, 128), (3072, 512, 64), (3072, 96, 256),
                                       (12288, 64, 64), (4096, 1032, 128), (6144, 40, 64)])
@pytest.mark.parametrize("m", [1, 3, 9])
@pytest.mark.parametrize("bits", [4, 8])
def test_gemv_mma_shapes_and_groups(oracle, k, n, group, m, bits):
    packed, scales, offsets, bias = random_layer(n, k, bits, group, seed=k + n + group + m + bits)
    lin = make_linear(packed, scales, offsets, bias, bits, group)
    x = sin_input(m, k)
    try:
        got = run(lin, x, path=_lib.QMM_PATH_GEMV)
    except _lib.QmmError as exc:
        # x staged for many tokens at large k (twice as large for 8-bit codes,
        # staged as nibble pairs) does not fit shared memory next to the ring:
        # no GEMV covers the layout, and QMM_PATH_AUTO takes the GEMM instead.
        assert exc.status == _lib.QMM_ERR_UNSUPPORTED and (m > 8 or k * bits >= 6144 * 4)
        got = run(lin, x)
        w = oracle.bf16_to_f32(oracle.dequantize_bf16(packed, scales, offsets, bits, group))
        assert_one_rounding(got, oracle.matmul_f32(oracle.bf16_to_f32(x), w, bias), oracle)
        return
    assert_one_rounding(got, oracle.linear_f32(x, packed, scales, offsets, bits, group, bias), oracle)


@pytest.mark.parametrize("bits", [4, 8])
def test_gemv_mma_adaln_shape(oracle, bits):
    # 4-bit: the 1024x1024 stack's modulation; 8-bit: the 2048x2048 stack's
    m, k, n = 1, 3072, 18432
    packed, scales, offsets, bias = random_layer(n, k, bits, 64, seed=5 + bits)
    lin = make_linear(packed, scales, offsets, bias, bits, 64)
    rng = np.random.default_rng(6)
    xf = rng.standard_normal((m, k)).astype(np.float32)
    x = oracle.f32_to_bf16(xf / (1.0 + np.exp(-xf)))  # SiLU input, as the modulation linear sees it
    got = run(lin, x)
    assert_one_rounding(got, oracle.linear_f32(x, packed, scales, offsets, bits, 64, bias), oracle)


@pytest.mark.parametrize("activation,act_code", [(None, 0), ("gelu_tanh", 1), ("silu", 2)])
@pytest.mark.parametrize("m", [1, 12])
@pytest.mark.parametrize("bits", [4, 8])
def test_gemv_mma_fused_epilogue(oracle, activation, act_code, m, bits):
    k, n = 512, 384
    packed, scales, offsets, bias = random_layer(n, k, bits, 64, seed=40 + act_code + m + bits)
    rng = np.random.default_rng(41)
    gate = oracle.f32_to_bf16(rng.standard_normal(n).astype(np.float32))
    residual = oracle.f32_to_bf16(rng.standard_normal((m, n)).astype(np.float32))
    lin = make_linear(packed, scales, offsets, bias, bits, 64)
    x = sin_input(m, k)
    got = run(lin, x, path=_lib.QMM_PATH_GEMV, gate=to_dev_u16(gate), residual=to_dev_u16(residual),
              activation=activation)
    y = oracle.linear_f32(x, packed, scales, offsets, bits, 64, bias)
    ref = oracle.epilogue_bf16(y, gate, residual, act_code)
    d = np.abs(oracle.bf16_to_f32(got) - oracle.bf16_to_f32(ref))
    assert d.max() <= np.abs(oracle.bf16_to_f32(ref)).max() * 2.0**-7


@pytest.mark.parametrize("bits", [4, 8])
def test_gemv_mma_waits_for_the_kernels_before_it(oracle, bits):
    """The GEMV is launched as a programmatic dependent of the kernel before it
    and reads nothing that kernel may write until it has completed.  Here the
    codes, scales, offsets and x are rewritten by elementwise kernels on the
    same stream right before every launch, and every launch's residual is the
    previous launch's output; each result must match the oracle for the data
    of its own iteration."""
    import torch

    k, n, m, iters = 3072, 2048, 1, 8
    packed0, scales0, offsets0, bias = random_layer(n, k, bits, 64, seed=70)
    lin = make_linear(packed0, scales0, offsets0, bias, bits, 64)
    a = lin.affine
    data = []
    for i in range(iters):
        packed, scales, offsets, _ = random_layer(n, k, bits, 64, seed=71 + i, bias=False)
        x = oracle.f32_to_bf16(np.cos(np.arange(k, dtype=np.float64) * (0.11 + 0.07 * i)).astype(np.float32)
                               .reshape(m, k))
        data.append((packed, scales, offsets, x))
    dev = [(to_dev_u32_i32(p), to_dev_u16(s), to_dev_u16(o), to_dev_u16(x)) for p, s, o, x in data]
    xbuf = torch.empty((m, k), dtype=torch.bfloat16, device="cuda")
    residual0 = oracle.f32_to_bf16(np.linspace(-1.0, 1.0, m * n, dtype=np.float32).reshape(m, n))
    prev = to_dev_u16(residual0)
    outs = [torch.empty((m, n), dtype=torch.bfloat16, device="cuda") for _ in range(iters)]
    torch.cuda.synchronize()
    for i, (p, s, o, x) in enumerate(dev):
        torch.add(p, 0, out=a.packed.view(torch.int32))  # kernels, not copies: the launch before the GEMV
        torch.mul(s, 1.0, out=a.scales)
        torch.mul(o, 1.0, out=a.offsets)
        torch.mul(x, 1.0, out=xbuf)
        lin.forward_fused(xbuf, residual=prev, out=outs[i], path=_lib.QMM_PATH_GEMV)
        prev = outs[i]
    torch.cuda.synchronize()
    got = [from_dev(t) for t in outs]
    for i, (packed, scales, offsets, x) in enumerate(data):
        res = residual0 if i == 0 else got[i - 1]
        y = oracle.linear_f32(x, packed, scales, offsets, bits, 64, bias)
        ref = oracle.epilogue_bf16(y, None, res, 0)
        d = np.abs(oracle.bf16_to_f32(got[i]) - oracle.bf16_to_f32(ref))
        assert d.max() <= np.abs(oracle.bf16_to_f32(ref)).max() * 2.0**-7, (i, d.max())


@pytest.mark.parametrize("bits", [4, 8])
def test_gemv_weights_immutable_prefetch_still_waits_for_inputs(oracle, bits):
    """With qmm_set_weights_immutable(1) the GEMV streams its weights before
    the dependency wait; x, the residual and y are still ordered after the
    kernel before it.  Back-to-back launches over different (unchanging)
    weights, with x rewritten by a kernel before each and each residual the
    previous output, also as one CUDA graph."""
    import torch

    lib = _lib.load()
    k, n, m, layers = 3072, 4096, 1, 6
    lins, data = [], []
    for i in range(layers):
        packed, scales, offsets, bias = random_layer(n, k, bits, 64, seed=90 + i)
        lins.append(make_linear(packed, scales, offsets, bias, bits, 64))
        x = oracle.f32_to_bf16(np.sin(np.arange(k, dtype=np.float64) * (0.05 + 0.03 * i)).astype(np.float32)
                               .reshape(m, k))
        data.append((packed, scales, offsets, bias, x))
    xs = [to_dev_u16(d[4]) for d in data]
    xbuf = torch.empty((m, k), dtype=torch.bfloat16, device="cuda")
    residual0 = oracle.f32_to_bf16(np.linspace(-1.0, 1.0, m * n, dtype=np.float32).reshape(m, n))
    r0 = to_dev_u16(residual0)
    outs = [torch.empty((m, n), dtype=torch.bfloat16, device="cuda") for _ in range(layers)]

    def chain():
        prev = r0
        for i, lin in enumerate(lins):
            torch.mul(xs[i], 1.0, out=xbuf)
            lin.forward_fused(xbuf, residual=prev, out=outs[i], path=_lib.QMM_PATH_GEMV)
            prev = outs[i]

    def check():
        got = [from_dev(t) for t in outs]
        for i, (packed, scales, offsets, bias, x) in enumerate(data):
            res = residual0 if i == 0 else got[i - 1]
            ref = oracle.epilogue_bf16(oracle.linear_f32(x, packed, scales, offsets, bits, 64, bias), None, res, 0)
            d = np.abs(oracle.bf16_to_f32(got[i]) - oracle.bf16_to_f32(ref))
            assert d.max() <= np.abs(oracle.bf16_to_f32(ref)).max() * 2.0**-7, (i, d.max())

    prev_mode = lib.qmm_set_weights_immutable(1)
    try:
        chain()
        torch.cuda.synchronize()
        check()
        for t in outs:
            t.zero_()
        cap = torch.cuda.Stream()
        with torch.cuda.stream(cap):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cap):
                chain()
        torch.cuda.synchronize()
        for t in outs:
            t.zero_()
        g.replay()
        torch.cuda.synchronize()
        check()
        del g
    finally:
        lib.qmm_set_weights_immutable(prev_mode)


def to_dev_u32_i32(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a).view(np.int32)).cuda()


def from_dev(t):
    import torch

    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)
