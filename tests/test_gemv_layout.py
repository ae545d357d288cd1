"""The index arithmetic of the tensor-core GEMV (qwen_imager_b200/csrc/qmm_gemv_mma.cu), restated on the
CPU.

Each check mirrors a piece of the kernel:
- the quad shared-memory layout of a 32-row block;
- the lane-to-row mapping;
- the bf16 code pairs made by byte permutes;
- the K-permuted staging of x;
- the m16n8k16 fragment layouts.

Together they must reproduce sum_k x_k (s q_k + o) for every row and token. The 8-byte fragment loads of
each half-warp must also hit 16 distinct bank pairs. The GPU tests check the kernel itself; this pins the
layout reasoning the kernel's comments state.
"""
import numpy as np
import pytest


def bf16_pair(u32):
    lo = np.array([(u32 & 0xFFFF) << 16], dtype=np.uint32).view(np.float32)[0]
    hi = np.array([u32 & 0xFFFF0000], dtype=np.uint32).view(np.float32)[0]
    return float(lo), float(hi)


def byte_perm(a, b, sel):
    """CUDA __byte_perm: result byte i is byte (sel >> 4i) & 7 of the 8 bytes of (b:a)."""
    src = [(a >> (8 * i)) & 0xFF for i in range(4)] + [(b >> (8 * i)) & 0xFF for i in range(4)]
    return sum(src[(sel >> (4 * i)) & 7] << (8 * i) for i in range(4))


def code_pair(nibbles, sel):
    return byte_perm(nibbles, 0x43434343, sel)


def bf16_bits(v):
    return int(np.array([v], dtype=np.float32).view(np.uint32)[0] >> 16)  # exact for bf16-valued floats


def stage_entry(x_tok, u, t, e):
    """xp[tok][u * 32 + t * 8 + e]: x at codes c0 and c0 + 2 (low half c0)."""
    jj, r = e >> 1, e & 1
    c0 = 8 * (jj >> 1) + (jj & 1) + 4 * r
    base = 64 * u + 16 * t
    return bf16_bits(x_tok[base + c0]) | (bf16_bits(x_tok[base + c0 + 2]) << 16)


def block_row(tile, g, hr):
    """Block row read by lane group g for MMA row g (hr = 0) or g + 8 (hr = 1) of a 16-row tile."""
    return tile * 16 + 4 * (g & 3) + (g >> 2) + 2 * hr


@pytest.mark.parametrize("units,m", [(1, 1), (3, 1), (2, 5), (2, 8)])
def test_fragments_reproduce_the_affine_dot_product(units, m):
    rng = np.random.default_rng(units * 10 + m)
    k, rb = 64 * units, 32
    codes = rng.integers(0, 16, size=(rb, k))
    words = np.zeros((rb, k // 8), dtype=np.int64)
    for c in range(8):
        words |= codes[:, c::8].astype(np.int64) << (4 * c)
    s = rng.uniform(-0.01, 0.01, size=(rb, units))
    o = rng.uniform(-0.05, 0.05, size=(rb, units))
    # bf16-exact x, tokens >= m read the zero row
    x = np.zeros((8, k), dtype=np.float32)
    x[:m] = (rng.integers(-128, 128, size=(m, k)) / 64.0).astype(np.float32)
    xsum = x.reshape(8, units, 64).sum(axis=2)
    got = np.zeros((rb, 8))
    for tile in range(rb // 16):
        for u in range(units):
            d = np.zeros((16, 8))
            for j in range(4):
                h, hi = j // 2, j % 2
                A, B = np.zeros((16, 16)), np.zeros((16, 8))
                for lane in range(32):
                    g, t = lane >> 2, lane & 3
                    wa = int(words[block_row(tile, g, 0), 8 * u + 2 * t + h])
                    wb = int(words[block_row(tile, g, 1), 8 * u + 2 * t + h])
                    la, lb = (wa >> (4 * hi)) & 0x0F0F0F0F, (wb >> (4 * hi)) & 0x0F0F0F0F
                    A[g, 2 * t:2 * t + 2] = bf16_pair(code_pair(la, 0x4140))
                    A[g + 8, 2 * t:2 * t + 2] = bf16_pair(code_pair(lb, 0x4140))
                    A[g, 2 * t + 8:2 * t + 10] = bf16_pair(code_pair(la, 0x4342))
                    A[g + 8, 2 * t + 8:2 * t + 10] = bf16_pair(code_pair(lb, 0x4342))
                    B[2 * t:2 * t + 2, g] = bf16_pair(stage_entry(x[g], u, t, 4 * h + 2 * hi))
                    B[2 * t + 8:2 * t + 10, g] = bf16_pair(stage_entry(x[g], u, t, 4 * h + 2 * hi + 1))
                d += A @ B
            for mr in range(16):
                row = block_row(tile, mr & 7, mr >> 3)
                got[row] += s[row, u] * d[mr] + (o[row, u] - 128 * s[row, u]) * xsum[:, u]
    want = (s.repeat(64, axis=1) * codes + o.repeat(64, axis=1)) @ x.T.astype(np.float64)
    np.testing.assert_allclose(got[:, :m], want[:, :m], rtol=1e-9, atol=1e-12)


@pytest.mark.parametrize("row_bytes", [32, 64, 96, 512, 1536, 6144])
def test_quad_slots_keep_fragment_loads_conflict_free(row_bytes):
    quad_stride = 4 * row_bytes + 32
    for tile in range(2):
        for u in range(row_bytes // 32):
            for hr in range(2):
                for phase in range(2):  # an 8-byte warp load is served as two 16-lane phases
                    words = {}
                    for lane in range(16 * phase, 16 * phase + 16):
                        g, t = lane >> 2, lane & 3
                        row = block_row(tile, g, hr)
                        addr = (row // 4) * quad_stride + (row % 4) * row_bytes + 8 * t + 32 * u
                        for w in (addr // 4, addr // 4 + 1):
                            words.setdefault(w % 32, set()).add(w)
                    assert max(len(v) for v in words.values()) == 1


def test_every_block_row_is_read_once():
    rows = sorted(block_row(tile, g, hr) for tile in range(2) for g in range(8) for hr in range(2))
    assert rows == list(range(32))
