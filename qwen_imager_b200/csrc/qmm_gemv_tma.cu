// Streaming GEMV for small m (the adaLN modulation linear runs at m = 1).
//
// HBM-bound: every packed byte is read once.  One persistent CTA per SM.  A
// producer warp streams contiguous blocks of RB weight rows (codes only; a
// row block is one contiguous range of the packed tensor) into a ring of
// shared-memory stages with cp.async.bulk; 16 consumer warps dot the rows
// against x, which each CTA stages once, as f32, in a bank-padded layout.
// A row is handled by WPR = 16 / RB warps; lane l of a warp takes 16-byte
// chunks l, l + 32 WPR, ... of its share and reduces with shuffles (and
// shared memory when WPR > 1).  Scales and offsets are read by the consumer
// lanes themselves, prefetched one row block ahead.
//
// Arithmetic per chunk (all codes of a chunk share one group):
//   sum_k x_k (s q_k + o) = s * sum_k x_k q_k + o * sum_k x_k,
// with the per-chunk sums of x precomputed at staging.  4-bit codes are
// expanded to the float 2 + q/64 by one byte permute (see chunk_dot).
// Reference computation: image-forger src/quant.rs:105-113 (f32 weights, f32
// accumulation), here with the weights never materialized.
#include <algorithm>

#include "qmm_epilogue.cuh"
#include "qmm_internal.h"
#include "qmm_unpack.cuh"

namespace qmm {
namespace gemv {

constexpr int kConsumerWarps = 16;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kMaxChunksPerLane = 8;
constexpr int kMaxStages = 4;
constexpr size_t kSmemLimit = 227 * 1024;

template <int MT>
struct Pad {
    static constexpr int kMP = MT == 1 ? 1 : (MT + 3) / 4 * 4;  // token slots per code
};

struct Params {
    const uint16_t *x;
    const uint32_t *packed;
    const uint16_t *scales;
    const uint16_t *offsets;
    uint16_t *y;
    EpilogueArgs ep;
    int64_t n;
    int32_t k, m, groups, cpg_shift;
    int32_t rb, wpr, stages;     // rows per stage, warps per row, ring depth
    int32_t row_bytes, nblocks;  // bytes per packed row, row blocks
    int32_t xs_floats;           // floats of the staged x (padded)
    uint32_t *err;
};

template <int I>
__device__ __forceinline__ float two_plus_q_over_64(uint32_t v) {
    // bytes [0x00, 0x00, v.b[I], 0x40] = 2 * (1 + q * 2^-7)
    return __uint_as_float(__byte_perm(v, 0x40000000u, 0x7044u | (I << 8)));
}

// S_t = sum over the chunk's codes of x[t][k] * f(q_k).  4-bit: f = 2 + q/64,
// so sum x q = 64 S - 128 X; 2- and 8-bit: f = q exactly.
template <int BITS, int MT>
__device__ __forceinline__ void chunk_dot(const uint4 &w, const float *__restrict__ xc, float (&dot)[MT]) {
    constexpr int CPW = 32 / BITS;
    constexpr int MP = Pad<MT>::kMP;
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int wi = 0; wi < 4; ++wi) {
        float q[CPW];
        if constexpr (BITS == 4) {
            const uint32_t lo = words[wi] & 0x0F0F0F0Fu, hi = (words[wi] >> 4) & 0x0F0F0F0Fu;
            q[0] = two_plus_q_over_64<0>(lo);
            q[1] = two_plus_q_over_64<0>(hi);
            q[2] = two_plus_q_over_64<1>(lo);
            q[3] = two_plus_q_over_64<1>(hi);
            q[4] = two_plus_q_over_64<2>(lo);
            q[5] = two_plus_q_over_64<2>(hi);
            q[6] = two_plus_q_over_64<3>(lo);
            q[7] = two_plus_q_over_64<3>(hi);
        } else {
            WordCodes<BITS>::unpack(words[wi], q);
        }
        if constexpr (MT == 1) {
            // Two f32x2 accumulators (even / odd code pairs) per chunk.
            float2 d0 = make_float2(0.0f, 0.0f), d1 = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int j = 0; j < CPW; j += 4) {
                const float4 xv = *reinterpret_cast<const float4 *>(xc + wi * CPW + j);
                d0 = fma_f32x2(make_float2(xv.x, xv.y), make_float2(q[j], q[j + 1]), d0);
                d1 = fma_f32x2(make_float2(xv.z, xv.w), make_float2(q[j + 2], q[j + 3]), d1);
            }
            dot[0] += (d0.x + d0.y) + (d1.x + d1.y);
        } else {
#pragma unroll
            for (int j = 0; j < CPW; ++j) {
                const float *xk = xc + (wi * CPW + j) * MP;
#pragma unroll
                for (int t = 0; t < MT; t += 4) {
                    const float4 xv = *reinterpret_cast<const float4 *>(xk + t);
                    dot[t] = fmaf(xv.x, q[j], dot[t]);
                    if (t + 1 < MT) dot[t + 1] = fmaf(xv.y, q[j], dot[t + 1]);
                    if (t + 2 < MT) dot[t + 2] = fmaf(xv.z, q[j], dot[t + 2]);
                    if (t + 3 < MT) dot[t + 3] = fmaf(xv.w, q[j], dot[t + 3]);
                }
            }
        }
    }
}

// Shared memory (16-byte aligned regions):
//   stages  [stages][rb * row_bytes]      packed rows
//   xs      [nchunks][CPC * MP + 4] f32   x, one padded record per chunk
//   xsum    [nchunks][MT] f32             per-chunk sums of x
//   part    [2][16][MT] f32               cross-warp partial sums
//   bars    full[stages], empty[stages]
// NCL > 0: every lane owns exactly NCL chunks of its row share (the loops
// below are fully unrolled with no guards); NCL == 0: generic, up to
// kMaxChunksPerLane chunks with guards.
template <int BITS, int MT, int NCL>
__global__ void __launch_bounds__(kThreads, 1) qmm_gemv_tma_kernel(const Params p) {
    constexpr int CPC = 128 / BITS;
    constexpr int MP = Pad<MT>::kMP;
    constexpr int XREC = CPC * MP + 4;
    constexpr float kMul = BITS == 4 ? 64.0f : 1.0f;
    constexpr float kAdd = BITS == 4 ? -128.0f : 0.0f;
    extern __shared__ __align__(1024) uint8_t smem[];
    const int nchunks = p.row_bytes / 16;
    const size_t stage_bytes = (size_t)p.rb * p.row_bytes;
    uint8_t *stages = smem;
    float *xs = reinterpret_cast<float *>(smem + p.stages * stage_bytes);
    float *xsum = xs + p.xs_floats;
    float *part = xsum + (size_t)nchunks * MT;
    uint64_t *full = reinterpret_cast<uint64_t *>(part + 2 * kConsumerWarps * MT + 2);
    full = reinterpret_cast<uint64_t *>((reinterpret_cast<uintptr_t>(full) + 7) & ~uintptr_t(7));
    uint64_t *empty = full + kMaxStages;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        // ---------------------------------------------------------- producer
        if (lane == 0) {
            const uint8_t *src = reinterpret_cast<const uint8_t *>(p.packed);
            int j = 0;
            for (int b = blockIdx.x; b < p.nblocks; b += gridDim.x, ++j) {
                const int s = j % p.stages;
                if (!mbar_wait(&empty[s], ((j / p.stages) & 1) ^ 1, p.err, kErrTimeoutProducer)) break;
                const int64_t row0 = (int64_t)b * p.rb;
                const int rows = (int)std::min<int64_t>(p.rb, p.n - row0);
                const uint32_t bytes = (uint32_t)rows * (uint32_t)p.row_bytes;
                mbar_arrive_expect_tx(&full[s], bytes);
                bulk_load(stages + s * stage_bytes, src + row0 * p.row_bytes, bytes, &full[s]);
            }
        }
        __syncwarp();
        return;  // consumers never wait on the producer warp's exit
    }

    // Stage x as f32 (tokens >= m are zero), 8 bf16 per load; chunk c's record
    // starts at c * XREC floats, code j of the chunk at j * MP + t.
    const int consumer_threads = kConsumerWarps * 32;
    for (int i = threadIdx.x; i < (p.k / 8) * MP; i += consumer_threads) {
        const int t = i % MP, k8 = (i / MP) * 8;
        float v[8];
        if (t < p.m) {
            const uint4 raw = __ldg(reinterpret_cast<const uint4 *>(p.x + (size_t)t * p.k + k8));
            const uint32_t r[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                v[2 * j] = __uint_as_float(r[j] << 16);
                v[2 * j + 1] = __uint_as_float(r[j] & 0xFFFF0000u);
            }
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = 0.0f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int kk = k8 + j, c = kk / CPC, jc = kk - c * CPC;
            xs[(size_t)c * XREC + jc * MP + t] = v[j];
        }
    }
    named_barrier(1, consumer_threads);
    for (int i = threadIdx.x; i < nchunks * MT; i += consumer_threads) {
        const int c = i / MT, t = i - c * MT;
        float sum = 0.0f;
        for (int j = 0; j < CPC; ++j) sum += xs[(size_t)c * XREC + j * MP + t];
        xsum[i] = sum;
    }
    named_barrier(1, consumer_threads);

    // ---------------------------------------------------------- consumers
    const int wpr = p.wpr;
    const int rloc = warp / wpr;      // row within the block
    const int share = warp - rloc * wpr;
    const int stride = 32 * wpr;      // chunk stride between a lane's chunks
    constexpr int kCL = NCL > 0 ? NCL : kMaxChunksPerLane;
    const int nloc = NCL > 0 ? NCL : (nchunks - share * 32 - lane + stride - 1) / stride;  // chunks of this lane
    float sc[kCL], of[kCL];
    auto load_meta = [&](int b) {
        const int64_t n = (int64_t)b * p.rb + rloc;
        const bool ok = b < p.nblocks && n < p.n;
#pragma unroll
        for (int u = 0; u < kCL; ++u) {
            const int c = share * 32 + lane + u * stride;
            sc[u] = of[u] = 0.0f;
            if (ok && (NCL > 0 || u < nloc)) {
                const int64_t g = n * p.groups + (c >> p.cpg_shift);
                sc[u] = bf16_bits_to_f32(__ldg(p.scales + g));
                of[u] = bf16_bits_to_f32(__ldg(p.offsets + g));
            }
        }
    };
    load_meta(blockIdx.x);
    // A failed (timed-out) wait does not leave the loop: every consumer warp
    // keeps taking the same named barriers, skipping the work, so that no warp
    // waits at a barrier for one that left.
    bool ok = true;
    int j = 0;
    for (int b = blockIdx.x; b < p.nblocks; b += gridDim.x, ++j) {
        const int s = j % p.stages;
        float csc[kCL], cof[kCL];
#pragma unroll
        for (int u = 0; u < kCL; ++u) {
            csc[u] = sc[u];
            cof[u] = of[u];
        }
        load_meta(b + gridDim.x);  // next block's scales, in flight while this one computes
        ok = ok && mbar_wait(&full[s], (j / p.stages) & 1, p.err, kErrTimeoutDequant);
        const int64_t row0 = (int64_t)b * p.rb;
        const int64_t n = row0 + rloc;
        float acc[MT];
#pragma unroll
        for (int t = 0; t < MT; ++t) acc[t] = 0.0f;
        if (ok && n < p.n) {
            const uint8_t *rowp = stages + s * stage_bytes + (size_t)rloc * p.row_bytes;
#pragma unroll
            for (int u = 0; u < kCL; ++u) {
                if (NCL > 0 || u < nloc) {
                    const int c = share * 32 + lane + u * stride;
                    const uint4 w4 = *reinterpret_cast<const uint4 *>(rowp + (size_t)c * 16);
                    float dot[MT];
#pragma unroll
                    for (int t = 0; t < MT; ++t) dot[t] = 0.0f;
                    chunk_dot<BITS, MT>(w4, xs + (size_t)c * XREC, dot);
                    const float a = csc[u] * kMul;
                    const float bb = fmaf(csc[u], kAdd, cof[u]);
#pragma unroll
                    for (int t = 0; t < MT; ++t) acc[t] = fmaf(a, dot[t], fmaf(bb, xsum[(size_t)c * MT + t], acc[t]));
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);  // this warp is done reading the stage
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            float v = acc[t];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
            acc[t] = v;
        }
        if (wpr > 1) {
            float *pb = part + (j & 1) * kConsumerWarps * MT;
            if (lane == 0) {
#pragma unroll
                for (int t = 0; t < MT; ++t) pb[warp * MT + t] = acc[t];
            }
            named_barrier(1, consumer_threads);
            if (share == 0) {
#pragma unroll
                for (int t = 0; t < MT; ++t) {
                    float v = 0.0f;
                    for (int q = 0; q < wpr; ++q) v += pb[(warp + q) * MT + t];
                    acc[t] = v;
                }
            }
        }
        if (ok && share == 0 && n < p.n) {
            const FeatureConsts fc = load_feature_consts(p.ep, n, true);
#pragma unroll
            for (int t = 0; t < MT; ++t) {
                if (lane == t && t < p.m) {
                    const int64_t idx = (int64_t)t * p.n + n;
                    const float v = epilogue_value(p.ep, fc, acc[t], p.ep.residual ? p.ep.residual + idx : nullptr);
                    p.y[idx] = f32_to_bf16_bits(v);
                }
            }
        }
    }
}

struct Plan {
    int rb, wpr, stages, xs_floats, ncl;  // ncl > 0: exact chunks per lane
    size_t smem;
};

template <int MT>
static bool plan_for(const qmm_weight &w, int64_t m, Plan &pl) {
    const int cpc = 128 / w.bits;
    const int mp = Pad<MT>::kMP;
    const int64_t row_bytes = w.k * w.bits / 8;
    const int64_t nchunks = row_bytes / 16;
    int rb = 16;
    while (rb > 1 && rb * row_bytes > 48 * 1024) rb >>= 1;
    int wpr = kConsumerWarps / rb;
    if ((nchunks + 32 * wpr - 1) / (32 * wpr) > kMaxChunksPerLane) return false;
    pl.ncl = 0;
    if (MT == 1) {
        // Prefer a split where every lane owns the same number of chunks.
        for (int w2 = wpr; w2 <= kConsumerWarps; w2 *= 2) {
            const int64_t per = 32 * (int64_t)w2;
            const int64_t ncl = nchunks / per;
            if (nchunks % per == 0 && (ncl == 1 || ncl == 2 || ncl == 3 || ncl == 4 || ncl == 6 || ncl == 8)) {
                wpr = w2;
                rb = kConsumerWarps / w2;
                pl.ncl = (int)ncl;
                break;
            }
        }
    }
    pl.rb = rb;
    pl.wpr = wpr;
    pl.xs_floats = (int)(nchunks * (cpc * mp + 4));
    const size_t fixed = (size_t)pl.xs_floats * 4 + (size_t)nchunks * MT * 4 + 2 * kConsumerWarps * MT * 4 + 16 +
                         2 * kMaxStages * 8 + 64;
    const size_t stage = (size_t)rb * row_bytes;
    int stages = kMaxStages;
    while (stages >= 2 && fixed + stages * stage > kSmemLimit) --stages;
    if (stages < 2) return false;
    pl.stages = stages;
    pl.smem = fixed + stages * stage;
    (void)m;
    return true;
}

template <int BITS, int MT, int NCL>
static qmm_status launch_k(const Params &p, const Plan &pl, cudaStream_t st) {
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(qmm_gemv_tma_kernel<BITS, MT, NCL>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemLimit);
        if (e != cudaSuccess) return cuda_fail(e, "gemv smem attribute");
        configured[dev] = true;
    }
    const int grid = (int)std::min<int64_t>(p.nblocks, sm_count());
    qmm_gemv_tma_kernel<BITS, MT, NCL><<<grid, kThreads, pl.smem, st>>>(p);
    count_launch();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? QMM_OK : cuda_fail(e, "gemv launch");
}

template <int BITS, int MT>
static qmm_status launch_t(const qmm_weight &w, const uint16_t *x, int64_t m, const qmm_epilogue &ep,
                           uint16_t *y, cudaStream_t st) {
    Plan pl;
    if (!plan_for<MT>(w, m, pl)) return fail(QMM_ERR_UNSUPPORTED, "gemv: layout does not fit shared memory");
    Params p;
    p.x = x;
    p.packed = w.packed;
    p.scales = w.scales;
    p.offsets = w.biases;
    p.y = y;
    p.ep = epilogue_args(ep);
    p.n = w.n;
    p.k = (int32_t)w.k;
    p.m = (int32_t)m;
    p.groups = (int32_t)(w.k / w.group);
    int cps = 0;
    while ((1 << cps) < w.group / (128 / BITS)) ++cps;
    p.cpg_shift = cps;
    p.rb = pl.rb;
    p.wpr = pl.wpr;
    p.stages = pl.stages;
    p.row_bytes = (int32_t)(w.k * BITS / 8);
    p.nblocks = (int32_t)((w.n + pl.rb - 1) / pl.rb);
    p.xs_floats = pl.xs_floats;
    p.err = device_error_word();
    if constexpr (MT == 1) {
        switch (pl.ncl) {
            case 1: return launch_k<BITS, 1, 1>(p, pl, st);
            case 2: return launch_k<BITS, 1, 2>(p, pl, st);
            case 3: return launch_k<BITS, 1, 3>(p, pl, st);
            case 4: return launch_k<BITS, 1, 4>(p, pl, st);
            case 6: return launch_k<BITS, 1, 6>(p, pl, st);
            case 8: return launch_k<BITS, 1, 8>(p, pl, st);
            default: break;
        }
    }
    return launch_k<BITS, MT, 0>(p, pl, st);
}

static int tile_for(int64_t m) {
    if (m <= 1) return 1;
    if (m <= 2) return 2;
    if (m <= 4) return 4;
    if (m <= 8) return 8;
    return 16;
}

}  // namespace gemv

bool gemv_tma_supported(const qmm_weight &w, int64_t m) {
    if (m < 1 || m > 16) return false;
    if (w.bits != 2 && w.bits != 4 && w.bits != 8) return false;
    const int cpc = 128 / w.bits;
    if (w.k % cpc != 0 || w.group % cpc != 0) return false;
    if (((w.group / cpc) & (w.group / cpc - 1)) != 0) return false;
    if (w.k > (1 << 24) || w.n > ((int64_t)1 << 31)) return false;
    gemv::Plan pl;
    switch (gemv::tile_for(m)) {
        case 1: return gemv::plan_for<1>(w, m, pl);
        case 2: return gemv::plan_for<2>(w, m, pl);
        case 4: return gemv::plan_for<4>(w, m, pl);
        case 8: return gemv::plan_for<8>(w, m, pl);
        default: return gemv::plan_for<16>(w, m, pl);
    }
}

qmm_status launch_gemv_tma(const qmm_weight &w, const uint16_t *x, int64_t m, const qmm_epilogue &ep,
                           uint16_t *y, cudaStream_t st) {
    const int mt = gemv::tile_for(m);
#define QMM_GT_CASE(B, MT) \
    if (w.bits == B && mt == MT) return gemv::launch_t<B, MT>(w, x, m, ep, y, st);
#define QMM_GT_BITS(B) QMM_GT_CASE(B, 1) QMM_GT_CASE(B, 2) QMM_GT_CASE(B, 4) QMM_GT_CASE(B, 8) QMM_GT_CASE(B, 16)
    QMM_GT_BITS(2)
    QMM_GT_BITS(4)
    QMM_GT_BITS(8)
#undef QMM_GT_BITS
#undef QMM_GT_CASE
    return fail(QMM_ERR_UNSUPPORTED, "gemv: no kernel for %d-bit, m=%lld", w.bits, (long long)m);
}

}  // namespace qmm
