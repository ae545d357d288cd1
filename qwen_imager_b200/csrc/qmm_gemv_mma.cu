// Tensor-core GEMV for 4-bit weights and m <= 16 tokens (the adaLN
// modulation linear runs at m = 1).
//
// HBM-bound: every packed byte is read once, so the kernel's job is to keep
// the copy engine busy and spend as few instructions per code as possible.
// One persistent CTA per SM.  A producer warp streams blocks of RB weight
// rows (codes with one bulk copy per row into a bank-staggered row stride,
// plus the block's scales and offsets) into a ring of shared-memory stages.
// Sixteen consumer warps split a block into 16-row tiles x K slices.
//
// Arithmetic.  Per 64-code unit u of a row (inside one quantization group),
//   sum_k x_k (s q_k + o) = s * D_u + (o - 128 s) * X_u,
// where D_u = sum_k x_k (128 + q_k) and X_u = sum_k x_k.  A 4-bit code q
// becomes the exact bf16 value 128 + q with one byte permute per two codes
// (bytes [q, 0x43] are the bf16 bit pattern of 128 + q for q < 128), and D_u
// is four m16n8k16 bf16 MMAs with f32 accumulation: A = 16 weight rows x 16
// codes, B = 16 codes x 8 tokens.  A dot product is invariant under a common
// permutation of its K index, so the codes are fed to the MMA in the order
// they sit in the packed words and x is staged once, in shared memory, in the
// matching order:  lane (g, t) of a warp holds words 2t and 2t+1 of the unit
// for rows g and g+8; MMA j takes word j/2, low nibbles (codes 0,2 | 4,6) for
// even j, high nibbles (codes 1,3 | 5,7) for odd j.  About one instruction
// per code instead of a multiply-add per code on the FMA pipe.
//
// Reference computation: image-forger src/quant.rs:105-113 (weights
// dequantized to f32 as scale * q + offset, f32 accumulation); the products
// x * (128 + q) are exact in f32.  Every wait is bounded (qmm_common.cuh).
#include <algorithm>

#include "qmm_epilogue.cuh"
#include "qmm_internal.h"

namespace qmm {
namespace gemvtc {

constexpr int kConsumerWarps = 16;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kMaxStages = 4;
constexpr size_t kSmemLimit = 227 * 1024;
constexpr int kUnit = 64;  // codes per four-MMA unit

struct Params {
    const uint16_t *x;
    const uint8_t *packed;
    const uint16_t *scales;
    const uint16_t *offsets;
    uint16_t *y;
    EpilogueArgs ep;
    int64_t n;
    int32_t k, m, groups, units, unit_shift;  // unit u lies in group u >> unit_shift
    int32_t rb, ks, upw, stages;              // rows per block, K slices, units per slice, ring depth
    int32_t row_bytes, row_stride, nblocks;
    int32_t stage_bytes, meta_off;            // scales at meta_off, offsets after them
    int32_t xp_stride;                        // u32 words per staged token
    uint32_t *err;
};

__device__ __forceinline__ void mma_bf16_m16n8k16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                                  uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// bf16 pairs (128 + q_a, 128 + q_b) from bytes 0,1 (SEL 0x4140) or 2,3
// (SEL 0x4342) of a word of nibble-wide codes.
template <uint32_t SEL>
__device__ __forceinline__ uint32_t code_pair(uint32_t nibbles) {
    return __byte_perm(nibbles, 0x43434343u, SEL);
}

// Shared memory (16-byte aligned regions):
//   stages [stages][rb * row_stride codes | rb*groups scales | rb*groups offsets]
//   xp     [m][units][4 lanes t][4 MMAs j][2] u32   x in MMA order, bf16 pairs
//   xsum   [units][MP] f32                            X_u per token (zero beyond m)
//   part   [2][ks][rb][m] f32                         partial sums per K slice
//   bars   full[kMaxStages], empty[kMaxStages]
template <int MT>
__global__ void __launch_bounds__(kThreads, 1) qmm_gemv_mma_kernel(const Params p) {
    constexpr int MP = 8 * MT;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t *stages = smem;
    uint32_t *xp = reinterpret_cast<uint32_t *>(smem + (size_t)p.stages * p.stage_bytes);
    float *xsum = reinterpret_cast<float *>(xp + (size_t)p.m * p.xp_stride);
    float *part = xsum + (size_t)p.units * MP;
    uint64_t *full = reinterpret_cast<uint64_t *>(
        (reinterpret_cast<uintptr_t>(part + 2 * (size_t)p.ks * p.rb * p.m) + 15) & ~uintptr_t(15));
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
        int j = 0;
        for (int b = blockIdx.x; b < p.nblocks; b += gridDim.x, ++j) {
            const int s = j % p.stages;
            int okp = 1;
            if (lane == 0) okp = mbar_wait(&empty[s], ((j / p.stages) & 1) ^ 1, p.err, kErrTimeoutProducer);
            if (!__shfl_sync(0xffffffffu, okp, 0)) break;
            const int64_t row0 = (int64_t)b * p.rb;
            const int rows = (int)(p.n - row0 < p.rb ? p.n - row0 : p.rb);
            const uint32_t meta = (uint32_t)rows * (uint32_t)p.groups * 2u;
            if (lane == 0) mbar_arrive_expect_tx(&full[s], (uint32_t)rows * (uint32_t)p.row_bytes + 2u * meta);
            __syncwarp();
            uint8_t *st = stages + (size_t)s * p.stage_bytes;
            for (int r = lane; r < rows; r += 32)
                bulk_load(st + (size_t)r * p.row_stride, p.packed + (row0 + r) * p.row_bytes,
                          (uint32_t)p.row_bytes, &full[s]);
            if (lane == 0) bulk_load(st + p.meta_off, p.scales + row0 * p.groups, meta, &full[s]);
            if (lane == 1)
                bulk_load(st + p.meta_off + (size_t)p.rb * p.groups * 2, p.offsets + row0 * p.groups, meta,
                          &full[s]);
        }
        return;  // consumers never wait on the producer warp's exit
    }

    // ------------------------------------------------- stage x in MMA order
    // Entry (token, u, t, j, r) holds x at codes c0 = 64u + 16t + 8(j/2) +
    // (j%2) + 4r and c0 + 2 of the token (low half c0).
    const int consumer_threads = kConsumerWarps * 32;
    const int per_token = p.units * 32;
    for (int i = threadIdx.x; i < p.m * per_token; i += consumer_threads) {
        const int tok = i / per_token, e = i - tok * per_token;
        const int u = e >> 5, t = (e >> 3) & 3, jj = (e >> 1) & 3, r = e & 1;
        const int c0 = u * kUnit + 16 * t + 8 * (jj >> 1) + (jj & 1) + 4 * r;
        const uint16_t *xt = p.x + (size_t)tok * p.k;
        xp[(size_t)tok * p.xp_stride + e] = (uint32_t)__ldg(xt + c0) | ((uint32_t)__ldg(xt + c0 + 2) << 16);
    }
    // X_u: eight lanes per (unit, token), 8 codes each, reduced with shuffles.
    for (int i = threadIdx.x; i < p.units * MP * 8; i += consumer_threads) {
        const int c = i & 7, ut = i >> 3;
        const int u = ut / MP, tok = ut - u * MP;
        float sum = 0.0f;
        if (tok < p.m) {
            const uint4 raw = __ldg(reinterpret_cast<const uint4 *>(p.x + (size_t)tok * p.k + u * kUnit) + c);
            const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) sum += __uint_as_float(w[q] << 16) + __uint_as_float(w[q] & 0xFFFF0000u);
        }
        // units * MP * 8 and the stride are multiples of 32: a warp's lanes
        // are all in the loop or all out of it, so the full-mask shuffles are safe.
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        sum += __shfl_xor_sync(0xffffffffu, sum, 4);
        if (c == 0) xsum[ut] = sum;
    }
    named_barrier(1, consumer_threads);

    // ---------------------------------------------------------- consumers
    const int g = lane >> 2, t = lane & 3;
    const int rt = warp / p.ks, ksl = warp - rt * p.ks;
    const int row_a = rt * 16 + g, row_b = row_a + 8;
    const int u0 = ksl * p.upw, u1 = min(p.units, u0 + p.upw);
    // B fragments: lanes whose token (g, plus 8 per token tile) is >= m use zeros.
    const uint32_t *xb[MT];
    bool has_tok[MT];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
        has_tok[mt] = mt * 8 + g < p.m;
        xb[mt] = xp + (size_t)(has_tok[mt] ? mt * 8 + g : 0) * p.xp_stride + t * 8;
    }
    bool ok = true;
    int j = 0;
    for (int b = blockIdx.x; b < p.nblocks; b += gridDim.x, ++j) {
        const int s = j % p.stages;
        ok = ok && mbar_wait(&full[s], (j / p.stages) & 1, p.err, kErrTimeoutDequant);
        const uint8_t *st = stages + (size_t)s * p.stage_bytes;
        const uint16_t *ssc = reinterpret_cast<const uint16_t *>(st + p.meta_off);
        const uint16_t *sof = ssc + (size_t)p.rb * p.groups;
        float acc[MT][4];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[mt][q] = 0.0f;
        if (ok) {
            const uint8_t *ra = st + (size_t)row_a * p.row_stride + t * 8;
            const uint8_t *rbp = st + (size_t)row_b * p.row_stride + t * 8;
#pragma unroll 2
            for (int u = u0; u < u1; ++u) {
                const uint2 wa = *reinterpret_cast<const uint2 *>(ra + u * 32);
                const uint2 wb = *reinterpret_cast<const uint2 *>(rbp + u * 32);
                uint32_t bfr[MT][8];
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    if (has_tok[mt]) {
                        const uint4 v0 = *reinterpret_cast<const uint4 *>(xb[mt] + u * 32);
                        const uint4 v1 = *reinterpret_cast<const uint4 *>(xb[mt] + u * 32 + 4);
                        bfr[mt][0] = v0.x; bfr[mt][1] = v0.y; bfr[mt][2] = v0.z; bfr[mt][3] = v0.w;
                        bfr[mt][4] = v1.x; bfr[mt][5] = v1.y; bfr[mt][6] = v1.z; bfr[mt][7] = v1.w;
                    } else {
#pragma unroll
                        for (int q = 0; q < 8; ++q) bfr[mt][q] = 0u;
                    }
                }
                // Two independent accumulator chains (low- and high-nibble MMAs).
                float d[MT][4], e[MT][4];
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int q = 0; q < 4; ++q) d[mt][q] = e[mt][q] = 0.0f;
                const uint32_t wa_[2] = {wa.x, wa.y}, wb_[2] = {wb.x, wb.y};
#pragma unroll
                for (int h = 0; h < 2; ++h) {  // word 2t + h of the unit
                    const uint32_t la = wa_[h] & 0x0F0F0F0Fu, ha = (wa_[h] >> 4) & 0x0F0F0F0Fu;
                    const uint32_t lb = wb_[h] & 0x0F0F0F0Fu, hb = (wb_[h] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) {
                        // MMA 2h: low nibbles; MMA 2h + 1: high nibbles.
                        mma_bf16_m16n8k16(d[mt], code_pair<0x4140>(la), code_pair<0x4140>(lb),
                                          code_pair<0x4342>(la), code_pair<0x4342>(lb), bfr[mt][4 * h + 0],
                                          bfr[mt][4 * h + 1]);
                        mma_bf16_m16n8k16(e[mt], code_pair<0x4140>(ha), code_pair<0x4140>(hb),
                                          code_pair<0x4342>(ha), code_pair<0x4342>(hb), bfr[mt][4 * h + 2],
                                          bfr[mt][4 * h + 3]);
                    }
                }
                const int gi = u >> p.unit_shift;
                const float sa = bf16_bits_to_f32(ssc[row_a * p.groups + gi]);
                const float sb = bf16_bits_to_f32(ssc[row_b * p.groups + gi]);
                const float ca = fmaf(-128.0f, sa, bf16_bits_to_f32(sof[row_a * p.groups + gi]));
                const float cb = fmaf(-128.0f, sb, bf16_bits_to_f32(sof[row_b * p.groups + gi]));
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) d[mt][q] += e[mt][q];
                    const float2 xs2 = *reinterpret_cast<const float2 *>(xsum + u * MP + mt * 8 + 2 * t);
                    acc[mt][0] = fmaf(sa, d[mt][0], fmaf(ca, xs2.x, acc[mt][0]));
                    acc[mt][1] = fmaf(sa, d[mt][1], fmaf(ca, xs2.y, acc[mt][1]));
                    acc[mt][2] = fmaf(sb, d[mt][2], fmaf(cb, xs2.x, acc[mt][2]));
                    acc[mt][3] = fmaf(sb, d[mt][3], fmaf(cb, xs2.y, acc[mt][3]));
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);  // this warp is done reading the stage
        // Partial sums of this K slice: rows row_a, row_b; tokens mt*8 + 2t, +1.
        float *pb = part + ((size_t)(j & 1) * p.ks + ksl) * p.rb * p.m;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            const int t0 = mt * 8 + 2 * t;
            if (t0 < p.m) {
                pb[row_a * p.m + t0] = acc[mt][0];
                pb[row_b * p.m + t0] = acc[mt][2];
            }
            if (t0 + 1 < p.m) {
                pb[row_a * p.m + t0 + 1] = acc[mt][1];
                pb[row_b * p.m + t0 + 1] = acc[mt][3];
            }
        }
        named_barrier(1, consumer_threads);
        // Reduce over K slices, epilogue, store.  (The next block writes the
        // other half of `part`; the barrier of the block after that orders
        // these reads before its writes.)
        const int64_t row0 = (int64_t)b * p.rb;
        const float *pr = part + (size_t)(j & 1) * p.ks * p.rb * p.m;
        for (int i = threadIdx.x; i < p.rb * p.m; i += consumer_threads) {
            const int row = i / p.m, tok = i - row * p.m;
            const int64_t n = row0 + row;
            if (!ok || n >= p.n) continue;
            float v = 0.0f;
            for (int q = 0; q < p.ks; ++q) v += pr[(size_t)q * p.rb * p.m + i];
            const FeatureConsts fc = load_feature_consts(p.ep, n, true);
            const int64_t idx = (int64_t)tok * p.n + n;
            p.y[idx] = f32_to_bf16_bits(epilogue_value(p.ep, fc, v, p.ep.residual ? p.ep.residual + idx : nullptr));
        }
    }
}

struct Plan {
    int rb, ks, stages, row_stride, stage_bytes, meta_off, xp_stride;
    size_t smem;
};

static bool plan_for(const qmm_weight &w, int64_t m, Plan &pl) {
    const int mt = m <= 8 ? 1 : 2;
    const int64_t units = w.k / kUnit, groups = w.k / w.group;
    const int64_t row_bytes = w.k / 2;
    // Row stride = 32 or 96 (mod 128) bytes: the 16 lanes of an 8-byte load
    // phase (rows g = 0..3 of a tile) then hit disjoint banks.
    const int64_t r128 = row_bytes % 128;
    pl.row_stride = (int)(r128 == 32 || r128 == 96 ? row_bytes : row_bytes + 32);
    pl.xp_stride = (int)(units * 32 + 4);  // +16 bytes: tokens start in different bank quads
    const size_t xs = (size_t)m * pl.xp_stride * 4 + (size_t)units * 8 * mt * 4;
    for (int rb = 32; rb >= 16; rb /= 2) {
        const int ks = kConsumerWarps / (rb / 16);
        const int64_t meta = (int64_t)rb * groups * 2;
        const int64_t stage = (int64_t)rb * pl.row_stride + 2 * meta;
        const size_t fixed = xs + 2 * (size_t)ks * rb * m * 4 + 16 + 2 * kMaxStages * 8 + 64;
        int stages = kMaxStages;
        while (stages >= 2 && fixed + (size_t)stages * stage > kSmemLimit) --stages;
        if (stages < 2) continue;
        pl.rb = rb;
        pl.ks = ks;
        pl.stages = stages;
        pl.stage_bytes = (int)stage;
        pl.meta_off = rb * pl.row_stride;
        pl.smem = fixed + (size_t)stages * stage;
        return true;
    }
    return false;
}

template <int MT>
static qmm_status launch_t(const qmm_weight &w, const uint16_t *x, int64_t m, const qmm_epilogue &ep,
                           uint16_t *y, cudaStream_t st) {
    Plan pl;
    if (!plan_for(w, m, pl)) return fail(QMM_ERR_UNSUPPORTED, "gemv (mma): layout does not fit shared memory");
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(qmm_gemv_mma_kernel<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)kSmemLimit);
        if (e != cudaSuccess) return cuda_fail(e, "gemv (mma) smem attribute");
        configured[dev] = true;
    }
    Params p;
    p.x = x;
    p.packed = reinterpret_cast<const uint8_t *>(w.packed);
    p.scales = w.scales;
    p.offsets = w.biases;
    p.y = y;
    p.ep = EpilogueArgs{ep.bias, ep.gate, ep.residual, ep.activation};
    p.n = w.n;
    p.k = (int32_t)w.k;
    p.m = (int32_t)m;
    p.groups = (int32_t)(w.k / w.group);
    p.units = (int32_t)(w.k / kUnit);
    int us = 0;
    while ((kUnit << us) < w.group) ++us;
    p.unit_shift = us;
    p.rb = pl.rb;
    p.ks = pl.ks;
    p.upw = (p.units + pl.ks - 1) / pl.ks;
    p.stages = pl.stages;
    p.row_bytes = (int32_t)(w.k / 2);
    p.row_stride = pl.row_stride;
    p.nblocks = (int32_t)((w.n + pl.rb - 1) / pl.rb);
    p.stage_bytes = pl.stage_bytes;
    p.meta_off = pl.meta_off;
    p.xp_stride = pl.xp_stride;
    p.err = device_error_word();
    const int grid = (int)std::min<int64_t>(p.nblocks, sm_count());
    qmm_gemv_mma_kernel<MT><<<grid, kThreads, pl.smem, st>>>(p);
    count_launch();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? QMM_OK : cuda_fail(e, "gemv (mma) launch");
}

}  // namespace gemvtc

bool gemv_mma_supported(const qmm_weight &w, int64_t m) {
    if (w.bits != 4 || m < 1 || m > 16) return false;
    if (w.k % gemvtc::kUnit != 0 || w.group % gemvtc::kUnit != 0) return false;
    const int per = w.group / gemvtc::kUnit;
    if ((per & (per - 1)) != 0) return false;
    if (w.n % 8 != 0 || w.k > (1 << 20) || w.n > ((int64_t)1 << 31)) return false;
    // Bulk copies of scale/offset blocks need 16-byte aligned sources.
    if ((reinterpret_cast<uintptr_t>(w.scales) | reinterpret_cast<uintptr_t>(w.biases)) & 15u) return false;
    gemvtc::Plan pl;
    return gemvtc::plan_for(w, m, pl);
}

qmm_status launch_gemv_mma(const qmm_weight &w, const uint16_t *x, int64_t m, const qmm_epilogue &ep,
                           uint16_t *y, cudaStream_t st) {
    return m <= 8 ? gemvtc::launch_t<1>(w, x, m, ep, y, st) : gemvtc::launch_t<2>(w, x, m, ep, y, st);
}

}  // namespace qmm
