// Tensor-core GEMV for 4-bit weights and m <= 16 tokens (the adaLN
// modulation linear runs at m = 1).
//
// HBM-bound: every packed byte is read once, so the kernel's job is to keep
// the copy engine busy and spend as few instructions per code as possible.
// One persistent CTA per SM.  A producer warp streams blocks of RB weight
// rows into a ring of shared-memory stages: the codes with one bulk copy per
// quad of 4 consecutive rows (contiguous in memory) into quad slots 32 bytes
// longer than the quad, plus the block's scales and offsets.  Per-row copies
// (34 per 56 KB block) were bound by the copy queue, ~3000 cycles per block
// per SM; a quad copy moves 4 rows at once.
// Consumer warps split a block into tile groups x K slices and leave
// per-slice partial sums in a double buffer; a reducer warp
// sums the slices, applies the epilogue and stores y, so consumer warps never
// wait for one another.
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
// for MMA rows g and g+8; MMA j takes word j/2, low nibbles (codes 0,2 | 4,6)
// for even j, high nibbles (codes 1,3 | 5,7) for odd j.  About one
// instruction per code instead of a multiply-add per code on the FMA pipe.
// MMA row g of a 16-row tile is row g >> 2 of the tile's quad g & 3 and MMA
// row g + 8 is row 2 + (g >> 2) of that quad: the 4 rows an 8-byte load phase
// reads (g = 0..3 or 4..7) sit in different quads, whose slots start 32 bytes
// apart modulo 128, so they hit disjoint banks.
//
// 8-bit codes.  An 8-bit code q = lo + 16 hi is two consecutive nibbles of
// the packed word, so an 8-bit row of K codes is a row of 2K nibbles and runs
// through the same MMAs: x is staged as the pair (x_j, 16 x_j) for the
// nibbles (lo_j, hi_j) (exact in bf16), so that D_u = sum x'(128 + nibble)
// and sum_j x_j q_j = D_u - 128 * 17 * X_u; per unit of 32 codes (64 nibbles)
//   sum_j x_j (s q_j + o) = s * D_u + (o - 2176 s) * X_u.
//
// Weights immutable (qmm_set_weights_immutable): the producer streams the
// first ring stages of codes, scales and offsets without waiting for the
// previous kernel, so they arrive while that kernel drains; x and the
// epilogue inputs are still read only after the dependency wait.
//
// Launch.  With programmatic dependent launch the next launch's CTAs take
// each SM as soon as this grid's CTA there exits, instead of after the whole
// grid drains and a new launch ramps up.  Every read of codes, scales, x,
// bias, gate, residual and every write of y comes after griddepcontrol.wait,
// so weights or x written by the kernel just before are seen in full.
//
// Reference computation: image-forger src/quant.rs:105-113 (weights
// dequantized to f32 as scale * q + offset, f32 accumulation); the products
// x * (128 + q) are exact in f32.  Every wait is bounded (qmm_common.cuh).
#include <algorithm>
#include <cstdlib>

#include "qmm_epilogue.cuh"
#include "qmm_internal.h"

namespace qmm {
namespace gemvtc {

// CW consumer warps (16: measured faster than 24 single-tile warps, because
// two tiles per warp share their x fragments), then the producer warp and the
// reducer warp (at most 32 warps per block).
template <int CW>
struct Warps {
    static_assert(CW + 2 <= 32, "at most 1024 threads per block");
    static constexpr int kProducer = CW;
    static constexpr int kReducer = CW + 1;
    static constexpr int kThreads = (CW + 2) * 32;
};
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
    int32_t row_bytes, quad_stride, nblocks;   // quad slot = 4 rows + 32 bytes
    int32_t stage_bytes, meta_off;            // scales at meta_off, offsets after them
    int32_t xp_stride;                        // u32 words per staged token
    int32_t prefetch_weights;                 // codes/scales/offsets streamed before the dependency wait
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

// Stages x in MMA order (threads [0, nthreads) of the block, whole warps).
// Entry (token, u, t, j, r) of xp holds x at codes c0 = 64u + 16t + 8(j/2) +
// (j%2) + 4r and c0 + 2 of the token (low half c0).  One task per
// (token, u, t) reads its 16 codes with two 16-byte loads and writes its 8
// entries; the four tasks of a unit sum X_u with shuffles.  Token row m of xp
// is zero: B fragments of lanes whose token is >= m read it.
template <int MP>
__device__ __forceinline__ void stage_x(const uint16_t *x, uint32_t *xp, float *xsum, int m, int k, int units,
                                        int xp_stride, int tid, int nthreads) {
    for (int i = tid; i < units * 32; i += nthreads) xp[(size_t)m * xp_stride + i] = 0u;
    for (int i = tid; i < units * MP; i += nthreads)
        if (i % MP >= m) xsum[i] = 0.0f;
    const int tasks = m * units * 4;
    const int tasks_rounded = (tasks + 31) & ~31;  // whole warps: the shuffles below see all lanes
    for (int base = 0; base < tasks_rounded; base += nthreads) {
        const int i = base + tid;
        const bool act = i < tasks;
        const int t = i & 3, ut = i >> 2;
        const int tok = act ? ut / units : 0, u = act ? ut - tok * units : 0;
        float sum = 0.0f;
        if (act) {
            const uint4 *src = reinterpret_cast<const uint4 *>(x + (size_t)tok * k + u * kUnit + 16 * t);
            const uint4 v0 = __ldg(src), v1 = __ldg(src + 1);
            const uint32_t w[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};  // codes 2i | 2i+1
            uint32_t out[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const int jj = e >> 1, r = e & 1;
                const int c0 = 8 * (jj >> 1) + (jj & 1) + 4 * r, c1 = c0 + 2;
                const uint32_t lo = (w[c0 >> 1] >> ((c0 & 1) * 16)) & 0xFFFFu;
                const uint32_t hi = (w[c1 >> 1] >> ((c1 & 1) * 16)) & 0xFFFFu;
                out[e] = lo | (hi << 16);
            }
            uint4 *dst = reinterpret_cast<uint4 *>(xp + (size_t)tok * xp_stride + u * 32 + t * 8);
            dst[0] = make_uint4(out[0], out[1], out[2], out[3]);
            dst[1] = make_uint4(out[4], out[5], out[6], out[7]);
#pragma unroll
            for (int q = 0; q < 8; ++q) sum += __uint_as_float(w[q] << 16) + __uint_as_float(w[q] & 0xFFFF0000u);
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        if (act && t == 0) xsum[u * MP + tok] = sum;
    }
}

// 8-bit codes as nibble pairs: unit u of the nibble row covers codes
// [32u, 32u + 32); nibble c of the unit is code 32u + c/2, with x weighted by
// 16 for odd c (the high nibble).  Entry (token, u, t, j, r) holds x' at
// nibbles c0 = 16t + 8(j/2) + (j%2) + 4r and c0 + 2, as in stage_x; one task
// per (token, u, t) reads its 8 codes with one 16-byte load.  X_u is the sum
// of the 32 codes' x (not x').
template <int MP>
__device__ __forceinline__ void stage_x8(const uint16_t *x, uint32_t *xp, float *xsum, int m, int k, int units,
                                         int xp_stride, int tid, int nthreads) {
    for (int i = tid; i < units * 32; i += nthreads) xp[(size_t)m * xp_stride + i] = 0u;
    for (int i = tid; i < units * MP; i += nthreads)
        if (i % MP >= m) xsum[i] = 0.0f;
    const int tasks = m * units * 4;
    const int tasks_rounded = (tasks + 31) & ~31;
    for (int base = 0; base < tasks_rounded; base += nthreads) {
        const int i = base + tid;
        const bool act = i < tasks;
        const int t = i & 3, ut = i >> 2;
        const int tok = act ? ut / units : 0, u = act ? ut - tok * units : 0;
        float sum = 0.0f;
        if (act) {
            const uint4 v = __ldg(reinterpret_cast<const uint4 *>(x + (size_t)tok * k + u * (kUnit / 2) + 8 * t));
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};  // codes 2i | 2i+1
            auto xnib = [&](int c) -> uint32_t {  // x' of nibble c of this task (bf16 bits)
                const int code = c >> 1;
                const uint32_t b = (w[code >> 1] >> ((code & 1) * 16)) & 0xFFFFu;
                if (!(c & 1)) return b;
                const __nv_bfloat16 h = __float2bfloat16_rn(bf16_bits_to_f32(b) * 16.0f);  // exact
                return *reinterpret_cast<const uint16_t *>(&h);
            };
            uint32_t out[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const int jj = e >> 1, r = e & 1;
                const int c0 = 8 * (jj >> 1) + (jj & 1) + 4 * r;
                out[e] = xnib(c0) | (xnib(c0 + 2) << 16);
            }
            uint4 *dst = reinterpret_cast<uint4 *>(xp + (size_t)tok * xp_stride + u * 32 + t * 8);
            dst[0] = make_uint4(out[0], out[1], out[2], out[3]);
            dst[1] = make_uint4(out[4], out[5], out[6], out[7]);
#pragma unroll
            for (int q = 0; q < 4; ++q) sum += __uint_as_float(w[q] << 16) + __uint_as_float(w[q] & 0xFFFF0000u);
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        if (act && t == 0) xsum[u * MP + tok] = sum;
    }
}

// Shared memory (16-byte aligned regions):
//   stages [stages][rb / 4 quad slots of codes | rb*groups scales | rb*groups offsets]
//   xp     [m + 1][units][4 lanes t][4 MMAs j][2] u32   x in MMA order (bf16 pairs); row m zero
//   xsum   [units][MP] f32                            X_u per token (zero beyond m)
//   part   [2][ks][rb][m] f32                         partial sums per K slice (ks = 16 warps)
//   bars   full[kMaxStages], empty[kMaxStages], pready[2], pfree[2]
template <int BITS, int MT, int TPW, int CW>
__global__ void __launch_bounds__(Warps<CW>::kThreads, CW == 8 ? 2 : 1) qmm_gemv_mma_kernel(const Params p) {
    // sum_j x_j q_j = D_u - kOff * X_u (see the header comment).
    constexpr float kOff = BITS == 4 ? 128.0f : 2176.0f;
    using W = Warps<CW>;
    constexpr int MP = 8 * MT;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t *stages = smem;
    uint32_t *xp = reinterpret_cast<uint32_t *>(smem + (size_t)p.stages * p.stage_bytes);
    float *xsum = reinterpret_cast<float *>(xp + (size_t)(p.m + 1) * p.xp_stride);  // after the zero row m
    float *part = xsum + (size_t)p.units * MP;
    uint64_t *full = reinterpret_cast<uint64_t *>(
        (reinterpret_cast<uintptr_t>(part + 2 * (size_t)p.ks * p.rb * p.m) + 15) & ~uintptr_t(15));
    uint64_t *empty = full + kMaxStages;
    uint64_t *pready = empty + kMaxStages;  // [2] consumer warps -> reducer
    uint64_t *pfree = pready + 2;           // [2] reducer -> consumer warps
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_launch_dependents();

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CW);
        }
        for (int q = 0; q < 2; ++q) {
            mbar_init(&pready[q], CW);
            mbar_init(&pfree[q], 1);
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == W::kReducer) {
        // ----------------------------------------------------------- reducer
        // Block j's partials are in part[j & 1]; the (j >> 1)-th completion of
        // pready[j & 1] says every consumer warp has written its slice.
        pdl_dependency_wait();  // bias, gate and residual may come from the previous kernel; y may be read by it
        bool rok = true;
        int j = 0;
        for (int b = blockIdx.x; b < p.nblocks; b += gridDim.x, ++j) {
            const int q = j & 1;
            rok = rok && mbar_wait(&pready[q], (j >> 1) & 1, p.err, kErrTimeoutEpilogue);
            const int64_t row0 = (int64_t)b * p.rb;
            const float *pr = part + (size_t)q * p.ks * p.rb * p.m;
            for (int i = lane; rok && i < p.rb * p.m; i += 32) {
                const int row = i / p.m, tok = i - row * p.m;
                const int64_t n = row0 + row;
                if (n >= p.n) continue;
                float v = 0.0f;
#pragma unroll 4
                for (int ks = 0; ks < p.ks; ++ks) v += pr[(size_t)ks * p.rb * p.m + i];
                const FeatureConsts fc = load_feature_consts(p.ep, n, true);
                const int64_t idx = (int64_t)tok * p.n + n;
                p.y[idx] = f32_to_bf16_bits(epilogue_value(p.ep, fc, v, p.ep.residual ? p.ep.residual + idx : nullptr));
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&pfree[q]);
        }
        return;
    }

    if (warp == W::kProducer) {
        // ---------------------------------------------------------- producer
        // Weights that no kernel writes need not wait for the previous one.
        if (!p.prefetch_weights) pdl_dependency_wait();
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
            for (int q = lane; q * 4 < rows; q += 32)  // rows is a multiple of 8 (n % 8 == 0)
                bulk_load(st + (size_t)q * p.quad_stride, p.packed + (row0 + 4 * q) * p.row_bytes,
                          4u * (uint32_t)p.row_bytes, &full[s]);
            if (lane == 0) bulk_load(st + p.meta_off, p.scales + row0 * p.groups, meta, &full[s]);
            if (lane == 1)
                bulk_load(st + p.meta_off + (size_t)p.rb * p.groups * 2, p.offsets + row0 * p.groups, meta,
                          &full[s]);
        }
        return;  // consumers never wait on the producer warp's exit
    }

    // ------------------------------------------------- stage x in MMA order
    const int consumer_threads = CW * 32;
    pdl_dependency_wait();  // x may come from the previous kernel
    if constexpr (BITS == 4) stage_x<MP>(p.x, xp, xsum, p.m, p.k, p.units, p.xp_stride, threadIdx.x, consumer_threads);
    else stage_x8<MP>(p.x, xp, xsum, p.m, p.k, p.units, p.xp_stride, threadIdx.x, consumer_threads);
    named_barrier(1, consumer_threads);

    // ---------------------------------------------------------- consumers
    // Warp w takes K slice w % ks (units [slice * upw, (slice + 1) * upw)) of
    // the TPW 16-row tiles of tile group w / ks; lane (g, t) holds rows
    // 16 tile + g and 16 tile + g + 8, tokens 2t and 2t + 1 of each 8-token tile.
    const int g = lane >> 2, t = lane & 3;
    const int tg = warp / p.ks, ksl = warp - tg * p.ks;
    const int tile0 = tg * TPW;
    const int u0 = ksl * p.upw, u1 = min(p.units, u0 + p.upw);
    const uint32_t *xb[MT];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
        const int tok = mt * 8 + g;
        xb[mt] = xp + (size_t)(tok < p.m ? tok : p.m) * p.xp_stride + t * 8;
    }
    bool ok = true;
    int j = 0;
    for (int b = blockIdx.x; b < p.nblocks; b += gridDim.x, ++j) {
        const int s = j % p.stages;
        ok = ok && mbar_wait(&full[s], (j / p.stages) & 1, p.err, kErrTimeoutDequant);
        const uint8_t *st = stages + (size_t)s * p.stage_bytes;
        const uint16_t *ssc = reinterpret_cast<const uint16_t *>(st + p.meta_off);
        const uint16_t *sof = ssc + (size_t)p.rb * p.groups;
        float2 acc[MT][TPW][2];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int tl = 0; tl < TPW; ++tl) acc[mt][tl][0] = acc[mt][tl][1] = make_float2(0.0f, 0.0f);
        if (ok) {
            const uint8_t *rowp = st + (size_t)(tile0 * 4 + (g & 3)) * p.quad_stride + (size_t)(g >> 2) * p.row_bytes + t * 8;
            const size_t tile_bytes = (size_t)4 * p.quad_stride, half_bytes = (size_t)2 * p.row_bytes;
#pragma unroll 2
            for (int u = u0; u < u1; ++u) {
                uint32_t bfr[MT][8];
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    const uint4 v0 = *reinterpret_cast<const uint4 *>(xb[mt] + u * 32);
                    const uint4 v1 = *reinterpret_cast<const uint4 *>(xb[mt] + u * 32 + 4);
                    bfr[mt][0] = v0.x; bfr[mt][1] = v0.y; bfr[mt][2] = v0.z; bfr[mt][3] = v0.w;
                    bfr[mt][4] = v1.x; bfr[mt][5] = v1.y; bfr[mt][6] = v1.z; bfr[mt][7] = v1.w;
                }
                // Per tile: two independent chains (low- and high-nibble MMAs).
                float d[MT][TPW][4], e[MT][TPW][4];
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int tl = 0; tl < TPW; ++tl)
#pragma unroll
                        for (int q = 0; q < 4; ++q) d[mt][tl][q] = e[mt][tl][q] = 0.0f;
#pragma unroll
                for (int tl = 0; tl < TPW; ++tl) {
                    const uint2 wa = *reinterpret_cast<const uint2 *>(rowp + tl * tile_bytes + u * 32);
                    const uint2 wb = *reinterpret_cast<const uint2 *>(rowp + tl * tile_bytes + half_bytes + u * 32);
                    const uint32_t wa_[2] = {wa.x, wa.y}, wb_[2] = {wb.x, wb.y};
#pragma unroll
                    for (int h = 0; h < 2; ++h) {  // word 2t + h of the unit
                        const uint32_t la = wa_[h] & 0x0F0F0F0Fu, ha = (wa_[h] >> 4) & 0x0F0F0F0Fu;
                        const uint32_t lb = wb_[h] & 0x0F0F0F0Fu, hb = (wb_[h] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt) {
                            // MMA 2h: low nibbles; MMA 2h + 1: high nibbles.
                            mma_bf16_m16n8k16(d[mt][tl], code_pair<0x4140>(la), code_pair<0x4140>(lb),
                                              code_pair<0x4342>(la), code_pair<0x4342>(lb), bfr[mt][4 * h + 0],
                                              bfr[mt][4 * h + 1]);
                            mma_bf16_m16n8k16(e[mt][tl], code_pair<0x4140>(ha), code_pair<0x4140>(hb),
                                              code_pair<0x4342>(ha), code_pair<0x4342>(hb), bfr[mt][4 * h + 2],
                                              bfr[mt][4 * h + 3]);
                        }
                    }
                }
                const int gi = u >> p.unit_shift;
                float2 sc[TPW][2], cc[TPW][2];
#pragma unroll
                for (int tl = 0; tl < TPW; ++tl) {
#pragma unroll
                    for (int hr = 0; hr < 2; ++hr) {
                        const int row = (tile0 + tl) * 16 + 4 * (g & 3) + (g >> 2) + 2 * hr;  // block row
                        const float sv = bf16_bits_to_f32(ssc[row * p.groups + gi]);
                        const float cv = fmaf(-kOff, sv, bf16_bits_to_f32(sof[row * p.groups + gi]));
                        sc[tl][hr] = make_float2(sv, sv);
                        cc[tl][hr] = make_float2(cv, cv);
                    }
                }
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    const float2 xs2 = *reinterpret_cast<const float2 *>(xsum + u * MP + mt * 8 + 2 * t);
#pragma unroll
                    for (int tl = 0; tl < TPW; ++tl) {
                        const float2 da = add_f32x2(make_float2(d[mt][tl][0], d[mt][tl][1]),
                                                    make_float2(e[mt][tl][0], e[mt][tl][1]));
                        const float2 db = add_f32x2(make_float2(d[mt][tl][2], d[mt][tl][3]),
                                                    make_float2(e[mt][tl][2], e[mt][tl][3]));
                        acc[mt][tl][0] = fma_f32x2(sc[tl][0], da, fma_f32x2(cc[tl][0], xs2, acc[mt][tl][0]));
                        acc[mt][tl][1] = fma_f32x2(sc[tl][1], db, fma_f32x2(cc[tl][1], xs2, acc[mt][tl][1]));
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);  // this warp is done reading the stage
        // Partial sums of this K slice into part[j & 1], once the reducer has
        // finished block j - 2 there.
        const int q = j & 1;
        ok = ok && mbar_wait(&pfree[q], ((j >> 1) & 1) ^ 1, p.err, kErrTimeoutDequant);
        float *pb = part + ((size_t)q * p.ks + ksl) * p.rb * p.m;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            const int t0 = mt * 8 + 2 * t;
#pragma unroll
            for (int tl = 0; tl < TPW; ++tl) {
#pragma unroll
                for (int hr = 0; hr < 2; ++hr) {
                    const int row = (tile0 + tl) * 16 + 4 * (g & 3) + (g >> 2) + 2 * hr;  // block row
                    if (t0 < p.m) pb[row * p.m + t0] = acc[mt][tl][hr].x;
                    if (t0 + 1 < p.m) pb[row * p.m + t0 + 1] = acc[mt][tl][hr].y;
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&pready[q]);
    }
}

struct Plan {
    int rb, ks, tpw, cw, stages, quad_stride, stage_bytes, meta_off, xp_stride;
    int ctas_per_sm;  // 1: 16 consumer warps and the whole shared memory; 2: two CTAs of 8 warps per SM
    size_t smem;
};

// Two CTAs per SM (8 consumer warps, 16-row blocks, half the shared memory
// each): twice the copy producers per SM, and the next launch's CTAs could
// stream next to the previous launch's last ones.  Measured slower than one
// CTA of 16 warps (adaLN 1 x 3072 x 18432: 11.65 vs 10.47 us at 4-bit, 22.79
// vs 18.50 us at 8-bit), so it runs only with QMM_GEMV_CTAS=2 (read once).
static int gemv_ctas_choice() {
    static const int v = [] {
        const char *e = getenv("QMM_GEMV_CTAS");
        return (e && (e[0] == '1' || e[0] == '2') && e[1] == '\0') ? e[0] - '0' : 0;
    }();
    return v;
}

// Units are 64 nibbles: 64 codes at 4 bits, 32 codes at 8 bits.
static int64_t units_of(const qmm_weight &w) { return w.k * w.bits / 4 / kUnit; }

static bool plan_for_ctas(const qmm_weight &w, int64_t m, int ctas, Plan &pl) {
    pl.cw = ctas == 2 ? 8 : 16;
    pl.ctas_per_sm = ctas;
    const size_t limit = ctas == 2 ? (size_t)(227 * 1024) / 2 - 1024 : kSmemLimit;
    const int mt = m <= 8 ? 1 : 2;
    const int64_t units = units_of(w), groups = w.k / w.group;
    const int64_t row_bytes = w.k * w.bits / 8;
    // 4 * row_bytes is a multiple of 128 (k % 64 == 0): quad slots 32 bytes
    // longer start 0, 32, 64, 96 bytes modulo 128 apart.
    pl.quad_stride = (int)(4 * row_bytes + 32);
    pl.xp_stride = (int)(units * 32 + 4);  // +16 bytes: tokens start in different bank quads
    const size_t xs = (size_t)(m + 1) * pl.xp_stride * 4 + (size_t)units * 8 * mt * 4;
    // A 32-row block (two tiles per warp) when three ring stages fit, else a
    // 16-row block; with neither, any that fits two stages.  Two CTAs per SM
    // use 16-row blocks.
    for (int pass = 0; pass < 2; ++pass)
    for (int rb = ctas == 2 ? 16 : 32; rb >= 16; rb /= 2) {
        // 16 warps on a 32-row block: one tile group of two tiles; otherwise
        // one tile per warp and rb / 16 tile groups.
        const int tpw = (pl.cw == 16 && rb == 32) ? 2 : 1;
        const int ks = pl.cw / ((rb / 16) / tpw);
        const int64_t meta = (int64_t)rb * groups * 2;
        const int64_t stage = (int64_t)(rb / 4) * pl.quad_stride + 2 * meta;
        const size_t fixed = xs + 2 * (size_t)ks * rb * m * 4 + 16 + (2 * kMaxStages + 4) * 8 + 64;
        int stages = kMaxStages;
        while (stages >= 2 && fixed + (size_t)stages * stage > limit) --stages;
        if (stages < (pass == 0 ? 3 : 2)) continue;
        pl.rb = rb;
        pl.ks = ks;
        pl.tpw = tpw;
        pl.stages = stages;
        pl.stage_bytes = (int)stage;
        pl.meta_off = (rb / 4) * pl.quad_stride;
        pl.smem = fixed + (size_t)stages * stage;
        return true;
    }
    return false;
}

static bool plan_for(const qmm_weight &w, int64_t m, Plan &pl) {
    if (gemv_ctas_choice() == 2) return plan_for_ctas(w, m, 2, pl);
    return plan_for_ctas(w, m, 1, pl);
}

template <int BITS, int MT, int TPW, int CW>
static qmm_status launch_t(const qmm_weight &w, const uint16_t *x, int64_t m, const qmm_epilogue &ep,
                           uint16_t *y, cudaStream_t st) {
    Plan pl;
    if (!plan_for(w, m, pl) || pl.tpw != TPW || pl.cw != CW)
        return fail(QMM_ERR_UNSUPPORTED, "gemv (mma): layout does not fit shared memory");
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(qmm_gemv_mma_kernel<BITS, MT, TPW, CW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
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
    p.ep = epilogue_args(ep);
    p.n = w.n;
    p.k = (int32_t)w.k;
    p.m = (int32_t)m;
    p.groups = (int32_t)(w.k / w.group);
    p.units = (int32_t)units_of(w);
    int us = 0;  // units per group = 2^us
    while ((kUnit << us) < w.group * BITS / 4) ++us;
    p.unit_shift = us;
    p.rb = pl.rb;
    p.ks = pl.ks;
    p.upw = (p.units + pl.ks - 1) / pl.ks;
    p.stages = pl.stages;
    p.row_bytes = (int32_t)(w.k * BITS / 8);
    p.quad_stride = pl.quad_stride;
    p.nblocks = (int32_t)((w.n + pl.rb - 1) / pl.rb);
    p.stage_bytes = pl.stage_bytes;
    p.meta_off = pl.meta_off;
    p.xp_stride = pl.xp_stride;
    p.err = device_error_word();
    const bool pdl = gemv_pdl_enabled();
    p.prefetch_weights = (pdl && weights_immutable()) ? 1 : 0;
    const int grid = (int)std::min<int64_t>(p.nblocks, (int64_t)sm_count() * pl.ctas_per_sm);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(Warps<CW>::kThreads);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, qmm_gemv_mma_kernel<BITS, MT, TPW, CW>, p);
    count_launch();
    if (e == cudaSuccess) e = cudaGetLastError();
    return e == cudaSuccess ? QMM_OK : cuda_fail(e, "gemv (mma) launch");
}

}  // namespace gemvtc


bool gemv_mma_supported(const qmm_weight &w, int64_t m) {
    if ((w.bits != 4 && w.bits != 8) || m < 1 || m > 16) return false;
    if (w.k % gemvtc::kUnit != 0 || w.group % gemvtc::kUnit != 0) return false;
    const int per = w.group * w.bits / 4 / gemvtc::kUnit;  // units per group
    if ((per & (per - 1)) != 0) return false;
    if (w.n % 8 != 0 || w.k > (1 << 20) || w.n > ((int64_t)1 << 31)) return false;
    // Scale/offset blocks are copied in 16-byte pieces.
    if ((reinterpret_cast<uintptr_t>(w.scales) | reinterpret_cast<uintptr_t>(w.biases)) & 15u) return false;
    gemvtc::Plan pl;
    return gemvtc::plan_for(w, m, pl);
}

qmm_status launch_gemv_mma(const qmm_weight &w, const uint16_t *x, int64_t m, const qmm_epilogue &ep,
                           uint16_t *y, cudaStream_t st) {
    gemvtc::Plan pl;
    if (!gemvtc::plan_for(w, m, pl)) return fail(QMM_ERR_UNSUPPORTED, "gemv (mma): layout does not fit shared memory");
    if (pl.cw == 8) {  // two CTAs per SM: 16-row blocks, one tile per warp
        if (w.bits == 8)
            return m <= 8 ? gemvtc::launch_t<8, 1, 1, 8>(w, x, m, ep, y, st) : gemvtc::launch_t<8, 2, 1, 8>(w, x, m, ep, y, st);
        return m <= 8 ? gemvtc::launch_t<4, 1, 1, 8>(w, x, m, ep, y, st) : gemvtc::launch_t<4, 2, 1, 8>(w, x, m, ep, y, st);
    }
    if (w.bits == 8) {
        if (m <= 8)
            return pl.tpw == 2 ? gemvtc::launch_t<8, 1, 2, 16>(w, x, m, ep, y, st) : gemvtc::launch_t<8, 1, 1, 16>(w, x, m, ep, y, st);
        return pl.tpw == 2 ? gemvtc::launch_t<8, 2, 2, 16>(w, x, m, ep, y, st) : gemvtc::launch_t<8, 2, 1, 16>(w, x, m, ep, y, st);
    }
    if (m <= 8)
        return pl.tpw == 2 ? gemvtc::launch_t<4, 1, 2, 16>(w, x, m, ep, y, st) : gemvtc::launch_t<4, 1, 1, 16>(w, x, m, ep, y, st);
    return pl.tpw == 2 ? gemvtc::launch_t<4, 2, 2, 16>(w, x, m, ep, y, st) : gemvtc::launch_t<4, 2, 1, 16>(w, x, m, ep, y, st);
}

}  // namespace qmm
