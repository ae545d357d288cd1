// tcgen05 quantized GEMM for sm_100a:  y [m, n] = epilogue(x [m, k] . W^T).
//
// Replaces the Metal `qmm` kernel of image-forger (src/quant.rs:208-319) and
// its host op (src/quant.rs:427-502).  The reference widens x and W tiles to
// f32 in threadgroup memory and runs f32 8x8 simdgroup MMAs; here W is
// unpacked to bf16 (bit-exact with the reference dequantization) and fed to
// the 5th-generation tensor cores, which accumulate in f32 in tensor memory.
//
// Orientation: the CTA computes a tile D = Wt . xt^T of 128 weight rows
// (output features) by T tokens.  The dequantized weight tile is the MMA A
// operand and lives in TMEM (written with tcgen05.st, so the weights never
// touch shared memory in dense form); x is the B operand, loaded by TMA into
// 128-byte-swizzled shared memory.  Accumulators: two T-column buffers in
// TMEM so that the epilogue of one tile overlaps the main loop of the next.
//
// Warp roles (one persistent CTA per SM):
//   warps 0-3        epilogue: TMEM -> registers, bias/act/gate/residual, bf16 stores
//   next 4*SETS      dequant: packed codes (smem) -> bf16 -> TMEM A slots; SETS
//                    groups of four warps take alternate K-blocks so several
//                    blocks are in flight
//   next warp        producer: TMA for x and packed tiles
//   last warp        MMA issuer (one thread) and TMEM allocator
// Pipeline: a ring of shared-memory stages (x tile, packed codes) deep enough to
// cover TMA latency, decoupled from a ring of 4 TMEM A slots.  Each dequant
// thread owns one weight row and prefetches its row's scale and offset one
// block ahead from global memory (they are tiny and stay in L1/L2).
// Every wait is bounded (qmm_common.cuh): on expiry the CTA records an error
// code, drains its own in-flight copies and MMAs, frees TMEM and exits.
#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "qmm_epilogue.cuh"
#include "qmm_internal.h"
#include "qmm_unpack.cuh"

namespace qmm {
namespace gemm {

constexpr int kWRows = 128;  // weight rows per tile = TMEM lanes = MMA M
constexpr int kBK = 64;      // K per pipeline block (4 MMAs of K = 16)
constexpr int kASlots = 4;   // TMEM A slots (32 columns each)
constexpr int kEpiWarps = 4;
constexpr int kTmemCols = 512;

// Warp layout: epilogue warps 0-3, dequant warps 4 .. 4 + 4*SETS - 1 (set j
// handles K-blocks i with i % SETS == j, quadrant = warp % 4), then the
// producer warp and the MMA warp.
template <int SETS>
struct Warps {
    static constexpr int kDq0 = kEpiWarps;
    static constexpr int kDqWarps = 4 * SETS;
    static constexpr int kProducer = kDq0 + kDqWarps;
    static constexpr int kMma = kProducer + 1;
    static constexpr int kThreads = (kMma + 1) * 32;
};

template <int BITS, int T>
struct Cfg {
    static_assert(T % 32 == 0 && T >= 32 && T <= 256, "token tile");
    static constexpr int kXStageBytes = T * kBK * 2;               // bf16 [T][64], 128B-swizzled
    static constexpr int kPWords = kBK * BITS / 32;                // packed words per row per block
    static constexpr int kPStageBytes = kWRows * kPWords * 4;      // uint32 [128][kPWords], swizzled
    static constexpr int kStageBytes = kXStageBytes + kPStageBytes;
    static constexpr int kSmemBudget = 227 * 1024 - 2048;
    static constexpr int kStages = kSmemBudget / kStageBytes > 8 ? 8 : kSmemBudget / kStageBytes;
    static constexpr int kXOff = 0;
    static constexpr int kPOff = kXOff + kStages * kXStageBytes;
    static constexpr int kBarOff = kPOff + kStages * kPStageBytes;
    static constexpr int kNumBars = 2 * kStages + 2 * kASlots + 4 + 1;
    static constexpr int kTmemPtrOff = kBarOff + kNumBars * 8;
    static constexpr int kSmemBytes = kTmemPtrOff + 16 + 1024;  // + alignment slack
    static constexpr int kAcc0 = 0;                              // accumulator b at b*T
    static constexpr int kASlot0 = 2 * T;                        // A slot a at kASlot0 + 32 a
    static_assert(kStages >= 3, "pipeline depth");
    static_assert(2 * T + kASlots * 32 <= kTmemCols, "TMEM budget");
    static_assert(kXStageBytes % 1024 == 0 && kPStageBytes % 1024 == 0, "stage alignment");
    static_assert(kSmemBytes <= 232448, "shared memory");
    static constexpr uint32_t kIdesc = idesc_bf16_f32(kWRows, T);
};

struct Params {
    const uint16_t *scales;
    const uint16_t *offsets;
    uint16_t *y;
    EpilogueArgs ep;
    int32_t m, n, k;
    int32_t group, groups, group_shift;
    int32_t w_tiles, num_tiles;
    uint32_t *err;
};

// Byte offset of 16-byte chunk `c` of row `r` in a TMA tile written with
// 32-byte (4-bit rows) or 64-byte (8-bit rows) swizzling.
template <int BITS>
__device__ __forceinline__ uint32_t packed_chunk_offset(int r, int c) {
    if constexpr (BITS == 4) return r * 32 + ((c ^ ((r >> 2) & 1)) << 4);
    else return r * 64 + ((c ^ ((r >> 1) & 3)) << 4);
}

// Dequantizes the 64 codes of weight row `row` of one pipeline block into 32
// bf16 pairs (k order), bit-exact with the reference's f32-then-bf16 rounding.
// m0 / m1 = scale | offset << 16 (bf16 bits) of the groups holding codes
// [0, 32) and [32, 64) of the block (equal unless group == 32).
template <int BITS>
__device__ __forceinline__ void dequant_row_block(const uint8_t *pst, uint32_t m0, uint32_t m1, int row,
                                                  uint32_t (&a)[32]) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {  // 32-code halves (a group of 32 each when group == 32)
        const uint32_t mh = h == 0 ? m0 : m1;
        const float sc1 = bf16_bits_to_f32(mh & 0xFFFFu);
        const float of1 = bf16_bits_to_f32(mh >> 16);
        const float2 sc = make_float2(sc1, sc1), of = make_float2(of1, of1);
        if constexpr (BITS == 4) {
            const uint4 w4 = *reinterpret_cast<const uint4 *>(pst + packed_chunk_offset<4>(row, h));
            const uint32_t ws[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint32_t o4[4];
                dequant_word_bf16x2_packed<4>(ws[j], sc, of, o4);
#pragma unroll
                for (int t = 0; t < 4; ++t) a[h * 16 + j * 4 + t] = o4[t];
            }
        } else {
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
                const uint4 w4 = *reinterpret_cast<const uint4 *>(pst + packed_chunk_offset<8>(row, h * 2 + cc));
                const uint32_t ws[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    uint32_t o2[2];
                    dequant_word_bf16x2_packed<8>(ws[j], sc, of, o2);
                    a[h * 16 + cc * 8 + j * 2 + 0] = o2[0];
                    a[h * 16 + cc * 8 + j * 2 + 1] = o2[1];
                }
            }
        }
    }
}

template <int BITS, int T, int SETS>
__global__ void __launch_bounds__(Warps<SETS>::kThreads, 1)
    qmm_gemm_kernel(const __grid_constant__ CUtensorMap tmap_x,
                    const __grid_constant__ CUtensorMap tmap_w, const Params p) {
    using C = Cfg<BITS, T>;
    using W = Warps<SETS>;
    constexpr int S = C::kStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::kBarOff);  // [S] x + codes + meta landed
    uint64_t *sempty = full + S;                                       // [S] stage consumed
    uint64_t *afull = sempty + S;                                      // [A] A slot written
    uint64_t *aempty = afull + kASlots;                                // [A] MMAs reading the slot done
    uint64_t *acc_full = aempty + kASlots;                             // [2] tile accumulated
    uint64_t *acc_empty = acc_full + 2;                                // [2] tile drained
    uint64_t *drain = acc_empty + 2;                                   // error-path MMA drain
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + C::kTmemPtrOff);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&sempty[s], 1 + 4);  // MMA commit + the 4 dequant warps of the block's set
        }
        for (int a = 0; a < kASlots; ++a) {
            mbar_init(&afull[a], 4);
            mbar_init(&aempty[a], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], kEpiWarps);
        }
        mbar_init(drain, 1);
        fence_barrier_init();
    }
    if (warp == W::kMma) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    if (warp == W::kProducer && lane == 0) {
        tma_prefetch_desc(&tmap_x);
        tma_prefetch_desc(&tmap_w);
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    const int nkb = p.k / kBK;
    const int local_tiles = (p.num_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
    const uint32_t total_blocks = (uint32_t)local_tiles * (uint32_t)nkb;

    if (warp == W::kProducer) {
        // ---------------------------------------------------------- producer
        uint32_t i = 0;
        bool ok = true;
        for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
            const int n0 = (tile % p.w_tiles) * kWRows;
            const int m0 = (tile / p.w_tiles) * T;
            for (int kb = 0; kb < nkb; ++kb, ++i) {
                const int s = i % S;
                if (!mbar_wait(&sempty[s], ((i / S) & 1) ^ 1, p.err, kErrTimeoutProducer)) {
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    mbar_arrive_expect_tx(&full[s], C::kXStageBytes + C::kPStageBytes);
                    tma_load_2d(smem + C::kXOff + s * C::kXStageBytes, &tmap_x, &full[s], kb * kBK, m0);
                    tma_load_2d(smem + C::kPOff + s * C::kPStageBytes, &tmap_w, &full[s], kb * C::kPWords, n0);
                }
                __syncwarp();
            }
        }
        if (!ok) {
            // Let the copies already issued land before the CTA exits.
            const uint32_t first = i > (uint32_t)S ? i - S : 0;
            for (uint32_t j = first; j < i; ++j)
                mbar_wait(&full[j % S], (j / S) & 1, p.err, kErrTimeoutDrain);
        }
    } else if (warp == W::kMma) {
        // ---------------------------------------------------------- MMA issuer
        if (lane == 0) {
            uint32_t i = 0;
            int lt = 0;
            bool ok = true;
            bool issued = false;
            for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x, ++lt) {
                const int b = lt & 1;
                const uint32_t u = lt >> 1;
                if (!mbar_wait(&acc_empty[b], (u & 1) ^ 1, p.err, kErrTimeoutMma)) {
                    ok = false;
                    break;
                }
                tc_fence_after_sync();
                const uint32_t d = tmem + C::kAcc0 + b * T;
                for (int kb = 0; kb < nkb; ++kb, ++i) {
                    const int s = i % S;
                    const int a = i % kASlots;
                    if (!mbar_wait(&afull[a], (i / kASlots) & 1, p.err, kErrTimeoutMma) ||
                        !mbar_wait(&full[s], (i / S) & 1, p.err, kErrTimeoutMma)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after_sync();
                    const uint32_t atm = tmem + C::kASlot0 + a * 32;
                    const uint64_t bdesc =
                        sdesc_kmajor_sw128(smem_u32(smem + C::kXOff + s * C::kXStageBytes));
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk)
                        tc_mma_ts(d, atm + kk * 8, bdesc + (uint64_t)(kk * 2), C::kIdesc,
                                  (kb | kk) != 0 ? 1u : 0u);
                    issued = true;
                    tc_commit(&aempty[a]);
                    tc_commit(&sempty[s]);
                }
                if (!ok) break;
                tc_commit(&acc_full[b]);
            }
            if (!ok && issued) {
                tc_commit(drain);
                mbar_wait(drain, 0, p.err, kErrTimeoutDrain);
            }
        }
        __syncwarp();
    } else if (warp >= W::kDq0) {
        // ---------------------------------------------------------- dequant
        const int quad = warp & 3;                 // TMEM lane quadrant
        const int set = (warp - W::kDq0) >> 2;     // blocks i with i % SETS == set
        const int row = quad * 32 + lane;          // weight row within the tile
        const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
        // Scale/offset of this thread's row for block (tile_local, kb), one
        // block ahead.  Group index of codes [0,32) / [32,64) of block kb:
        // (kb * 64) >> log2(group) and (kb * 64 + 32) >> log2(group).
        const int gshift = p.group_shift;
        auto load_meta = [&](int tile_local, int kb, uint32_t &m0, uint32_t &m1) {
            m0 = m1 = 0;
            const int tile = (int)blockIdx.x + tile_local * (int)gridDim.x;
            const int wt = tile - (tile / p.w_tiles) * p.w_tiles;
            const int n = wt * kWRows + row;
            if (tile < p.num_tiles && n < p.n) {
                const uint16_t *sp = p.scales + (int64_t)n * p.groups;
                const uint16_t *op = p.offsets + (int64_t)n * p.groups;
                const int g0 = (kb * kBK) >> gshift;
                const int g1 = (kb * kBK + 32) >> gshift;
                m0 = (uint32_t)__ldg(sp + g0) | ((uint32_t)__ldg(op + g0) << 16);
                m1 = g1 == g0 ? m0 : ((uint32_t)__ldg(sp + g1) | ((uint32_t)__ldg(op + g1) << 16));
            }
        };
        int tl = set / nkb, kb = set - (set / nkb) * nkb;
        uint32_t m0 = 0, m1 = 0;
        if ((uint32_t)set < total_blocks) load_meta(tl, kb, m0, m1);
        int s = set % S, a = set % kASlots;
        uint32_t ph_s = (set / S) & 1, ph_a = (set / kASlots) & 1;
        for (uint32_t i = set; i < total_blocks; i += SETS) {
            int ntl = tl, nkb_i = kb + SETS;
            while (nkb_i >= nkb) {
                nkb_i -= nkb;
                ++ntl;
            }
            uint32_t n0m = 0, n1m = 0;
            if (i + SETS < total_blocks) load_meta(ntl, nkb_i, n0m, n1m);
            if (!mbar_wait(&full[s], ph_s, p.err, kErrTimeoutDequant) ||
                !mbar_wait(&aempty[a], ph_a ^ 1, p.err, kErrTimeoutDequant))
                break;
            uint32_t v[32];
            dequant_row_block<BITS>(smem + C::kPOff + s * C::kPStageBytes, m0, m1, row, v);
            tmem_st_32x32b_x32(tmem + lane_addr + C::kASlot0 + a * 32, v);
            __syncwarp();
            if (lane == 0) mbar_arrive(&sempty[s]);  // the stage's codes are in registers
            tc_wait_st();
            tc_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(&afull[a]);
            m0 = n0m;
            m1 = n1m;
            tl = ntl;
            kb = nkb_i;
            s += SETS;
            if (s >= S) {
                s -= S;
                ph_s ^= 1;
            }
            a += SETS;
            if (a >= kASlots) {
                a -= kASlots;
                ph_a ^= 1;
            }
        }
    } else {
        // ---------------------------------------------------------- epilogue
        const int quad = warp;
        const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
        int lt = 0;
        for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++lt) {
            const int b = lt & 1;
            const uint32_t u = lt >> 1;
            const int n0 = (tile % p.w_tiles) * kWRows;
            const int m0 = (tile / p.w_tiles) * T;
            if (!mbar_wait(&acc_full[b], u & 1, p.err, kErrTimeoutEpilogue)) break;
            tc_fence_after_sync();
            const int64_t n = n0 + quad * 32 + lane;
            const bool nvalid = n < p.n;
            const FeatureConsts fc = load_feature_consts(p.ep, n, nvalid);
#pragma unroll 1
            for (int c0 = 0; c0 < T; c0 += 32) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(tmem + lane_addr + C::kAcc0 + b * T + c0, v);
                tc_wait_ld();
                if (c0 + 32 >= T) {
                    // Accumulator drained into registers: let the MMA reuse it.
                    tc_fence_before_sync();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&acc_empty[b]);
                }
                if (nvalid) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int64_t mm = m0 + c0 + j;
                        if (mm < p.m) {
                            const int64_t idx = mm * p.n + n;
                            const float val = epilogue_value(
                                p.ep, fc, __uint_as_float(v[j]),
                                p.ep.residual ? p.ep.residual + idx : nullptr);
                            p.y[idx] = f32_to_bf16_bits(val);
                        }
                    }
                }
            }
        }
    }

    // ------------------------------------------------------------------ teardown
    __syncwarp();
    tc_fence_before_sync();
    __syncthreads();
    if (warp == W::kMma) {
        tc_fence_after_sync();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ---------------------------------------------------------------------- host
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    });
    return fn;
}

static qmm_status make_map_2d(CUtensorMap *map, CUtensorMapDataType dtype, int esize,
                              const void *base, uint64_t inner, uint64_t outer,
                              uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                              CUtensorMapSwizzle swz) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(QMM_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    (void)esize;
    CUresult r = fn(map, dtype, 2, const_cast<void *>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(QMM_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return QMM_OK;
}

template <int BITS, int T, int SETS>
static qmm_status launch_t(const qmm_weight &w, const uint16_t *x, int64_t m,
                           const qmm_epilogue &ep, uint16_t *y, cudaStream_t st) {
    using C = Cfg<BITS, T>;
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(qmm_gemm_kernel<BITS, T, SETS>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             C::kSmemBytes);
        if (e != cudaSuccess) return cuda_fail(e, "gemm smem attribute");
        configured[dev] = true;
    }
    CUtensorMap tx, tw;
    qmm_status s = make_map_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, (uint64_t)w.k,
                               (uint64_t)m, (uint64_t)w.k * 2, kBK, T,
                               CU_TENSOR_MAP_SWIZZLE_128B);
    if (s != QMM_OK) return s;
    const uint64_t words = (uint64_t)w.k * BITS / 32;
    s = make_map_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, w.packed, words, (uint64_t)w.n,
                    words * 4, C::kPWords, kWRows,
                    BITS == 4 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B);
    if (s != QMM_OK) return s;

    Params p;
    p.scales = w.scales;
    p.offsets = w.biases;
    p.y = y;
    p.ep = EpilogueArgs{ep.bias, ep.gate, ep.residual, ep.activation};
    p.m = (int32_t)m;
    p.n = (int32_t)w.n;
    p.k = (int32_t)w.k;
    p.group = w.group;
    p.groups = (int32_t)(w.k / w.group);
    p.group_shift = 0;
    while ((1 << p.group_shift) < w.group) ++p.group_shift;
    p.w_tiles = (int32_t)((w.n + kWRows - 1) / kWRows);
    const int64_t t_tiles = (m + T - 1) / T;
    p.num_tiles = (int32_t)(p.w_tiles * t_tiles);
    p.err = device_error_word();
    const int grid = (int)std::min<int64_t>(p.num_tiles, sm_count());
    qmm_gemm_kernel<BITS, T, SETS><<<grid, Warps<SETS>::kThreads, C::kSmemBytes, st>>>(tx, tw, p);
    count_launch();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? QMM_OK : cuda_fail(e, "gemm launch");
}

}  // namespace gemm

bool gemm_supported(const qmm_weight &w) {
    if (w.bits != 4 && w.bits != 8) return false;
    if (w.k % gemm::kBK != 0) return false;
    if (!(w.group == 32 || w.group % gemm::kBK == 0)) return false;
    if ((w.group & (w.group - 1)) != 0) return false;  // power-of-two groups (MLX: 32, 64, 128)
    if (w.n > (int64_t)INT32_MAX - gemm::kWRows || w.k > (int64_t)INT32_MAX / 8) return false;
    return true;
}

qmm_status launch_gemm(const qmm_weight &w, const uint16_t *x, int64_t m, const qmm_epilogue &ep,
                       uint16_t *y, cudaStream_t st) {
    if (m > (int64_t)INT32_MAX - 256) return fail(QMM_ERR_UNSUPPORTED, "gemm: m too large");
    static const int sets = [] {
        const char *e = getenv("QMM_GEMM_SETS");
        return (e && atoi(e) == 2) ? 2 : 4;
    }();
    if (w.bits == 4)
        return sets == 2 ? gemm::launch_t<4, 192, 2>(w, x, m, ep, y, st)
                         : gemm::launch_t<4, 192, 4>(w, x, m, ep, y, st);
    return sets == 2 ? gemm::launch_t<8, 192, 2>(w, x, m, ep, y, st)
                     : gemm::launch_t<8, 192, 4>(w, x, m, ep, y, st);
}

}  // namespace qmm
