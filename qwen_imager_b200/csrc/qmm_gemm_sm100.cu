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
// Warp roles (448 threads, one persistent CTA per SM):
//   warps 0-3   epilogue: TMEM -> registers, bias/act/gate/residual, bf16 stores
//   warps 4-11  dequant:  packed codes (smem) -> bf16 -> TMEM A slots
//   warp 12     producer: TMA for x and packed tiles, scale/offset staging
//   warp 13     MMA issuer (one thread) and TMEM allocator
// Every wait is bounded (qmm_common.cuh): on expiry the CTA records an error
// code, drains its own in-flight copies and MMAs, frees TMEM and exits.
#include <algorithm>
#include <mutex>

#include "qmm_epilogue.cuh"
#include "qmm_internal.h"
#include "qmm_unpack.cuh"

namespace qmm {
namespace gemm {

constexpr int kWRows = 128;  // weight rows per tile = TMEM lanes = MMA M
constexpr int kBK = 64;      // K per pipeline stage (4 MMAs of K = 16)
constexpr int kStages = 4;   // smem stages = TMEM A slots
constexpr int kEpiWarps = 4;
constexpr int kDqWarps = 8;
constexpr int kProducerWarp = 12;
constexpr int kMmaWarp = 13;
constexpr int kThreads = 14 * 32;
constexpr int kTmemCols = 512;

template <int BITS, int T>
struct Cfg {
    static_assert(T % 32 == 0 && T >= 32 && T <= 256, "token tile");
    static constexpr int kXStageBytes = T * kBK * 2;               // bf16 [T][64]
    static constexpr int kPWords = kBK * BITS / 32;                // words per row per stage
    static constexpr int kPStageBytes = kWRows * kPWords * 4;      // uint32 [128][kPWords]
    static constexpr int kMetaStageBytes = kWRows * 2 * 4;         // (s,o) x 2 groups per row
    static constexpr int kXOff = 0;
    static constexpr int kPOff = kXOff + kStages * kXStageBytes;
    static constexpr int kMetaOff = kPOff + kStages * kPStageBytes;
    static constexpr int kBarOff = kMetaOff + kStages * kMetaStageBytes;
    static constexpr int kNumBars = 3 * kStages + 4 + 1;
    static constexpr int kTmemPtrOff = kBarOff + kNumBars * 8;
    static constexpr int kSmemBytes = kTmemPtrOff + 16 + 1024;  // + alignment slack
    static constexpr int kAcc0 = 0;                              // accumulator b at b*T
    static constexpr int kASlot0 = 2 * T;                        // A slot s at kASlot0 + 32 s
    static_assert(2 * T + kStages * 32 <= kTmemCols, "TMEM budget");
    static_assert(kXStageBytes % 1024 == 0 && kPStageBytes % 1024 == 0, "stage alignment");
    static constexpr uint32_t kIdesc = idesc_bf16_f32(kWRows, T);
};

struct Params {
    const uint16_t *scales;
    const uint16_t *offsets;
    uint16_t *y;
    EpilogueArgs ep;
    int32_t m, n, k;
    int32_t group, groups;
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

template <int BITS, int T>
__global__ void __launch_bounds__(kThreads, 1)
    qmm_gemm_kernel(const __grid_constant__ CUtensorMap tmap_x,
                    const __grid_constant__ CUtensorMap tmap_w, const Params p) {
    using C = Cfg<BITS, T>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::kBarOff);  // TMA + meta landed
    uint64_t *afull = full + kStages;                                  // A slot written
    uint64_t *empty = afull + kStages;                                 // MMAs of the stage done
    uint64_t *acc_full = empty + kStages;                              // [2] tile accumulated
    uint64_t *acc_empty = acc_full + 2;                                // [2] tile drained
    uint64_t *drain = acc_empty + 2;                                   // error-path MMA drain
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + C::kTmemPtrOff);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 32);
            mbar_init(&afull[s], kDqWarps);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], kEpiWarps);
        }
        mbar_init(drain, 1);
        fence_barrier_init();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    if (warp == kProducerWarp && lane == 0) {
        tma_prefetch_desc(&tmap_x);
        tma_prefetch_desc(&tmap_w);
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    const int nkb = p.k / kBK;

    if (warp == kProducerWarp) {
        // ---------------------------------------------------------- producer
        uint32_t i = 0;
        bool ok = true;
        for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
            const int n0 = (tile % p.w_tiles) * kWRows;
            const int m0 = (tile / p.w_tiles) * T;
            for (int kb = 0; kb < nkb; ++kb, ++i) {
                const int s = i % kStages;
                const uint32_t r = i / kStages;
                if (!mbar_wait(&empty[s], (r & 1) ^ 1, p.err, kErrTimeoutProducer)) {
                    ok = false;
                    break;
                }
                // Scales and offsets of this stage: meta[row][h] = s | o << 16, where
                // h selects the 32-code half of the stage (two groups when group == 32).
                uint32_t *meta = reinterpret_cast<uint32_t *>(smem + C::kMetaOff + s * C::kMetaStageBytes);
#pragma unroll
                for (int j = 0; j < kWRows / 32; ++j) {
                    const int row = lane + 32 * j;
                    const int64_t n = n0 + row;
                    uint32_t v0 = 0, v1 = 0;
                    if (n < p.n) {
                        const int64_t base = n * p.groups;
                        const int g0 = (kb * kBK) / p.group;
                        const int g1 = (kb * kBK + 32) / p.group;
                        v0 = (uint32_t)__ldg(p.scales + base + g0) |
                             ((uint32_t)__ldg(p.offsets + base + g0) << 16);
                        v1 = g1 == g0 ? v0
                                      : ((uint32_t)__ldg(p.scales + base + g1) |
                                         ((uint32_t)__ldg(p.offsets + base + g1) << 16));
                    }
                    meta[row * 2 + 0] = v0;
                    meta[row * 2 + 1] = v1;
                }
                if (lane == 0) {
                    mbar_arrive_expect_tx(&full[s], C::kXStageBytes + C::kPStageBytes);
                    tma_load_2d(smem + C::kXOff + s * C::kXStageBytes, &tmap_x, &full[s], kb * kBK, m0);
                    tma_load_2d(smem + C::kPOff + s * C::kPStageBytes, &tmap_w, &full[s], kb * C::kPWords, n0);
                } else {
                    mbar_arrive(&full[s]);
                }
            }
        }
        if (!ok) {
            // Let the copies already issued land before the CTA exits.
            const uint32_t first = i > (uint32_t)kStages ? i - kStages : 0;
            for (uint32_t j = first; j < i; ++j)
                mbar_wait(&full[j % kStages], (j / kStages) & 1, p.err, kErrTimeoutDrain);
        }
    } else if (warp == kMmaWarp) {
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
                    const int s = i % kStages;
                    const uint32_t r = i / kStages;
                    if (!mbar_wait(&afull[s], r & 1, p.err, kErrTimeoutMma) ||
                        !mbar_wait(&full[s], r & 1, p.err, kErrTimeoutMma)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after_sync();
                    const uint32_t a = tmem + C::kASlot0 + s * 32;
                    const uint64_t bdesc =
                        sdesc_kmajor_sw128(smem_u32(smem + C::kXOff + s * C::kXStageBytes));
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk)
                        tc_mma_ts(d, a + kk * 8, bdesc + (uint64_t)(kk * 2), C::kIdesc,
                                  (kb | kk) != 0 ? 1u : 0u);
                    issued = true;
                    tc_commit(&empty[s]);
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
    } else if (warp >= kEpiWarps) {
        // ---------------------------------------------------------- dequant
        const int quad = warp & 3;           // TMEM lane quadrant
        const int half = (warp - 4) >> 2;    // codes [32 half, 32 half + 32) of the stage
        const int row = quad * 32 + lane;    // weight row within the tile
        const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
        uint32_t i = 0;
        bool ok = true;
        for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
            for (int kb = 0; kb < nkb; ++kb, ++i) {
                const int s = i % kStages;
                const uint32_t r = i / kStages;
                if (!mbar_wait(&full[s], r & 1, p.err, kErrTimeoutDequant) ||
                    !mbar_wait(&empty[s], (r & 1) ^ 1, p.err, kErrTimeoutDequant)) {
                    ok = false;
                    break;
                }
                const uint32_t meta = reinterpret_cast<const uint32_t *>(
                    smem + C::kMetaOff + s * C::kMetaStageBytes)[row * 2 + half];
                const float sc = bf16_bits_to_f32(meta & 0xFFFFu);
                const float of = bf16_bits_to_f32(meta >> 16);
                const uint8_t *pst = smem + C::kPOff + s * C::kPStageBytes;
                uint32_t a[16];
                if constexpr (BITS == 4) {
                    const uint4 w4 = *reinterpret_cast<const uint4 *>(pst + packed_chunk_offset<4>(row, half));
                    const uint32_t ws[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        uint32_t o4[4];
                        dequant_word_bf16x2<4>(ws[j], sc, of, o4);
#pragma unroll
                        for (int t = 0; t < 4; ++t) a[j * 4 + t] = o4[t];
                    }
                } else {
#pragma unroll
                    for (int cc = 0; cc < 2; ++cc) {
                        const uint4 w4 = *reinterpret_cast<const uint4 *>(
                            pst + packed_chunk_offset<8>(row, half * 2 + cc));
                        const uint32_t ws[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            uint32_t o2[2];
                            dequant_word_bf16x2<8>(ws[j], sc, of, o2);
                            a[cc * 8 + j * 2 + 0] = o2[0];
                            a[cc * 8 + j * 2 + 1] = o2[1];
                        }
                    }
                }
                tmem_st_32x32b_x16(tmem + lane_addr + C::kASlot0 + s * 32 + half * 16, a);
                tc_wait_st();
                tc_fence_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive(&afull[s]);
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
            tc_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);
        }
    }

    // ------------------------------------------------------------------ teardown
    __syncwarp();
    tc_fence_before_sync();
    __syncthreads();
    if (warp == kMmaWarp) {
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

template <int BITS, int T>
static qmm_status launch_t(const qmm_weight &w, const uint16_t *x, int64_t m,
                           const qmm_epilogue &ep, uint16_t *y, cudaStream_t st) {
    using C = Cfg<BITS, T>;
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(qmm_gemm_kernel<BITS, T>,
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
    p.w_tiles = (int32_t)((w.n + kWRows - 1) / kWRows);
    const int64_t t_tiles = (m + T - 1) / T;
    p.num_tiles = (int32_t)(p.w_tiles * t_tiles);
    p.err = device_error_word();
    const int grid = (int)std::min<int64_t>(p.num_tiles, sm_count());
    qmm_gemm_kernel<BITS, T><<<grid, kThreads, C::kSmemBytes, st>>>(tx, tw, p);
    count_launch();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? QMM_OK : cuda_fail(e, "gemm launch");
}

}  // namespace gemm

bool gemm_supported(const qmm_weight &w) {
    if (w.bits != 4 && w.bits != 8) return false;
    if (w.k % gemm::kBK != 0) return false;
    if (!(w.group == 32 || w.group % gemm::kBK == 0)) return false;
    if (w.n > (int64_t)INT32_MAX - gemm::kWRows || w.k > (int64_t)INT32_MAX / 8) return false;
    return true;
}

qmm_status launch_gemm(const qmm_weight &w, const uint16_t *x, int64_t m, const qmm_epilogue &ep,
                       uint16_t *y, cudaStream_t st) {
    if (m > (int64_t)INT32_MAX - 256) return fail(QMM_ERR_UNSUPPORTED, "gemm: m too large");
    if (w.bits == 4) return gemm::launch_t<4, 192>(w, x, m, ep, y, st);
    return gemm::launch_t<8, 192>(w, x, m, ep, y, st);
}

}  // namespace qmm
