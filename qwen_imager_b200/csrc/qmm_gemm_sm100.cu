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
//   warps 0-3        epilogue: TMEM -> registers, bias/act/gate/residual in f32,
//                    bf16 chunks staged in shared memory and written by TMA stores
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
#include <atomic>
#include <mutex>

#include "qmm_epilogue.cuh"
#include "qmm_internal.h"
#include "qmm_unpack.cuh"

namespace qmm {
namespace gemm {

constexpr int kWRows = 128;  // weight rows per tile = TMEM lanes = MMA M
constexpr int kBK = 64;      // K per pipeline block (4 MMAs of K = 16)
constexpr int kEpiWarps = 4;
constexpr int kTmemCols = 512;

// Warp layout: epilogue warps 0-3, then 4 * SETS * HALVES dequant warps (set
// j handles K-blocks i with i % SETS == j; within a set, warp quadrant q and
// half h dequantize codes [32 h, 32 h + 32) of rows 32 q .. 32 q + 31), then
// the producer warp and the MMA warp.
template <int SETS, int HALVES>
struct Warps {
    static constexpr int kDq0 = kEpiWarps;
    static constexpr int kPerSet = 4 * HALVES;
    static constexpr int kDqWarps = kPerSet * SETS;
    static constexpr int kProducer = kDq0 + kDqWarps;
    static constexpr int kMma = kProducer + 1;
    static constexpr int kThreads = (kMma + 1) * 32;
};

// T: tokens per tile (MMA N, accumulator columns).  PAIR: the tile spans a CTA
// pair (cta_group::2, MMA M = 256), each CTA holding 128 weight rows and T/2
// of the tile's tokens in shared memory.
template <int BITS, int T, bool PAIR, bool F16 = false>
struct Cfg {
    static_assert(T % 32 == 0 && T >= 32 && T <= 256, "token tile");
    static constexpr int kXRows = PAIR ? T / 2 : T;                // x rows staged per CTA
    static constexpr int kXStageBytes = kXRows * kBK * 2;          // bf16 [kXRows][64], 128B-swizzled
    static constexpr int kPWords = kBK * BITS / 32;                // packed words per row per block
    static constexpr int kPStageBytes = kWRows * kPWords * 4;      // uint32 [128][kPWords], swizzled
    static constexpr int kStageBytes = kXStageBytes + kPStageBytes;
    // TMEM: two T-column accumulators, the rest as 32-column A slots (at most 8).
    static constexpr int kASlots = (512 - 2 * T) / 32 > 8 ? 8 : (512 - 2 * T) / 32;
    // Epilogue staging: one 32-token chunk of the 128-row tile, [32][128] f32
    // (bf16 outputs use the first half), written back with 16-byte stores.
    static constexpr int kEStageBytes = 32 * kWRows * 4;
    static constexpr int kSmemBudget = 227 * 1024 - 2048 - kEStageBytes;
    static constexpr int kStages = kSmemBudget / kStageBytes > 8 ? 8 : kSmemBudget / kStageBytes;
    static constexpr int kXOff = 0;
    static constexpr int kPOff = kXOff + kStages * kXStageBytes;
    static constexpr int kEOff = kPOff + kStages * kPStageBytes;
    static constexpr int kBarOff = kEOff + kEStageBytes;
    static constexpr int kNumBars = 3 * kStages + 2 * 8 + 4 + 1 + 2;
    static constexpr int kTmemPtrOff = kBarOff + kNumBars * 8;
    static constexpr int kSmemBytes = kTmemPtrOff + 16 + 1024;  // + alignment slack
    static constexpr int kAcc0 = 0;                              // accumulator b at b*T
    static constexpr int kASlot0 = 2 * T;                        // A slot a at kASlot0 + 32 a
    static_assert(kStages >= 3, "pipeline depth");
    static_assert(2 * T + kASlots * 32 <= kTmemCols, "TMEM budget");
    static_assert(kXStageBytes % 1024 == 0 && kPStageBytes % 1024 == 0, "stage alignment");
    static_assert(kSmemBytes <= 232448, "shared memory");
    static constexpr uint32_t kIdesc = F16 ? idesc_f16_f32(PAIR ? 2 * kWRows : kWRows, T)
                                           : idesc_bf16_f32(PAIR ? 2 * kWRows : kWRows, T);
};

// Work unit u of num_units = tiles * splits covers output tile u % tiles and
// k-blocks [split * kbs, (split + 1) * kbs) with split = u / tiles.  With
// splits > 1 the epilogue writes f32 partial tiles to ws[split][m][n] and
// qmm_splitk_reduce_kernel applies the epilogue.
struct Params {
    const uint16_t *scales;
    const uint16_t *offsets;
    uint16_t *y;
    float *ws;
    EpilogueArgs ep;
    int32_t m, n, k;
    int32_t group, groups, group_shift;
    int32_t w_tiles, tiles, num_units, splits, kbs;
    // k-block pairs: dequantization sets 2j and 2j+1 fill A slots 2j, 2j+1
    // and arrive on one barrier; the MMA warp waits once per two k-blocks.
    // Requires 4 sets, 4 A slots, 1 CTA and an even kbs.
    int32_t kpair;
    // The residual chunk of each write-back is loaded by TMA into the staging
    // buffer (needs a residual, no split-K and n % 8 == 0).
    int32_t res_tma;
    uint32_t *err;
};

// Test support (qmm_debug_gemm_stall), read only by the STALL instantiation
// of the kernel: every wait gives up after wait_ns, and the copy producer of
// every CTA stops before its `withhold`-th k-block, so that the waits for that
// block run out and the error path runs.  Set per device by gemm_set_stall.
struct StallConfig {
    uint64_t wait_ns;
    int32_t withhold;
};
__device__ StallConfig g_stall_cfg = {kWaitLimitNs, -1};

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
// [0, 32) and [32, 64) of the block (equal unless group == 32).  NH halves
// starting at half H0 (or at `hbase` when H0 < 0) are produced.
template <int BITS, int H0, int NH, bool F16 = false>
__device__ __forceinline__ void dequant_row_block(const uint8_t *pst, uint32_t m0, uint32_t m1, int row,
                                                  uint32_t (&a)[16 * NH], int hbase) {
#pragma unroll
    for (int hh = 0; hh < NH; ++hh) {  // 32-code halves (a group of 32 each when group == 32)
        const int h = H0 >= 0 ? H0 + hh : hbase + hh;
        const uint32_t mh = hh == 0 ? m0 : m1;
        const float sc1 = bf16_bits_to_f32(mh & 0xFFFFu);
        const float of1 = bf16_bits_to_f32(mh >> 16);
        const float2 sc = make_float2(sc1, sc1), of = make_float2(of1, of1);
        if constexpr (BITS == 4) {
            const uint4 w4 = *reinterpret_cast<const uint4 *>(pst + packed_chunk_offset<4>(row, h));
            const uint32_t ws[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint32_t o4[4];
                dequant_word_bf16x2_packed<4, F16>(ws[j], sc, of, o4);
#pragma unroll
                for (int t = 0; t < 4; ++t) a[hh * 16 + j * 4 + t] = o4[t];
            }
        } else {
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
                const uint4 w4 = *reinterpret_cast<const uint4 *>(pst + packed_chunk_offset<8>(row, h * 2 + cc));
                const uint32_t ws[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    uint32_t o2[2];
                    dequant_word_bf16x2_packed<8, F16>(ws[j], sc, of, o2);
                    a[hh * 16 + cc * 8 + j * 2 + 0] = o2[0];
                    a[hh * 16 + cc * 8 + j * 2 + 1] = o2[1];
                }
            }
        }
    }
}

template <int BITS, int T, int SETS, int HALVES, bool PAIR, bool STALL = false, bool F16 = false>
__global__ void __launch_bounds__(Warps<SETS, HALVES>::kThreads, 1)
    qmm_gemm_kernel(const __grid_constant__ CUtensorMap tmap_x,
                    const __grid_constant__ CUtensorMap tmap_w,
                    const __grid_constant__ CUtensorMap tmap_out,
                    const __grid_constant__ CUtensorMap tmap_res, const Params p) {
    using C = Cfg<BITS, T, PAIR, F16>;
    using W = Warps<SETS, HALVES>;
    // The normal instantiation waits with the constant limit and withholds
    // nothing (the same code as without test support).
    uint64_t wait_ns = kWaitLimitNs;
    int32_t withhold = -1;
    if constexpr (STALL) {
        wait_ns = g_stall_cfg.wait_ns;
        withhold = g_stall_cfg.withhold;
    }
    constexpr int S = C::kStages;
    constexpr int kASlots = C::kASlots;
    constexpr int kTileRows = PAIR ? 2 * kWRows : kWRows;  // weight rows per (pair) tile
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::kBarOff);  // [S] this CTA's stage landed
    uint64_t *xfull = full + S;                                        // [S] PAIR: both x halves (leader)
    uint64_t *sempty = xfull + S;                                      // [S] stage consumed
    uint64_t *afull = sempty + S;                                      // [A] A slot written
    uint64_t *aempty = afull + kASlots;                                // [A] MMAs reading the slot done
    uint64_t *acc_full = aempty + kASlots;                             // [2] tile accumulated
    uint64_t *acc_empty = acc_full + 2;                                // [2] tile drained
    uint64_t *drain = acc_empty + 2;                                   // error-path MMA drain
    uint64_t *rfull = drain + 1;                                       // [2] residual chunk landed
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + C::kTmemPtrOff);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    constexpr int kPairCtas = PAIR ? 2 : 1;
    const uint32_t rank = PAIR ? cluster_ctarank() : 0;  // 0 = the pair's leader (issues MMAs)
    const bool leader = rank == 0;
    // Scheduling unit: one CTA, or one CTA pair (cluster of two).
    const int unit = PAIR ? (int)cluster_id_x() : (int)blockIdx.x;
    const int nunits = PAIR ? (int)cluster_count_x() : (int)gridDim.x;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&xfull[s], 1);
            mbar_init(&sempty[s], 1 + W::kPerSet);  // MMA commit + the dequant warps of the block's set
        }
        for (int a = 0; a < kASlots; ++a) {
            mbar_init(&afull[a], kPairCtas * W::kPerSet * (p.kpair ? 2 : 1));
            mbar_init(&aempty[a], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], kPairCtas * kEpiWarps);
        }
        mbar_init(drain, 1);
        mbar_init(&rfull[0], 1);
        mbar_init(&rfull[1], 1);
        fence_barrier_init();
    }
    if (warp == W::kMma) {
        if constexpr (PAIR) {
            tmem_alloc_pair(tmem_slot, kTmemCols);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(tmem_slot, kTmemCols);
            tmem_relinquish();
        }
    }
    if (warp == W::kProducer && lane == 0) {
        tma_prefetch_desc(&tmap_x);
        tma_prefetch_desc(&tmap_w);
        tma_prefetch_desc(&tmap_out);
        if (p.res_tma) tma_prefetch_desc(&tmap_res);
    }
    tc_fence_before_sync();
    __syncthreads();
    if constexpr (PAIR) cluster_sync();  // peer barriers initialized, TMEM allocated in both CTAs
    tc_fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    const int nkb = p.kbs;  // k-blocks per work unit
    const int local_tiles = (p.num_units - unit + nunits - 1) / nunits;
    const uint32_t total_blocks = (uint32_t)local_tiles * (uint32_t)nkb;
    // Barriers of the pair's leader that every CTA of the pair signals.
    auto leader_bar = [&](uint64_t *bar) { return PAIR ? mapa_shared(smem_u32(bar), 0) : smem_u32(bar); };
    auto arrive_leader = [&](uint64_t *bar) {
        if constexpr (PAIR) mbar_arrive_cluster(mapa_shared(smem_u32(bar), 0));
        else mbar_arrive(bar);
    };

    if (warp == W::kProducer) {
        // ---------------------------------------------------------- producer
        uint32_t i = 0;
        bool ok = true;
        int s = 0;
        uint32_t ph_s = 0;
        for (int wu = unit; ok && wu < p.num_units; wu += nunits) {
            const int tile = wu % p.tiles, kb0 = (wu / p.tiles) * nkb;
            const int n0 = (tile % p.w_tiles) * kTileRows + (int)rank * kWRows;
            const int m0 = (tile / p.w_tiles) * T + (int)rank * C::kXRows;
            for (int kb = kb0; kb < kb0 + nkb; ++kb, ++i) {
                if constexpr (STALL) {
                    if ((int32_t)i == withhold) {  // this block's copies are never issued
                        ok = false;
                        break;
                    }
                }
                if (!mbar_wait<PAIR>(&sempty[s], ph_s ^ 1, p.err, kErrTimeoutProducer, wait_ns)) {
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    if constexpr (PAIR) {
                        // Both x halves complete on the leader's xfull; codes on this CTA's full.
                        if (leader) mbar_arrive_expect_tx(&xfull[s], 2 * C::kXStageBytes);
                        tma_load_2d_pair(smem + C::kXOff + s * C::kXStageBytes, &tmap_x, leader_bar(&xfull[s]),
                                         kb * kBK, m0);
                        mbar_arrive_expect_tx(&full[s], C::kPStageBytes);
                    } else {
                        mbar_arrive_expect_tx(&full[s], C::kXStageBytes + C::kPStageBytes);
                        tma_load_2d(smem + C::kXOff + s * C::kXStageBytes, &tmap_x, &full[s], kb * kBK, m0);
                    }
                    tma_load_2d(smem + C::kPOff + s * C::kPStageBytes, &tmap_w, &full[s], kb * C::kPWords, n0);
                }
                __syncwarp();
                if (++s == S) {
                    s = 0;
                    ph_s ^= 1;
                }
            }
        }
        // This CTA issues no more loads: a kernel launched after this one as a
        // programmatic dependent (the streaming GEMV) may take SMs as the
        // CTAs of this grid exit; it reads this grid's outputs only after
        // its dependency wait.
        pdl_launch_dependents();
        if (!ok) {
            // Let the copies already issued land before the CTA exits.
            const uint32_t first = i > (uint32_t)S ? i - S : 0;
            for (uint32_t j = first; j < i; ++j)
                mbar_wait<PAIR>(&full[j % S], (j / S) & 1, p.err, kErrTimeoutDrain, wait_ns);
        }
    } else if (warp == W::kMma) {
        // ---------------------------------------------------------- MMA issuer
        // The whole warp runs the loop (warp-uniform control flow keeps the
        // descriptors and TMEM addresses in uniform registers); one elected
        // lane issues the MMAs and commits.
        if (leader) {
            bool ok = true;
            bool issued = false;
            constexpr uint16_t kBoth = 0x3;
            const uint64_t bdesc0 = sdesc_kmajor_sw128(smem_u32(smem + C::kXOff));
            constexpr uint64_t kBStep = C::kXStageBytes >> 4;  // descriptor start-address units
            int s = 0, a = 0;
            uint32_t ph_s = 0, ph_a = 0;
            int lt = 0;
            for (int wu = unit; ok && wu < p.num_units; wu += nunits, ++lt) {
                const int b = lt & 1;
                ok = __all_sync(0xffffffffu, mbar_wait<PAIR>(&acc_empty[b], ((lt >> 1) & 1) ^ 1, p.err, kErrTimeoutMma, wait_ns));
                if (!ok) break;
                tc_fence_after_sync();
                const uint32_t d = tmem + C::kAcc0 + b * T;
                uint32_t acc = 0;
                if (!PAIR && p.kpair) {
                    // Two k-blocks per A-slot-pair barrier (see Params::kpair);
                    // afull implies full[s] and full[s + 1] as below.
                    for (int kb = 0; kb < nkb; kb += 2) {
                        const int pb = a >> 1;
                        ok = __all_sync(0xffffffffu, mbar_wait<PAIR>(&afull[pb], ph_a, p.err, kErrTimeoutMma, wait_ns));
                        if (!ok) break;
                        tc_fence_after_sync();
                        const int s1 = s + 1 == S ? 0 : s + 1;
                        if (lane_elect()) {
#pragma unroll
                            for (int h = 0; h < 2; ++h) {
                                const uint32_t atm = tmem + C::kASlot0 + (a + h) * 32;
                                const uint64_t bdesc = bdesc0 + (uint64_t)(h ? s1 : s) * kBStep;
#pragma unroll
                                for (int kk = 0; kk < kBK / 16; ++kk) {
                                    tc_mma_ts(d, atm + kk * 8, bdesc + (uint64_t)(kk * 2), C::kIdesc, acc);
                                    acc = 1;
                                }
                            }
                            tc_commit(&aempty[pb]);
                            tc_commit(&sempty[s]);
                            tc_commit(&sempty[s1]);
                        }
                        acc = 1;
                        issued = true;
                        for (int h = 0; h < 2; ++h) {
                            if (++s == S) {
                                s = 0;
                                ph_s ^= 1;
                            }
                        }
                        a += 2;
                        if (a == kASlots) {
                            a = 0;
                            ph_a ^= 1;
                        }
                    }
                }
                for (int kb = 0; (PAIR || !p.kpair) && kb < nkb; ++kb) {
                    // 1-CTA: afull[a] implies full[s].  The dequantization warps
                    // that arrive on afull[a] first waited on full[s], the
                    // barrier the TMA copies of this stage (x tile and codes)
                    // complete, so the release/acquire chain through afull[a]
                    // orders the MMA's shared-memory reads after those copies.
                    // A CTA pair also needs the peer's x tile: xfull[s].
                    ok = __all_sync(0xffffffffu, mbar_wait<PAIR>(&afull[a], ph_a, p.err, kErrTimeoutMma, wait_ns) &&
                                                     (!PAIR || mbar_wait<PAIR>(&xfull[s], ph_s, p.err,
                                                                               kErrTimeoutMma, wait_ns)));
                    if (!ok) break;
                    tc_fence_after_sync();
                    const uint32_t atm = tmem + C::kASlot0 + a * 32;
                    const uint64_t bdesc = bdesc0 + (uint64_t)s * kBStep;
                    if (lane_elect()) {
#pragma unroll
                        for (int kk = 0; kk < kBK / 16; ++kk) {
                            if constexpr (PAIR) tc_mma_ts_pair(d, atm + kk * 8, bdesc + (uint64_t)(kk * 2), C::kIdesc, acc);
                            else tc_mma_ts(d, atm + kk * 8, bdesc + (uint64_t)(kk * 2), C::kIdesc, acc);
                            acc = 1;
                        }
                        if constexpr (PAIR) {
                            tc_commit_pair_multicast(&aempty[a], kBoth);
                            tc_commit_pair_multicast(&sempty[s], kBoth);
                        } else {
                            tc_commit(&aempty[a]);
                            tc_commit(&sempty[s]);
                        }
                    }
                    // (No __syncwarp here: the next block's wait ends in
                    // __all_sync, which reconverges the warp.)
                    acc = 1;
                    issued = true;
                    if (++s == S) {
                        s = 0;
                        ph_s ^= 1;
                    }
                    if (++a == kASlots) {
                        a = 0;
                        ph_a ^= 1;
                    }
                }
                if (!ok) break;
                if (lane_elect()) {
                    if constexpr (PAIR) tc_commit_pair_multicast(&acc_full[b], kBoth);
                    else tc_commit(&acc_full[b]);
                }
                __syncwarp();
            }
            if (!ok && issued) {
                if (lane_elect()) {
                    if constexpr (PAIR) tc_commit_pair_multicast(drain, 0x1);
                    else tc_commit(drain);
                }
                __syncwarp();
                mbar_wait<PAIR>(drain, 0, p.err, kErrTimeoutDrain, wait_ns);
            }
        }
    } else if (warp >= W::kDq0) {
        // ---------------------------------------------------------- dequant
        const int quad = warp & 3;                          // TMEM lane quadrant
        const int widx = warp - W::kDq0;
        const int set = widx / W::kPerSet;                  // blocks i with i % SETS == set
        const int half = (widx % W::kPerSet) >> 2;          // HALVES == 2: codes [32 half, 32 half + 32)
        const int row = quad * 32 + lane;                   // weight row within the tile
        const uint32_t tcol = tmem + (static_cast<uint32_t>(quad * 32) << 16) + C::kASlot0 + half * 16;
        const int gshift = p.group_shift;
        // This thread's scale/offset row pointers for a work unit (null past
        // n), offset to the unit's first k-block.
        const uint16_t *sp = nullptr, *op = nullptr;
        int kbase = 0;
        auto set_tile = [&](int tile_local) {
            const int wu = unit + tile_local * nunits;
            const int tile = wu % p.tiles;
            const int n = (tile % p.w_tiles) * kTileRows + (int)rank * kWRows + row;
            kbase = (wu / p.tiles) * nkb;
            sp = op = nullptr;
            if (wu < p.num_units && n < p.n) {
                sp = p.scales + (int64_t)n * p.groups;
                op = p.offsets + (int64_t)n * p.groups;
            }
        };
        // (scale | offset << 16) of the group(s) this warp needs in block kb
        // of the current work unit.
        auto load_meta = [&](int kb, uint32_t &m0, uint32_t &m1) {
            m0 = m1 = 0;
            if (sp) {
                const int c0 = (kbase + kb) * kBK + (HALVES == 2 ? half * 32 : 0);
                const int g0 = c0 >> gshift;
                const int g1 = (c0 + 32) >> gshift;
                m0 = (uint32_t)__ldg(sp + g0) | ((uint32_t)__ldg(op + g0) << 16);
                if (HALVES == 1) m1 = g1 == g0 ? m0 : ((uint32_t)__ldg(sp + g1) | ((uint32_t)__ldg(op + g1) << 16));
            }
        };
        int tl = set / nkb, kb = set - (set / nkb) * nkb;
        set_tile(tl);
        uint32_t m0 = 0, m1 = 0;
        if ((uint32_t)set < total_blocks) load_meta(kb, m0, m1);
        int s = set % S, a = set % kASlots;
        uint32_t ph_s = (set / S) & 1, ph_a = (set / kASlots) & 1;
        for (uint32_t i = set; i < total_blocks; i += SETS) {
            // Advance to the next block of this set and prefetch its scales.
            int nkb_i = kb + SETS;
            if (nkb_i >= nkb) {
                while (nkb_i >= nkb) {
                    nkb_i -= nkb;
                    ++tl;
                }
                set_tile(tl);
            }
            uint32_t n0m = 0, n1m = 0;
            if (i + SETS < total_blocks) load_meta(nkb_i, n0m, n1m);
            // The codes are dequantized as soon as they land; only the store
            // into the TMEM A slot waits for the MMA that last read the slot.
            if (!mbar_wait<PAIR>(&full[s], ph_s, p.err, kErrTimeoutDequant, wait_ns)) break;
            const uint8_t *pst = smem + C::kPOff + s * C::kPStageBytes;
            constexpr int kV = HALVES == 1 ? 32 : 16;
            uint32_t v[kV];
            if constexpr (HALVES == 1) dequant_row_block<BITS, 0, 2, F16>(pst, m0, m1, row, v, 0);
            else dequant_row_block<BITS, -1, 1, F16>(pst, m0, m0, row, v, half);
            __syncwarp();
            if (lane == 0) mbar_arrive(&sempty[s]);  // the stage's codes are in registers
            const int ab = p.kpair ? (a >> 1) : a;  // the slot's barrier (shared by a slot pair)
            if (!mbar_wait<PAIR>(&aempty[ab], ph_a ^ 1, p.err, kErrTimeoutDequant, wait_ns)) break;
            if constexpr (HALVES == 1) tmem_st_32x32b_x32(tcol + a * 32, v);
            else tmem_st_32x32b_x16(tcol + a * 32, v);
            tc_wait_st();
            tc_fence_before_sync();
            __syncwarp();
            if (lane == 0) arrive_leader(&afull[ab]);
            m0 = n0m;
            m1 = n1m;
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
        uint32_t chunk = 0;  // write-back chunks so far (staging buffer parity)
        // Residual chunks by TMA: the chunk after the current one is requested
        // into the other staging buffer as soon as the store that last read
        // that buffer has finished reading it.
        constexpr uint32_t kResBytes = 32 * kWRows * 2;
        bool res_pending = false;  // a residual load is in flight (thread 0 of warp 0)
        auto load_residual = [&](uint32_t ch, int wu_c, int c0_c) {
            const int tile_c = wu_c % p.tiles;
            const int n0_c = (tile_c % p.w_tiles) * kTileRows + (int)rank * kWRows;
            const int m0_c = (tile_c / p.w_tiles) * T + c0_c;
            uint64_t *bar = &rfull[ch & 1];
            mbar_arrive_expect_tx(bar, kResBytes);
            tma_load_2d(smem + C::kEOff + (ch & 1) * (C::kEStageBytes / 2), &tmap_res, bar, n0_c, m0_c);
            res_pending = true;
        };
        if (p.res_tma && quad == 0 && lane == 0 && unit < p.num_units) load_residual(0, unit, 0);
        for (int wu = unit; wu < p.num_units; wu += nunits, ++lt) {
            const int b = lt & 1;
            const uint32_t u = lt >> 1;
            const int tile = wu % p.tiles, split = wu / p.tiles;
            const int n0 = (tile % p.w_tiles) * kTileRows + (int)rank * kWRows;
            const int m0 = (tile / p.w_tiles) * T;
            // The four epilogue warps leave together (they meet at named
            // barriers below): one expired wait ends the loop for all.
            const bool waited = mbar_wait<PAIR>(&acc_full[b], u & 1, p.err, kErrTimeoutEpilogue, wait_ns);
            if (named_barrier_or(1, kEpiWarps * 32, !waited)) break;
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
                    if (lane == 0) arrive_leader(&acc_empty[b]);
                }
                // Write-back of the chunk (32 tokens x 128 rows of the tile):
                // values go to a shared-memory staging tile that one thread
                // hands to the copy engine as one TMA store (8 KB bf16, 16 KB
                // f32; clipped at the m and n edges).  Per-thread global stores
                // of 64-byte row pieces were limited by outstanding stores per
                // SM, and per-row bulk copies by copy-engine issue.  bf16
                // chunks alternate between two staging buffers; f32 (split-K)
                // chunks use one.  Rows of y that are not 16-byte aligned
                // (n % 8 != 0) are written with element stores instead.
                const int64_t mrow = m0 + c0;
                const int lim = (int)(p.m - mrow < 32 ? p.m - mrow : 32);
                const int nrow = (int)(p.n - n0 < kWRows ? p.n - n0 : kWRows);  // valid rows of the tile
                const int eb = p.ws ? 0 : (chunk & 1);
                uint8_t *stg = smem + C::kEOff + eb * (C::kEStageBytes / 2);
                // The bulk stores that last read this staging buffer are done reading.
                if (quad == 0 && lane == 0) {
                    if (p.ws) bulk_wait_read<0>();
                    else bulk_wait_read<1>();
                }
                named_barrier(1, kEpiWarps * 32);
                if (p.ws) {
                    // Split-K: the f32 partial chunk, no epilogue (applied by the reduction).
                    float *st32 = reinterpret_cast<float *>(smem + C::kEOff);
#pragma unroll
                    for (int j = 0; j < 32; ++j) st32[j * kWRows + quad * 32 + lane] = __uint_as_float(v[j]);
                } else {
                    // Epilogue in f32, one bf16 rounding.  Residual values of 8
                    // tokens are loaded before the chunk is written back (y
                    // may alias the residual; this chunk's residual elements
                    // are all read before its bulk stores are issued).
                    uint16_t *st16 = reinterpret_cast<uint16_t *>(stg);
                    if (p.res_tma) {
                        // This chunk's residual is in the staging buffer: read
                        // it and overwrite it with the output in place.
                        mbar_wait<PAIR>(&rfull[eb], (chunk >> 1) & 1, p.err, kErrTimeoutEpilogue, wait_ns);
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            uint16_t &slot = st16[j * kWRows + quad * 32 + lane];
                            slot = f32_to_bf16_bits(
                                epilogue_value_rv(p.ep, fc, __uint_as_float(v[j]), bf16_bits_to_f32(slot)));
                        }
                    } else {
#pragma unroll
                    for (int h = 0; h < 32; h += 8) {
                        float rv[8];
                        if (p.ep.residual) {
#pragma unroll
                            for (int j = 0; j < 8; ++j)
                                rv[j] = (nvalid && h + j < lim) ? bf16_bits_to_f32(p.ep.residual[(mrow + h + j) * p.n + n])
                                                                : 0.0f;
                        }
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            st16[(h + j) * kWRows + quad * 32 + lane] =
                                f32_to_bf16_bits(epilogue_value_rv(p.ep, fc, __uint_as_float(v[h + j]), rv[j]));
                    }
                    }
                }
                fence_proxy_async_smem();
                named_barrier(1, kEpiWarps * 32);
                if (!p.ws && (p.n & 7) != 0) {
                    // Rows of y not 16-byte aligned (n % 8 != 0): element stores
                    // by all epilogue threads; the next chunk's first barrier
                    // orders these reads before the buffer is rewritten.
                    const uint16_t *st16 = reinterpret_cast<const uint16_t *>(stg);
                    for (int q = quad * 32 + lane; q < 32 * kWRows; q += kEpiWarps * 32) {
                        const int row = q / kWRows, col = q % kWRows;
                        if (row < lim && col < nrow) p.y[(mrow + row) * p.n + n0 + col] = st16[row * kWRows + col];
                    }
                } else if (quad == 0 && lane == 0 && lim > 0 && nrow > 0) {
                    if (p.ws) tma_store_3d(&tmap_out, smem + C::kEOff, n0, (int32_t)mrow, split);
                    else tma_store_2d(&tmap_out, stg, n0, (int32_t)mrow);
                }
                if (quad == 0 && lane == 0) {
                    bulk_commit();
                    res_pending = false;
                    if (p.res_tma) {
                        // Next chunk: in this tile, or the first of the next one.
                        int wu_n = wu, c0_n = c0 + 32;
                        if (c0_n >= T) {
                            wu_n = wu + nunits;
                            c0_n = 0;
                        }
                        if (wu_n < p.num_units) {
                            bulk_wait_read<1>();  // the store of chunk - 1 read the other buffer
                            load_residual(chunk + 1, wu_n, c0_n);
                        }
                    }
                }
                ++chunk;
            }
        }
        if (quad == 0 && lane == 0) {
            // On an early exit a prefetched residual chunk may still be landing.
            if (res_pending) mbar_wait<PAIR>(&rfull[chunk & 1], (chunk >> 1) & 1, p.err, kErrTimeoutDrain, wait_ns);
            bulk_wait_all();  // the stores have landed before the CTA exits
        }
    }

    // ------------------------------------------------------------------ teardown
    __syncwarp();
    tc_fence_before_sync();
    __syncthreads();
    if constexpr (PAIR) cluster_sync();  // the peer is done with this CTA's TMEM and barriers
    if (warp == W::kMma) {
        tc_fence_after_sync();
        if constexpr (PAIR) tmem_dealloc_pair(tmem, kTmemCols);
        else tmem_dealloc(tmem, kTmemCols);
    }
}

// Split-K reduction: y = epilogue(sum over splits of ws[split]), f32, one
// bf16 rounding; 4 consecutive outputs of a row per thread.
__global__ void __launch_bounds__(256) qmm_splitk_reduce_kernel(const float *__restrict__ ws, int splits,
                                                                int64_t m, int64_t n, EpilogueArgs ep,
                                                                uint16_t *y) {
    const int64_t quads = m * (n / 4);
    const int64_t plane = m * n;
    for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < quads;
         q += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = q / (n / 4), col = (q - row * (n / 4)) * 4;
        const int64_t idx = row * n + col;
        float4 acc = *reinterpret_cast<const float4 *>(ws + idx);
        for (int sp = 1; sp < splits; ++sp) {
            const float4 v = *reinterpret_cast<const float4 *>(ws + sp * plane + idx);
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        const float a[4] = {acc.x, acc.y, acc.z, acc.w};
        uint16_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const FeatureConsts fc = load_feature_consts(ep, col + j, true);
            o[j] = f32_to_bf16_bits(epilogue_value(ep, fc, a[j], ep.residual ? ep.residual + idx + j : nullptr));
        }
        *reinterpret_cast<uint2 *>(y + idx) = make_uint2(o[0] | ((uint32_t)o[1] << 16), o[2] | ((uint32_t)o[3] << 16));
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

static qmm_status make_map_3d_f32(CUtensorMap *map, const void *base, uint64_t inner, uint64_t mid,
                                  uint64_t outer, uint32_t box_inner, uint32_t box_mid) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(QMM_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[3] = {inner, mid, outer};
    cuuint64_t strides[2] = {inner * 4, inner * mid * 4};
    cuuint32_t box[3] = {box_inner, box_mid, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void *>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(QMM_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed (%d)", (int)r);
    return QMM_OK;
}

template <int BITS, int T, int SETS, int HALVES, bool PAIR, bool STALL = false, bool F16 = false>
static qmm_status launch_t(const qmm_weight &w, const uint16_t *x, int64_t m,
                           const qmm_epilogue &ep, uint16_t *y, int splits, float *ws, cudaStream_t st) {
    using C = Cfg<BITS, T, PAIR, F16>;
    auto kernel = qmm_gemm_kernel<BITS, T, SETS, HALVES, PAIR, STALL, F16>;
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             C::kSmemBytes);
        if (e != cudaSuccess) return cuda_fail(e, "gemm smem attribute");
        configured[dev] = true;
    }
    CUtensorMap tx, tw;
    qmm_status s = make_map_2d(&tx, F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                               x, (uint64_t)w.k,
                               (uint64_t)m, (uint64_t)w.k * 2, kBK, C::kXRows,
                               CU_TENSOR_MAP_SWIZZLE_128B);
    if (s != QMM_OK) return s;
    const uint64_t words = (uint64_t)w.k * BITS / 32;
    s = make_map_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, w.packed, words, (uint64_t)w.n,
                    words * 4, C::kPWords, kWRows,
                    BITS == 4 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B);
    if (s != QMM_OK) return s;
    // Output map for the epilogue's TMA stores: y [m, n] bf16, or for split-K
    // the workspace [splits, m, n] f32; box 128 rows of the tile x 32 tokens.
    // y rows that are not 16-byte aligned (n % 8 != 0) use element stores and
    // get a placeholder map.
    CUtensorMap tout;
    if (splits > 1) {
        s = make_map_3d_f32(&tout, ws, (uint64_t)w.n, (uint64_t)m, (uint64_t)splits, kWRows, 32);
    } else if (w.n % 8 == 0) {
        s = make_map_2d(&tout, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, y, (uint64_t)w.n, (uint64_t)m,
                        (uint64_t)w.n * 2, kWRows, 32, CU_TENSOR_MAP_SWIZZLE_NONE);
    } else {
        tout = tw;
    }
    if (s != QMM_OK) return s;
    // Residual map: the epilogue loads residual chunks by TMA (same box as y).
    CUtensorMap tres = tout;
    const bool res_tma = ep.residual && splits == 1 && w.n % 8 == 0;
    if (res_tma) {
        s = make_map_2d(&tres, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ep.residual, (uint64_t)w.n, (uint64_t)m,
                        (uint64_t)w.n * 2, kWRows, 32, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (s != QMM_OK) return s;
    }

    Params p;
    p.scales = w.scales;
    p.offsets = w.biases;
    p.y = y;
    p.ws = splits > 1 ? ws : nullptr;
    p.ep = epilogue_args(ep);
    p.m = (int32_t)m;
    p.n = (int32_t)w.n;
    p.k = (int32_t)w.k;
    p.group = w.group;
    p.groups = (int32_t)(w.k / w.group);
    p.group_shift = 0;
    while ((1 << p.group_shift) < w.group) ++p.group_shift;
    constexpr int kTileRows = PAIR ? 2 * kWRows : kWRows;
    p.w_tiles = (int32_t)((w.n + kTileRows - 1) / kTileRows);
    const int64_t t_tiles = (m + T - 1) / T;
    p.tiles = (int32_t)(p.w_tiles * t_tiles);
    p.splits = splits;
    p.kbs = (int32_t)(w.k / kBK / splits);
    p.num_units = p.tiles * splits;
    p.kpair = (!PAIR && SETS == 4 && HALVES == 1 && C::kASlots == 4 && p.kbs % 2 == 0) ? 1 : 0;
    p.res_tma = res_tma ? 1 : 0;
    p.err = device_error_word();
    const int ctas = PAIR ? 2 : 1;
    const int units = (int)std::min<int64_t>(p.num_units, sm_count() / ctas);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = dim3(units * ctas, 1, 1);
    cfg.blockDim = dim3(Warps<SETS, HALVES>::kThreads, 1, 1);
    cfg.dynamicSmemBytes = C::kSmemBytes;
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = ctas;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, tx, tw, tout, tres, p);
    count_launch();
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "gemm launch");
    if (splits > 1) {
        const int64_t quads = m * (w.n / 4);
        const int blocks = (int)std::min<int64_t>((quads + 255) / 256, (int64_t)sm_count() * 8);
        qmm_splitk_reduce_kernel<<<blocks, 256, 0, st>>>(ws, splits, m, w.n, p.ep, y);
        count_launch();
        e = cudaGetLastError();
        if (e != cudaSuccess) return cuda_fail(e, "split-k reduce launch");
    }
    return QMM_OK;
}

std::atomic<bool> g_stall_on{false};

}  // namespace gemm

qmm_status gemm_set_stall(int32_t withhold, uint64_t wait_ns) {
    const gemm::StallConfig cfg{wait_ns ? wait_ns : kWaitLimitNs, withhold};
    cudaError_t e = cudaMemcpyToSymbol(gemm::g_stall_cfg, &cfg, sizeof cfg);
    if (e != cudaSuccess) return cuda_fail(e, "gemm stall configuration");
    gemm::g_stall_on.store(withhold >= 0 || wait_ns != 0, std::memory_order_relaxed);
    return QMM_OK;
}

bool gemm_supported(const qmm_weight &w) {
    if (w.bits != 4 && w.bits != 8) return false;
    if (w.k % gemm::kBK != 0) return false;
    if (!(w.group == 32 || w.group % gemm::kBK == 0)) return false;
    if ((w.group & (w.group - 1)) != 0) return false;  // power-of-two groups (MLX: 32, 64, 128)
    if (w.n > (int64_t)INT32_MAX - gemm::kWRows || w.k > (int64_t)INT32_MAX / 8) return false;
    return true;
}

int gemm_recommended_splits(const qmm_weight &w, int64_t m) {
    // Split K only when the output tiles fill less than half of the SMs
    // (e.g. the DiT text stream, m = 256..512, or tensor-parallel shards):
    // the largest divisor of the k-block count, up to 8, that keeps the work
    // units within one wave.
    if (m <= 0 || w.n % 4 != 0 || !gemm_supported(w)) return 1;
    const int64_t tiles = ((w.n + gemm::kWRows - 1) / gemm::kWRows) * ((m + 191) / 192);
    const int sms = sm_count();
    if (tiles * 2 > sms) return 1;
    const int64_t nkb = w.k / gemm::kBK;
    int best = 1;
    // At least 8 k-blocks per split: below that the second (reduction) kernel
    // costs more than the idle SMs (measured at k = 384).
    for (int sp = 2; sp <= 8; ++sp)
        if (nkb % sp == 0 && nkb / sp >= 8 && tiles * sp <= sms) best = sp;
    return best;
}

qmm_status launch_gemm(const qmm_weight &w, const uint16_t *x, int64_t m, const qmm_epilogue &ep,
                       uint16_t *y, bool pair, int splits, float *ws, cudaStream_t st, bool f16) {
    if (m > (int64_t)INT32_MAX - 256) return fail(QMM_ERR_UNSUPPORTED, "gemm: m too large");
    if (f16) {
        // fp16 operands: x in fp16, the dequantized weights rounded to fp16.
        return w.bits == 4 ? gemm::launch_t<4, 192, 4, 1, false, false, true>(w, x, m, ep, y, splits, ws, st)
                           : gemm::launch_t<8, 192, 4, 1, false, false, true>(w, x, m, ep, y, splits, ws, st);
    }
    // Token tile 192 (two 192-column accumulators + four A slots fill TMEM);
    // four dequantization warp sets of full rows.  CTA pairs (cta_group::2)
    // on request: they halve the x traffic per SM but lengthen the A-slot
    // hand-off by a cross-SM round trip, which measured slower on B200.
    pair = pair && w.n > gemm::kWRows && splits == 1;
    if (gemm::g_stall_on.load(std::memory_order_relaxed) && !pair) {
        // Test support: the instantiation whose waits and producer follow
        // the stall configuration (qmm_debug_gemm_stall).
        return w.bits == 4 ? gemm::launch_t<4, 192, 4, 1, false, true>(w, x, m, ep, y, splits, ws, st)
                           : gemm::launch_t<8, 192, 4, 1, false, true>(w, x, m, ep, y, splits, ws, st);
    }
    if (w.bits == 4)
        return pair ? gemm::launch_t<4, 192, 4, 1, true>(w, x, m, ep, y, 1, nullptr, st)
                    : gemm::launch_t<4, 192, 4, 1, false>(w, x, m, ep, y, splits, ws, st);
    return pair ? gemm::launch_t<8, 192, 4, 1, true>(w, x, m, ep, y, 1, nullptr, st)
                : gemm::launch_t<8, 192, 4, 1, false>(w, x, m, ep, y, splits, ws, st);
}

}  // namespace qmm
