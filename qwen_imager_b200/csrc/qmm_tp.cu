// Tensor-parallel collectives of the DiT stack over peer memory (NVLink),
// fused with the residual update and the next LayerNorm + modulation.
//
// In the sequence-parallel stack every rank writes its gated row-parallel
// partial of every token into its own `part` buffer; rank r owns tokens
// [r L, (r + 1) L).  One kernel per rank then:
//   1. waits until every rank's partial is complete (a counter in its own
//      memory that every rank increments once per layer);
//   2. for each owned token, reads that token's row from every rank's `part`
//      (peer loads over NVLink for the other ranks) and sums them in f32;
//   3. x = bf16(x + sum + gate * bias), one rounding (the GEMM epilogue's
//      residual arithmetic);
//   4. n = bf16(LayerNorm(x) * (1 + scale) + shift);
//   5. stores n into every rank's `gathered` buffer at the token's row (peer
//      stores), the input of the next column-parallel linear on every rank;
//   6. counts itself done; the last CTA increments every rank's `done`
//      counter.
// A one-thread kernel before it signals "partial ready" to every rank, and a
// one-thread kernel after it waits until every rank is done before the next
// linear reads `gathered` (and before this rank's next row-parallel GEMM
// overwrites `part`, which the other ranks have then finished reading).
//
// This replaces an NCCL reduce-scatter, the residual + norm kernel and an
// NCCL all-gather: the same bytes cross NVLink (each rank receives (N-1)/N of
// its rows' partials and sends (N-1)/N of every normalised row), in one pass,
// with the partials summed in f32 instead of in bf16 along a ring.
//
// Counters are monotonic (no reset between layers): the k-th call of a stack
// on every rank waits for count >= k * world.  Every wait is bounded
// (%globaltimer); on expiry the kernel records an error in the library's
// device error word (qmm_device_error) and skips its work, so every rank's
// next wait expires too instead of hanging.  The reduction streams the
// partials with bulk copies (cp.async.bulk, no multicast) from every rank's
// memory into a shared-memory ring (reduce_pipelined_kernel); the normalised
// rows go out with plain 16-byte stores.
#include <algorithm>
#include <cstdlib>

#include "qmm_epilogue.cuh"
#include "qmm_internal.h"

namespace qmm {
namespace tp {

constexpr int kWarps = 8;
constexpr uint64_t kTpWaitLimitNs = 4000000000ull;
constexpr uint32_t kErrTimeoutPeer = 7;

// Counter slots in every rank's counter array.
enum Counter { kReady = 0, kDone = 1, kLocal = 2 };

struct Args {
    int32_t world, rank;
    uint16_t *part[QMM_TP_MAX_RANKS];
    uint16_t *gathered[QMM_TP_MAX_RANKS];
    uint64_t *counters[QMM_TP_MAX_RANKS];
    uint64_t epoch;
    int64_t rows, split;  // rows owned by this rank; local row where stream 1 begins
    uint16_t *x;          // [rows, hidden], this rank's tokens of the hidden state
    const uint16_t *bias[2], *gate[2], *shift[2], *scale[2];
    float eps;
    uint32_t *err;
    int32_t stages;       // pipelined kernel: shared-memory ring stages (a power of two, 2..16)
};

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t *p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_add_release_sys(uint64_t *p, uint64_t v) {
    asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Waits until *counter >= target; false (and the error recorded) on expiry
// or when another wait of this library already failed.
__device__ __forceinline__ bool wait_counter(const uint64_t *counter, uint64_t target, uint32_t *err) {
    if (ld_acquire_sys(counter) >= target) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 1;; ++it) {
        __nanosleep(64);
        if (ld_acquire_sys(counter) >= target) return true;
        if ((it & 63) == 0) {
            if (*reinterpret_cast<volatile uint32_t *>(err) != kErrNone) return false;
            if (global_timer_ns() - t0 > kTpWaitLimitNs) {
                atomicCAS(err, kErrNone, kErrTimeoutPeer);
                return false;
            }
        }
    }
}

// One thread: this rank's partial (written by the kernels before this one on
// the stream) is complete; tell every rank.
__global__ void signal_ready_kernel(Args a) {
    __threadfence_system();
    for (int j = 0; j < a.world; ++j) red_add_release_sys(a.counters[j] + kReady, 1);
}

// Orders this thread's generic-proxy accesses (the acquire of a counter)
// before its later async-proxy accesses of global memory (bulk copies, TMA).
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// One thread: wait until every rank has stored its normalised rows here (the
// next kernel reads them, also through TMA).
__global__ void wait_done_kernel(Args a) {
    wait_counter(a.counters[a.rank] + kDone, a.epoch * (uint64_t)a.world, a.err);
    fence_proxy_async_global();
}

template <int VPL, bool REDUCE, bool NORM>
__global__ void __launch_bounds__(kWarps * 32) reduce_norm_gather_kernel(Args a) {
    constexpr int H = VPL * 8 * 32;
    const int lane = threadIdx.x & 31;
    __shared__ int s_ok;
    if (threadIdx.x == 0) {
        bool ok = true;
        if constexpr (REDUCE) ok = wait_counter(a.counters[a.rank] + kReady, a.epoch * (uint64_t)a.world, a.err);
        s_ok = ok ? 1 : 0;
    }
    __syncthreads();
    const int64_t row = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
    if (s_ok && row < a.rows) {
        const int s = row >= a.split ? 1 : 0;
        const int64_t grow = (int64_t)a.rank * a.rows + row;  // the token's row in part / gathered
        if constexpr (REDUCE) (void)ld_acquire_sys(a.counters[a.rank] + kReady);  // this warp's acquire
        uint4 *xr = reinterpret_cast<uint4 *>(a.x + row * H);
        uint32_t xv[VPL][4];
        if constexpr (REDUCE) {
            float acc[VPL][8];
#pragma unroll
            for (int i = 0; i < VPL; ++i)
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[i][e] = 0.0f;
            for (int j = 0; j < a.world; ++j) {
                const uint4 *pr = reinterpret_cast<const uint4 *>(a.part[j] + grow * H);
#pragma unroll
                for (int i = 0; i < VPL; ++i) {
                    const uint4 v = pr[i * 32 + lane];
                    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        acc[i][2 * q] += __uint_as_float(w[q] << 16);
                        acc[i][2 * q + 1] += __uint_as_float(w[q] & 0xFFFF0000u);
                    }
                }
            }
            const uint4 *b4 = reinterpret_cast<const uint4 *>(a.bias[s]);
            const uint4 *g4 = reinterpret_cast<const uint4 *>(a.gate[s]);
#pragma unroll
            for (int i = 0; i < VPL; ++i) {
                const uint4 v = xr[i * 32 + lane];
                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
                uint4 bv = make_uint4(0, 0, 0, 0), gv = make_uint4(0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u);
                if (b4) bv = __ldg(b4 + i * 32 + lane);
                if (b4 && g4) gv = __ldg(g4 + i * 32 + lane);
                const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w}, gw[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    float lo = __uint_as_float(w[q] << 16) + acc[i][2 * q];
                    float hi = __uint_as_float(w[q] & 0xFFFF0000u) + acc[i][2 * q + 1];
                    lo += __uint_as_float(bw[q] << 16) * __uint_as_float(gw[q] << 16);
                    hi += __uint_as_float(bw[q] & 0xFFFF0000u) * __uint_as_float(gw[q] & 0xFFFF0000u);
                    xv[i][q] = pack_bf16x2_rn(lo, hi);
                }
                xr[i * 32 + lane] = make_uint4(xv[i][0], xv[i][1], xv[i][2], xv[i][3]);
            }
        } else {
#pragma unroll
            for (int i = 0; i < VPL; ++i) {
                const uint4 v = xr[i * 32 + lane];
                xv[i][0] = v.x;
                xv[i][1] = v.y;
                xv[i][2] = v.z;
                xv[i][3] = v.w;
            }
        }
        if constexpr (NORM) {
            float sum = 0.0f;
#pragma unroll
            for (int i = 0; i < VPL; ++i)
#pragma unroll
                for (int q = 0; q < 4; ++q) sum += __uint_as_float(xv[i][q] << 16) + __uint_as_float(xv[i][q] & 0xFFFF0000u);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
            const float mean = sum * (1.0f / H);
            float sq = 0.0f;
#pragma unroll
            for (int i = 0; i < VPL; ++i)
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float lo = __uint_as_float(xv[i][q] << 16) - mean;
                    const float hi = __uint_as_float(xv[i][q] & 0xFFFF0000u) - mean;
                    sq = fmaf(lo, lo, fmaf(hi, hi, sq));
                }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, off);
            const float rstd = rsqrtf(sq * (1.0f / H) + a.eps);
            const uint4 *sh4 = reinterpret_cast<const uint4 *>(a.shift[s]);
            const uint4 *sc4 = reinterpret_cast<const uint4 *>(a.scale[s]);
#pragma unroll
            for (int i = 0; i < VPL; ++i) {
                const uint4 c4 = __ldg(sc4 + i * 32 + lane), h4 = __ldg(sh4 + i * 32 + lane);
                const uint32_t cw[4] = {c4.x, c4.y, c4.z, c4.w}, hw[4] = {h4.x, h4.y, h4.z, h4.w};
                uint32_t o[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float lo = (__uint_as_float(xv[i][q] << 16) - mean) * rstd;
                    const float hi = (__uint_as_float(xv[i][q] & 0xFFFF0000u) - mean) * rstd;
                    o[q] = pack_bf16x2_rn(fmaf(lo, 1.0f + __uint_as_float(cw[q] << 16), __uint_as_float(hw[q] << 16)),
                                          fmaf(hi, 1.0f + __uint_as_float(cw[q] & 0xFFFF0000u),
                                               __uint_as_float(hw[q] & 0xFFFF0000u)));
                }
                const uint4 ov = make_uint4(o[0], o[1], o[2], o[3]);
                for (int j = 0; j < a.world; ++j)
                    reinterpret_cast<uint4 *>(a.gathered[j] + grow * H)[i * 32 + lane] = ov;
            }
        }
    }
    // Done: the last CTA of this rank tells every rank, after every CTA's
    // stores (peer stores included) are visible system-wide.
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        uint64_t *local = a.counters[a.rank] + kLocal;
        const unsigned long long old = atomicAdd(reinterpret_cast<unsigned long long *>(local), 1ull);
        if (old + 1 == gridDim.x) {
            *local = 0;  // no other CTA of this launch touches it again; the next launch follows this one
            __threadfence_system();
            for (int j = 0; j < a.world; ++j) red_add_release_sys(a.counters[j] + kDone, 1);
        }
    }
}

// The residual update and norm of one row, and the stores of the normalised
// row into every rank's `gathered`, from the row's f32 sum of partials
// `acc` (lane's elements, VPL groups of 8).  BULK: the normalised row goes to
// the warp's shared-memory row `out` instead, for the caller's bulk stores.
template <int VPL, bool NORM, bool BULK = false>
__device__ __forceinline__ void finish_row(const Args &a, int64_t row, int lane, float (&acc)[VPL][8],
                                           uint4 *out = nullptr) {
    constexpr int H = VPL * 8 * 32;
    const int s = row >= a.split ? 1 : 0;
    const int64_t grow = (int64_t)a.rank * a.rows + row;
    uint4 *xr = reinterpret_cast<uint4 *>(a.x + row * H);
    const uint4 *b4 = reinterpret_cast<const uint4 *>(a.bias[s]);
    const uint4 *g4 = reinterpret_cast<const uint4 *>(a.gate[s]);
    uint32_t xv[VPL][4];
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const uint4 v = xr[i * 32 + lane];
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint4 bv = make_uint4(0, 0, 0, 0), gv = make_uint4(0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u);
        if (b4) bv = __ldg(b4 + i * 32 + lane);
        if (b4 && g4) gv = __ldg(g4 + i * 32 + lane);
        const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w}, gw[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            float lo = __uint_as_float(w[q] << 16) + acc[i][2 * q];
            float hi = __uint_as_float(w[q] & 0xFFFF0000u) + acc[i][2 * q + 1];
            lo += __uint_as_float(bw[q] << 16) * __uint_as_float(gw[q] << 16);
            hi += __uint_as_float(bw[q] & 0xFFFF0000u) * __uint_as_float(gw[q] & 0xFFFF0000u);
            xv[i][q] = pack_bf16x2_rn(lo, hi);
        }
        xr[i * 32 + lane] = make_uint4(xv[i][0], xv[i][1], xv[i][2], xv[i][3]);
    }
    if constexpr (NORM) {
        float sum = 0.0f;
#pragma unroll
        for (int i = 0; i < VPL; ++i)
#pragma unroll
            for (int q = 0; q < 4; ++q) sum += __uint_as_float(xv[i][q] << 16) + __uint_as_float(xv[i][q] & 0xFFFF0000u);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
        const float mean = sum * (1.0f / H);
        float sq = 0.0f;
#pragma unroll
        for (int i = 0; i < VPL; ++i)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float lo = __uint_as_float(xv[i][q] << 16) - mean;
                const float hi = __uint_as_float(xv[i][q] & 0xFFFF0000u) - mean;
                sq = fmaf(lo, lo, fmaf(hi, hi, sq));
            }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, off);
        const float rstd = rsqrtf(sq * (1.0f / H) + a.eps);
        const uint4 *sh4 = reinterpret_cast<const uint4 *>(a.shift[s]);
        const uint4 *sc4 = reinterpret_cast<const uint4 *>(a.scale[s]);
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
            const uint4 c4 = __ldg(sc4 + i * 32 + lane), h4 = __ldg(sh4 + i * 32 + lane);
            const uint32_t cw[4] = {c4.x, c4.y, c4.z, c4.w}, hw[4] = {h4.x, h4.y, h4.z, h4.w};
            uint32_t o[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float lo = (__uint_as_float(xv[i][q] << 16) - mean) * rstd;
                const float hi = (__uint_as_float(xv[i][q] & 0xFFFF0000u) - mean) * rstd;
                o[q] = pack_bf16x2_rn(fmaf(lo, 1.0f + __uint_as_float(cw[q] << 16), __uint_as_float(hw[q] << 16)),
                                      fmaf(hi, 1.0f + __uint_as_float(cw[q] & 0xFFFF0000u),
                                           __uint_as_float(hw[q] & 0xFFFF0000u)));
            }
            const uint4 ov = make_uint4(o[0], o[1], o[2], o[3]);
            if constexpr (BULK) {
                out[i * 32 + lane] = ov;
            } else {
                for (int j = 0; j < a.world; ++j)
                    reinterpret_cast<uint4 *>(a.gathered[j] + grow * H)[i * 32 + lane] = ov;
            }
        }
    }
}

// Shared memory of the pipelined kernel: the ring (S stages of world rows),
// its full / empty barriers, then (bulk stores) one output row per consumer warp.
__host__ __device__ constexpr size_t out_offset(int S, size_t stage_bytes) {
    return ((size_t)S * stage_bytes + 2 * (size_t)S * 8 + 127) & ~(size_t)127;
}

// Pipelined reduce (+ norm + gather): a persistent grid of one CTA per SM.
// Warp 0's lane 0 bulk-copies, for each row this CTA owns (rows c, c + grid,
// ...), the row's slice of every rank's `part` into one stage of a shared-
// memory ring (world * hidden * 2 bytes per stage; copies from peer memory,
// no multicast).  Consumer warp w (of NW) takes the CTA's rows i with
// i % NW == w; stage = i % stages, and stages is a multiple of NW, so each
// stage has one consumer, which takes its phases in order.  The ring keeps
// up to ~190 KB per SM in flight over NVLink, where register loads kept a
// quarter of that.
//
// BULK (with NORM; the default): each consumer warp writes its normalised row into its own
// shared-memory row and lane 0 hands it to the copy engine as one bulk store
// per rank (6 KB at hidden 3072) instead of every lane storing 16 bytes per
// rank; the warp waits for those stores to have read the row before it
// writes the next one, and for them to complete before the CTA signals.
template <int VPL, bool NORM, bool BULK = false>
__global__ void __launch_bounds__(32 * 9, 1) reduce_pipelined_kernel(Args a) {
    constexpr int H = VPL * 8 * 32;
    constexpr int kRowBytes = H * 2;
    extern __shared__ __align__(128) uint8_t smem[];
    const int S = a.stages;
    const int NW = S < 8 ? S : 8;  // consumer warps
    const uint32_t stage_bytes = (uint32_t)a.world * kRowBytes;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)S * stage_bytes);
    uint64_t *empty = full + S;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        fence_barrier_init();
    }
    __syncthreads();
    const int64_t nrows = a.rows <= blockIdx.x ? 0 : (a.rows - 1 - blockIdx.x) / gridDim.x + 1;  // this CTA's rows
    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            bool ok = wait_counter(a.counters[a.rank] + kReady, a.epoch * (uint64_t)a.world, a.err);
            fence_proxy_async_global();  // the bulk copies below read what the acquire made visible
            int64_t i = 0;
            for (; ok && i < nrows; ++i) {
                const int s = (int)(i % S);
                if (i >= S && !mbar_wait(&empty[s], (uint32_t)(((i / S) - 1) & 1), a.err, kErrTimeoutPeer)) {
                    ok = false;
                    break;
                }
                const int64_t grow = (int64_t)a.rank * a.rows + (int64_t)blockIdx.x + i * gridDim.x;
                mbar_arrive_expect_tx(&full[s], stage_bytes);
                uint8_t *dst = smem + (size_t)s * stage_bytes;
                for (int j = 0; j < a.world; ++j)
                    bulk_load(dst + (size_t)j * kRowBytes, a.part[j] + grow * H, kRowBytes, &full[s]);
            }
            // Let the copies issued land before the CTA exits (the consumers
            // wait for every stage they take; after an error, wait here).
            if (!ok)
                for (int64_t k = i > S ? i - S : 0; k < i; ++k)
                    mbar_wait(&full[k % S], (uint32_t)((k / S) & 1), a.err, kErrTimeoutPeer);
        }
    } else if (warp - 1 < NW) {
        // ------------------------------------------------------------ consumers
        const int c = warp - 1;
        constexpr bool kBulk = BULK && NORM;
        uint4 *outb = nullptr;
        if constexpr (kBulk)
            outb = reinterpret_cast<uint4 *>(smem + out_offset(S, stage_bytes) + (size_t)c * kRowBytes);
        bool ok = true;
        for (int64_t i = c; ok && i < nrows; i += NW) {
            const int s = (int)(i % S);
            ok = mbar_wait(&full[s], (uint32_t)((i / S) & 1), a.err, kErrTimeoutPeer);
            if (!ok) break;
            const uint8_t *st = smem + (size_t)s * stage_bytes;
            float acc[VPL][8];
#pragma unroll
            for (int v = 0; v < VPL; ++v)
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[v][e] = 0.0f;
            for (int j = 0; j < a.world; ++j) {
                const uint4 *pr = reinterpret_cast<const uint4 *>(st + (size_t)j * kRowBytes);
#pragma unroll
                for (int v = 0; v < VPL; ++v) {
                    const uint4 u = pr[v * 32 + lane];
                    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        acc[v][2 * q] += __uint_as_float(w[q] << 16);
                        acc[v][2 * q + 1] += __uint_as_float(w[q] & 0xFFFF0000u);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);  // the stage's data is in registers
            const int64_t row = (int64_t)blockIdx.x + i * gridDim.x;
            if constexpr (kBulk) {
                if (lane == 0) bulk_wait_read<0>();  // the previous row's stores have read `outb`
                __syncwarp();
            }
            finish_row<VPL, NORM, kBulk>(a, row, lane, acc, outb);
            if constexpr (kBulk) {
                fence_proxy_async_smem();  // this lane's row elements before the copy engine reads them
                __syncwarp();
                if (lane == 0) {
                    const int64_t grow = (int64_t)a.rank * a.rows + row;
                    for (int j = 0; j < a.world; ++j) bulk_store(a.gathered[j] + grow * H, outb, kRowBytes);
                    bulk_commit();
                }
            }
        }
        if constexpr (kBulk) {
            if (lane == 0) {
                bulk_wait_all();             // the rows have landed in every rank's `gathered`
                fence_proxy_async_global();  // before the generic-proxy release below
            }
        }
    }
    // Done: as in reduce_norm_gather_kernel.
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        uint64_t *local = a.counters[a.rank] + kLocal;
        const unsigned long long old = atomicAdd(reinterpret_cast<unsigned long long *>(local), 1ull);
        if (old + 1 == gridDim.x) {
            *local = 0;
            __threadfence_system();
            for (int j = 0; j < a.world; ++j) red_add_release_sys(a.counters[j] + kDone, 1);
        }
    }
}

// Bulk stores of the normalised rows (the default; measured at 2 ranks: 178
// vs 188 us per exchange at hidden 3072) or, with QMM_TP_BULK_STORE=0,
// per-lane 16-byte stores.
static bool bulk_store_rows() {
    static const bool on = [] {
        const char *e = std::getenv("QMM_TP_BULK_STORE");
        return !(e && e[0] == '0');
    }();
    return on;
}

template <int VPL>
static qmm_status launch_pipelined(cudaStream_t st, Args &a, bool norm) {
    const size_t row = (size_t)VPL * 8 * 32 * 2;
    const size_t stage = (size_t)a.world * row;
    const bool bulk = norm && bulk_store_rows();
    int S = 0;
    size_t smem = 0;
    if (!bulk) {
        constexpr size_t kBudget = 200 * 1024;
        S = 16;
        while (S > 2 && (size_t)S * stage > kBudget) S >>= 1;
        if ((size_t)S * stage > kBudget) return fail(QMM_ERR_UNSUPPORTED, "tp: a row of every rank does not fit the ring");
        smem = (size_t)S * stage + 2 * (size_t)S * 8;
    } else {
        // Ring plus one output row per consumer warp (min(S, 8) of them); S is
        // at most 8 or 16 so that every stage has one consumer.
        constexpr size_t kLimit = 225 * 1024;
        static const int kCand[] = {16, 8, 7, 6, 5, 4, 3, 2};
        for (int cand : kCand) {
            const size_t need = out_offset(cand, stage) + (size_t)(cand < 8 ? cand : 8) * row;
            if (need <= kLimit) {
                S = cand;
                smem = need;
                break;
            }
        }
        if (!S) return fail(QMM_ERR_UNSUPPORTED, "tp: two rows of every rank do not fit the ring");
    }
    a.stages = S;
    auto kernel = !norm ? reduce_pipelined_kernel<VPL, false>
                        : (bulk ? reduce_pipelined_kernel<VPL, true, true> : reduce_pipelined_kernel<VPL, true>);
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_fail(e, "tp smem attribute");
    const unsigned grid = (unsigned)std::min<int64_t>(a.rows, sm_count());
    kernel<<<grid, 32 * 9, smem, st>>>(a);
    return QMM_OK;
}

template <int VPL>
static void launch_rng(unsigned grid, cudaStream_t st, const Args &a, bool reduce, bool norm) {
    const int kT = kWarps * 32;
    if (reduce && norm) reduce_norm_gather_kernel<VPL, true, true><<<grid, kT, 0, st>>>(a);
    else if (reduce) reduce_norm_gather_kernel<VPL, true, false><<<grid, kT, 0, st>>>(a);
    else reduce_norm_gather_kernel<VPL, false, true><<<grid, kT, 0, st>>>(a);
}

static qmm_status make_args(const qmm_tp_peers *p, Args &a) {
    if (!p) return fail(QMM_ERR_INVALID_ARGUMENT, "tp: null peer set");
    if (p->world < 1 || p->world > QMM_TP_MAX_RANKS || p->rank < 0 || p->rank >= p->world)
        return fail(QMM_ERR_INVALID_ARGUMENT, "tp: rank %d of %d (at most %d ranks)", p->rank, p->world,
                    QMM_TP_MAX_RANKS);
    a = Args{};
    a.world = p->world;
    a.rank = p->rank;
    for (int j = 0; j < p->world; ++j) {
        if (!p->part[j] || !p->gathered[j] || !p->counters[j])
            return fail(QMM_ERR_INVALID_ARGUMENT, "tp: rank %d's buffers are missing", j);
        const uintptr_t al = reinterpret_cast<uintptr_t>(p->part[j]) | reinterpret_cast<uintptr_t>(p->gathered[j]) |
                             reinterpret_cast<uintptr_t>(p->counters[j]);
        if (al & 15u) return fail(QMM_ERR_MISALIGNED, "tp: rank %d's buffers are not 16-byte aligned", j);
        a.part[j] = p->part[j];
        a.gathered[j] = p->gathered[j];
        a.counters[j] = p->counters[j];
    }
    a.err = device_error_word();
    return QMM_OK;
}

}  // namespace tp
}  // namespace qmm

extern "C" {

qmm_status qmm_tp_signal_ready(const qmm_tp_peers *peers, void *stream) {
    qmm::tp::Args a;
    qmm_status s = qmm::tp::make_args(peers, a);
    if (s != QMM_OK) return s;
    qmm::tp::signal_ready_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(a);
    qmm::count_launch();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? QMM_OK : qmm::cuda_fail(e, "tp signal launch");
}

qmm_status qmm_tp_wait_gathered(const qmm_tp_peers *peers, uint64_t epoch, void *stream) {
    qmm::tp::Args a;
    qmm_status s = qmm::tp::make_args(peers, a);
    if (s != QMM_OK) return s;
    if (epoch == 0) return qmm::fail(QMM_ERR_INVALID_ARGUMENT, "tp: epochs start at 1");
    a.epoch = epoch;
    qmm::tp::wait_done_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(a);
    qmm::count_launch();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? QMM_OK : qmm::cuda_fail(e, "tp wait launch");
}

qmm_status qmm_tp_reduce_norm_gather(const qmm_tp_peers *peers, uint64_t epoch, int64_t rows, int64_t hidden,
                                     uint16_t *x, const qmm_tp_norm *nrm, int32_t reduce, int32_t normalize,
                                     void *stream) {
    using qmm::fail;
    qmm::tp::Args a;
    qmm_status s = qmm::tp::make_args(peers, a);
    if (s != QMM_OK) return s;
    if (epoch == 0) return fail(QMM_ERR_INVALID_ARGUMENT, "tp: epochs start at 1");
    if (!nrm || !x) return fail(QMM_ERR_INVALID_ARGUMENT, "tp: null x or norm arguments");
    if (rows <= 0 || hidden <= 0) return fail(QMM_ERR_BAD_SHAPE, "tp: %lld rows of %lld", (long long)rows, (long long)hidden);
    if (!reduce && !normalize) return fail(QMM_ERR_INVALID_ARGUMENT, "tp: nothing to do");
    if (nrm->split < 0 || nrm->split > rows) return fail(QMM_ERR_BAD_SHAPE, "tp: stream split %lld of %lld rows",
                                                      (long long)nrm->split, (long long)rows);
    uintptr_t al = reinterpret_cast<uintptr_t>(x);
    for (int t = 0; t < 2; ++t) {
        const bool used = t == 0 ? nrm->split > 0 : nrm->split < rows;
        if (!used) continue;
        if (normalize && (!nrm->shift[t] || !nrm->scale[t]))
            return fail(QMM_ERR_INVALID_ARGUMENT, "tp: stream %d needs shift and scale", t);
        if (nrm->gate[t] && !nrm->bias[t])
            return fail(QMM_ERR_INVALID_ARGUMENT, "tp: stream %d's gate multiplies its bias; no bias given", t);
        al |= reinterpret_cast<uintptr_t>(nrm->bias[t]) | reinterpret_cast<uintptr_t>(nrm->gate[t]) |
              reinterpret_cast<uintptr_t>(nrm->shift[t]) | reinterpret_cast<uintptr_t>(nrm->scale[t]);
    }
    if (al & 15u) return fail(QMM_ERR_MISALIGNED, "tp: x and the per-feature vectors must be 16-byte aligned");
    a.epoch = epoch;
    a.rows = rows;
    a.split = nrm->split;
    a.x = x;
    for (int t = 0; t < 2; ++t) {
        a.bias[t] = nrm->bias[t];
        a.gate[t] = nrm->gate[t];
        a.shift[t] = nrm->shift[t];
        a.scale[t] = nrm->scale[t];
    }
    a.eps = nrm->eps;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const unsigned grid = (unsigned)((rows + qmm::tp::kWarps - 1) / qmm::tp::kWarps);
    const int vpl = (int)(hidden / 256) * (hidden % 256 == 0 ? 1 : 0);
    if (vpl != 1 && vpl != 2 && vpl != 4 && vpl != 12 && vpl != 16)
        return fail(QMM_ERR_UNSUPPORTED, "tp: hidden %lld is not 256, 512, 1024, 3072 or 4096", (long long)hidden);
    if (reduce) {
        // The reduction streams every rank's rows through the pipelined kernel.
        switch (vpl) {
            case 1: s = qmm::tp::launch_pipelined<1>(st, a, normalize); break;
            case 2: s = qmm::tp::launch_pipelined<2>(st, a, normalize); break;
            case 4: s = qmm::tp::launch_pipelined<4>(st, a, normalize); break;
            case 12: s = qmm::tp::launch_pipelined<12>(st, a, normalize); break;
            default: s = qmm::tp::launch_pipelined<16>(st, a, normalize); break;
        }
        if (s != QMM_OK) return s;
    } else {
        switch (vpl) {
            case 1: qmm::tp::launch_rng<1>(grid, st, a, reduce, normalize); break;
            case 2: qmm::tp::launch_rng<2>(grid, st, a, reduce, normalize); break;
            case 4: qmm::tp::launch_rng<4>(grid, st, a, reduce, normalize); break;
            case 12: qmm::tp::launch_rng<12>(grid, st, a, reduce, normalize); break;
            default: qmm::tp::launch_rng<16>(grid, st, a, reduce, normalize); break;
        }
    }
    qmm::count_launch();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? QMM_OK : qmm::cuda_fail(e, "tp reduce/norm/gather launch");
}

}  // extern "C"
