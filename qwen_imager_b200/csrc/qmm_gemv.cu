// Dequantize kernel and the small-m (GEMV) quantized linear.
//
// qmm_dequantize_kernel: dense W [n, k] from packed codes, bit-exact with
//   image-forger src/quant.rs:555-573 (Dequantize::cpu_fwd) and the Metal
//   `dequantize` kernel (src/quant.rs:186-206).  One thread per packed word:
//   adjacent threads read adjacent words and write adjacent outputs.
//
// qmm_gemv_kernel: y [m, n] for m <= 16 (the adaLN modulation linear runs at
//   m = 1).  HBM-bound: each weight byte is read once.  A warp owns R rows; its
//   lanes stream the rows' packed words with 128-bit loads (one 16-byte chunk
//   = 32 4-bit / 16 8-bit / 64 2-bit codes, all in one scale group), dot them
//   against x staged in shared memory as f32, and reduce with shuffles.
//   Per chunk it uses  sum_k x_k (s q_k + o) = s * sum_k x_k q_k + o * sum_k x_k
//   with the per-chunk sums of x precomputed once per block.
#include <algorithm>

#include "qmm_epilogue.cuh"
#include "qmm_internal.h"
#include "qmm_unpack.cuh"

namespace qmm {

// ------------------------------------------------------------------ dequantize
template <int BITS, bool F32OUT>
__global__ void __launch_bounds__(256) qmm_dequantize_kernel(const uint32_t *__restrict__ packed,
                                                             const uint16_t *__restrict__ scales,
                                                             const uint16_t *__restrict__ offsets,
                                                             int64_t n, int64_t k, int32_t group,
                                                             void *__restrict__ dst) {
    constexpr int C = WordCodes<BITS>::kCount;
    const int64_t words = k / C;
    const int64_t groups = k / group;
    const int64_t total = n * words;
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = idx / words;
        const int64_t col0 = (idx - row * words) * C;
        const uint32_t w = __ldg(packed + idx);
        float q[C];
        WordCodes<BITS>::unpack(w, q);
        float v[C];
#pragma unroll
        for (int j = 0; j < C; ++j) {
            const int64_t g = row * groups + (int32_t)(col0 + j) / group;
            const float s = bf16_bits_to_f32(__ldg(scales + g));
            const float o = bf16_bits_to_f32(__ldg(offsets + g));
            v[j] = fmaf(q[j], s, o);
        }
        if constexpr (F32OUT) {
            float4 *out = reinterpret_cast<float4 *>(static_cast<float *>(dst) + row * k + col0);
#pragma unroll
            for (int j = 0; j < C / 4; ++j)
                out[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        } else {
            uint32_t pk[C / 2];
#pragma unroll
            for (int j = 0; j < C / 2; ++j) pk[j] = pack_bf16x2_rn(v[2 * j], v[2 * j + 1]);
            uint16_t *out = static_cast<uint16_t *>(dst) + row * k + col0;
            if constexpr (C == 4) {
                *reinterpret_cast<uint2 *>(out) = make_uint2(pk[0], pk[1]);
            } else {
#pragma unroll
                for (int j = 0; j < C / 8; ++j)
                    reinterpret_cast<uint4 *>(out)[j] =
                        make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
            }
        }
    }
}

qmm_status launch_dequantize(const qmm_weight &w, void *dst, int32_t dtype, cudaStream_t st) {
    const int per_word = 32 / w.bits;
    const int64_t total = w.n * (w.k / per_word);
    if (total == 0) return QMM_OK;
    const int threads = 256;
    const int64_t want = (total + threads - 1) / threads;
    const int blocks = static_cast<int>(std::min<int64_t>(want, (int64_t)sm_count() * 16));
    const bool f32 = dtype == QMM_DTYPE_F32;
#define QMM_DQ_CASE(B)                                                                          \
    if (w.bits == B) {                                                                          \
        if (f32)                                                                                \
            qmm_dequantize_kernel<B, true><<<blocks, threads, 0, st>>>(w.packed, w.scales,      \
                                                                       w.biases, w.n, w.k,      \
                                                                       w.group, dst);           \
        else                                                                                    \
            qmm_dequantize_kernel<B, false><<<blocks, threads, 0, st>>>(w.packed, w.scales,     \
                                                                        w.biases, w.n, w.k,     \
                                                                        w.group, dst);          \
    }
    QMM_DQ_CASE(2)
    QMM_DQ_CASE(4)
    QMM_DQ_CASE(8)
#undef QMM_DQ_CASE
    count_launch();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? QMM_OK : cuda_fail(e, "dequantize launch");
}

// ------------------------------------------------------------------ GEMV
constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr size_t kGemvMaxSmem = 200 * 1024;

// Rows per warp task and 16-byte chunks in flight per lane and row: enough
// loads in flight to cover HBM latency at m = 1, fewer registers as m grows.
template <int MT>
struct GemvShape {
    static constexpr int kRows = MT <= 2 ? 2 : 1;
    static constexpr int kUnroll = MT == 1 ? 4 : (MT <= 4 ? 2 : 1);
};

__device__ __forceinline__ uint4 ld_stream_u4(const uint4 *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

struct GemvParams {
    const uint16_t *x;
    const uint32_t *packed;
    const uint16_t *scales;
    const uint16_t *offsets;
    uint16_t *y;
    EpilogueArgs ep;
    int64_t n;
    int32_t k;
    int32_t m;
    int32_t group;
    int32_t cpg_shift;  // log2(group / codes per 16-byte chunk)
};

// Sum over one 16-byte chunk of codes of x_k * f(q_k) for every token, where
// f is the float the code unpacks to.  4-bit codes unpack to 2 + q/64 (one
// byte permute: exponent byte 0x40, code in the mantissa's top byte, exact),
// so sum_k x_k q_k = 64 * S - 128 * X with X = sum_k x_k; 2- and 8-bit codes
// unpack to q exactly (the 2^23 + q trick), so the sum is S itself.
template <int BITS>
struct ChunkAffine {
    static constexpr float kMul = BITS == 4 ? 64.0f : 1.0f;   // sum x q = kMul * S + kAdd * X
    static constexpr float kAdd = BITS == 4 ? -128.0f : 0.0f;
};

// Shared memory: xs[k][MP] (token-minor f32, MP = MT rounded up to a multiple
// of 4 for vector loads; MP = 1 when MT = 1), then xsum[nchunks][MT].
template <int MT>
struct GemvPad {
    static constexpr int kMP = MT == 1 ? 1 : (MT + 3) / 4 * 4;
};

template <int I>
__device__ __forceinline__ float two_plus_q_over_64(uint32_t v) {
    // bytes: [0x00, 0x00, v.b[I], 0x40]  ->  2 * (1 + q * 2^-7)
    return __uint_as_float(__byte_perm(v, 0x40000000u, 0x7044u | (I << 8)));
}

template <int BITS, int MT>
__device__ __forceinline__ void chunk_dot(const uint4 &w, const float *__restrict__ xc, float (&dot)[MT]) {
    constexpr int CPW = 32 / BITS;
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
#pragma unroll
            for (int j = 0; j < CPW; j += 4) {
                const float4 xv = *reinterpret_cast<const float4 *>(xc + wi * CPW + j);
                dot[0] = fmaf(xv.x, q[j], dot[0]);
                dot[0] = fmaf(xv.y, q[j + 1], dot[0]);
                dot[0] = fmaf(xv.z, q[j + 2], dot[0]);
                dot[0] = fmaf(xv.w, q[j + 3], dot[0]);
            }
        } else {
#pragma unroll
            for (int j = 0; j < CPW; ++j) {
                const float *xk = xc + (wi * CPW + j) * GemvPad<MT>::kMP;
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

template <int BITS, int MT>
__global__ void __launch_bounds__(kGemvThreads) qmm_gemv_kernel(GemvParams p) {
    constexpr int CPC = 128 / BITS;  // codes per 16-byte chunk
    constexpr int MP = GemvPad<MT>::kMP;
    extern __shared__ __align__(16) float gemv_smem[];
    const int k = p.k;
    const int nchunks = k / CPC;
    float *xs = gemv_smem;
    float *xsum = gemv_smem + (size_t)k * MP;

    // Stage x as f32 (tokens >= m read as zero), 8 bf16 per load.
    for (int i = threadIdx.x; i < (k / 8) * MP; i += kGemvThreads) {
        const int t = i % MP, k8 = (i / MP) * 8;
        float v[8];
        if (t < p.m) {
            const uint4 raw = __ldg(reinterpret_cast<const uint4 *>(p.x + (size_t)t * k + k8));
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
        for (int j = 0; j < 8; ++j) xs[(size_t)(k8 + j) * MP + t] = v[j];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < nchunks * MT; i += kGemvThreads) {
        const int c = i / MT, t = i - c * MT;
        float sum = 0.0f;
        for (int j = 0; j < CPC; ++j) sum += xs[(size_t)(c * CPC + j) * MP + t];
        xsum[i] = sum;
    }
    __syncthreads();

    constexpr int kGemvRows = GemvShape<MT>::kRows;
    constexpr int kGemvUnroll = GemvShape<MT>::kUnroll;
    constexpr float kMul = ChunkAffine<BITS>::kMul, kAdd = ChunkAffine<BITS>::kAdd;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int groups = k / p.group;
    const int cpg_shift = p.cpg_shift;  // log2(chunks per group)
    const int64_t ntasks = (p.n + kGemvRows - 1) / kGemvRows;
    const uint4 *packed4 = reinterpret_cast<const uint4 *>(p.packed);

    for (int64_t task = (int64_t)blockIdx.x * kGemvWarps + warp; task < ntasks;
         task += (int64_t)gridDim.x * kGemvWarps) {
        const int64_t row0 = task * kGemvRows;
        float acc[kGemvRows][MT];
#pragma unroll
        for (int r = 0; r < kGemvRows; ++r)
#pragma unroll
            for (int t = 0; t < MT; ++t) acc[r][t] = 0.0f;

        for (int cb = 0; cb < nchunks; cb += 32 * kGemvUnroll) {
            uint4 wv[kGemvRows][kGemvUnroll];
            float sc[kGemvRows][kGemvUnroll], of[kGemvRows][kGemvUnroll];
#pragma unroll
            for (int r = 0; r < kGemvRows; ++r) {
#pragma unroll
                for (int u = 0; u < kGemvUnroll; ++u) {
                    const int c = cb + u * 32 + lane;
                    const int64_t row = row0 + r;
                    const bool ok = c < nchunks && row < p.n;
                    wv[r][u] = ok ? ld_stream_u4(packed4 + row * nchunks + c) : make_uint4(0, 0, 0, 0);
                    const int64_t g = row * groups + (c >> cpg_shift);
                    sc[r][u] = ok ? bf16_bits_to_f32(__ldg(p.scales + g)) : 0.0f;
                    of[r][u] = ok ? bf16_bits_to_f32(__ldg(p.offsets + g)) : 0.0f;
                }
            }
#pragma unroll
            for (int u = 0; u < kGemvUnroll; ++u) {
                const int c = cb + u * 32 + lane;
                if (c >= nchunks) break;
                const float *xc = xs + (size_t)c * CPC * MP;
#pragma unroll
                for (int r = 0; r < kGemvRows; ++r) {
                    float dot[MT];
#pragma unroll
                    for (int t = 0; t < MT; ++t) dot[t] = 0.0f;
                    chunk_dot<BITS, MT>(wv[r][u], xc, dot);
                    const float a = sc[r][u] * kMul;
                    const float b = fmaf(sc[r][u], kAdd, of[r][u]);
#pragma unroll
                    for (int t = 0; t < MT; ++t)
                        acc[r][t] = fmaf(a, dot[t], fmaf(b, xsum[(size_t)c * MT + t], acc[r][t]));
                }
            }
        }
        // Warp reduction; lane t writes token t of each row.
#pragma unroll
        for (int r = 0; r < kGemvRows; ++r) {
#pragma unroll
            for (int t = 0; t < MT; ++t) {
                float v = acc[r][t];
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
                acc[r][t] = v;
            }
        }
#pragma unroll
        for (int r = 0; r < kGemvRows; ++r) {
            const int64_t row = row0 + r;
            if (row >= p.n) break;
            const FeatureConsts fc = load_feature_consts(p.ep, row, true);
#pragma unroll
            for (int t = 0; t < MT; ++t) {
                if (lane == t && t < p.m) {
                    const int64_t idx = (int64_t)t * p.n + row;
                    const float v =
                        epilogue_value(p.ep, fc, acc[r][t], p.ep.residual ? p.ep.residual + idx : nullptr);
                    p.y[idx] = f32_to_bf16_bits(v);
                }
            }
        }
    }
}

static int gemv_tile(int64_t m) {
    if (m <= 1) return 1;
    if (m <= 2) return 2;
    if (m <= 4) return 4;
    if (m <= 8) return 8;
    return 16;
}

static size_t gemv_smem_bytes(const qmm_weight &w, int mt) {
    const int cpc = 128 / w.bits;
    const int mp = mt == 1 ? 1 : (mt + 3) / 4 * 4;
    return ((size_t)w.k * mp + (size_t)(w.k / cpc) * mt) * sizeof(float);
}

static int log2_exact(int v) {
    int s = 0;
    while ((1 << s) < v) ++s;
    return (1 << s) == v ? s : -1;
}

bool gemv_supported(const qmm_weight &w, int64_t m) {
    if (m < 1 || m > 16) return false;
    if (w.bits != 2 && w.bits != 4 && w.bits != 8) return false;
    const int cpc = 128 / w.bits;
    if (w.k % cpc != 0 || w.group % cpc != 0) return false;
    if (log2_exact(w.group / cpc) < 0) return false;
    if (w.k > (1 << 30)) return false;
    return gemv_smem_bytes(w, gemv_tile(m)) <= kGemvMaxSmem;
}

template <int BITS, int MT>
static qmm_status launch_gemv_t(const GemvParams &p, size_t smem, cudaStream_t st) {
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(qmm_gemv_kernel<BITS, MT>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)kGemvMaxSmem);
        if (e != cudaSuccess) return cuda_fail(e, "gemv smem attribute");
        configured[dev] = true;
    }
    const int64_t ntasks = (p.n + GemvShape<MT>::kRows - 1) / GemvShape<MT>::kRows;
    const int64_t want = (ntasks + kGemvWarps - 1) / kGemvWarps;
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, qmm_gemv_kernel<BITS, MT>, kGemvThreads,
                                                  smem);
    if (per_sm < 1) per_sm = 1;
    const int blocks = (int)std::min<int64_t>(want, (int64_t)sm_count() * per_sm);
    qmm_gemv_kernel<BITS, MT><<<blocks, kGemvThreads, smem, st>>>(p);
    count_launch();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? QMM_OK : cuda_fail(e, "gemv launch");
}

qmm_status launch_gemv(const qmm_weight &w, const uint16_t *x, int64_t m, const qmm_epilogue &ep,
                       uint16_t *y, cudaStream_t st) {
    GemvParams p;
    p.x = x;
    p.packed = w.packed;
    p.scales = w.scales;
    p.offsets = w.biases;
    p.y = y;
    p.ep = epilogue_args(ep);
    p.n = w.n;
    p.k = (int32_t)w.k;
    p.m = (int32_t)m;
    p.group = w.group;
    p.cpg_shift = log2_exact(w.group / (128 / w.bits));
    const int mt = gemv_tile(m);
    const size_t smem = gemv_smem_bytes(w, mt);
#define QMM_GEMV_CASE(B, MT) \
    if (w.bits == B && mt == MT) return launch_gemv_t<B, MT>(p, smem, st);
#define QMM_GEMV_BITS(B)   \
    QMM_GEMV_CASE(B, 1)    \
    QMM_GEMV_CASE(B, 2)    \
    QMM_GEMV_CASE(B, 4)    \
    QMM_GEMV_CASE(B, 8)    \
    QMM_GEMV_CASE(B, 16)
    QMM_GEMV_BITS(2)
    QMM_GEMV_BITS(4)
    QMM_GEMV_BITS(8)
#undef QMM_GEMV_BITS
#undef QMM_GEMV_CASE
    return fail(QMM_ERR_UNSUPPORTED, "gemv: no kernel for %d-bit, m=%lld", w.bits, (long long)m);
}

}  // namespace qmm
