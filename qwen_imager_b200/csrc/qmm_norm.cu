// Fused LayerNorm (no affine) + adaLN modulation of the DiT block:
//   out = bf16( (x - mean) / sqrt(var + eps) * (1 + scale) + shift ),
// f32 arithmetic, one rounding.  The reference applies the same pattern with
// separate tensor ops before every attention and feed-forward input
// (image-forger src/dit.rs:50, 91: ops::norm(x) * (1 + modulation)).
// One warp per row; the row stays in registers (hidden <= 4096, a multiple of
// 256), so x is read once; mean and variance in two passes over registers.
#include "qmm_epilogue.cuh"
#include "qmm_internal.h"

namespace qmm {
namespace {

constexpr int kNormWarps = 8;

template <int VPL>  // 16-byte vectors (8 bf16) per lane
__global__ void __launch_bounds__(kNormWarps * 32) layernorm_modulate_kernel(
    const uint16_t *__restrict__ x, int64_t rows, const uint16_t *__restrict__ shift,
    const uint16_t *__restrict__ scale, float eps, uint16_t *__restrict__ out) {
    constexpr int H = VPL * 8 * 32;
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * kNormWarps + (threadIdx.x >> 5);
    if (row >= rows) return;
    const uint4 *xr = reinterpret_cast<const uint4 *>(x + row * H);
    uint4 v[VPL];
#pragma unroll
    for (int i = 0; i < VPL; ++i) v[i] = __ldg(xr + i * 32 + lane);
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
        for (int q = 0; q < 4; ++q) sum += __uint_as_float(w[q] << 16) + __uint_as_float(w[q] & 0xFFFF0000u);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    const float mean = sum * (1.0f / H);
    float sq = 0.0f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float a = __uint_as_float(w[q] << 16) - mean, b = __uint_as_float(w[q] & 0xFFFF0000u) - mean;
            sq = fmaf(a, a, fmaf(b, b, sq));
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, off);
    const float rstd = rsqrtf(sq * (1.0f / H) + eps);
    uint4 *orow = reinterpret_cast<uint4 *>(out + row * H);
    const uint4 *sh4 = reinterpret_cast<const uint4 *>(shift), *sc4 = reinterpret_cast<const uint4 *>(scale);
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const uint4 s4 = __ldg(sc4 + i * 32 + lane), h4 = __ldg(sh4 + i * 32 + lane);
        const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
        const uint32_t sw[4] = {s4.x, s4.y, s4.z, s4.w}, hw[4] = {h4.x, h4.y, h4.z, h4.w};
        uint32_t o[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float a = (__uint_as_float(w[q] << 16) - mean) * rstd;
            const float b = (__uint_as_float(w[q] & 0xFFFF0000u) - mean) * rstd;
            const float ra = fmaf(a, 1.0f + __uint_as_float(sw[q] << 16), __uint_as_float(hw[q] << 16));
            const float rb = fmaf(b, 1.0f + __uint_as_float(sw[q] & 0xFFFF0000u), __uint_as_float(hw[q] & 0xFFFF0000u));
            o[q] = pack_bf16x2_rn(ra, rb);
        }
        orow[i * 32 + lane] = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

// Residual update of the hidden state followed by the next LayerNorm +
// modulation, for the sequence-parallel DiT stack: x holds this rank's rows
// of the hidden state, delta the reduce-scattered sum of the ranks' gated
// row-parallel partials.  x = bf16(x + delta + gate * bias) in f32 (one
// rounding, like the GEMM epilogue's residual), then, when `out` is given,
// out = bf16(LN(x) * (1 + scale) + shift) of the rounded x.
template <int VPL, bool BIAS, bool GATE, bool NORM>
__global__ void __launch_bounds__(kNormWarps * 32) residual_layernorm_modulate_kernel(
    uint16_t *__restrict__ x, int64_t rows, const uint16_t *__restrict__ delta, const uint16_t *__restrict__ bias,
    const uint16_t *__restrict__ gate, const uint16_t *__restrict__ shift, const uint16_t *__restrict__ scale,
    float eps, uint16_t *__restrict__ out) {
    constexpr int H = VPL * 8 * 32;
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * kNormWarps + (threadIdx.x >> 5);
    if (row >= rows) return;
    uint4 *xr = reinterpret_cast<uint4 *>(x + row * H);
    const uint4 *dr = reinterpret_cast<const uint4 *>(delta + row * H);
    const uint4 *b4 = reinterpret_cast<const uint4 *>(bias), *g4 = reinterpret_cast<const uint4 *>(gate);
    uint4 v[VPL];
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const uint4 xv = xr[i * 32 + lane], dv = __ldg(dr + i * 32 + lane);
        uint4 bv = make_uint4(0, 0, 0, 0), gv = make_uint4(0, 0, 0, 0);
        if constexpr (BIAS) bv = __ldg(b4 + i * 32 + lane);
        if constexpr (BIAS && GATE) gv = __ldg(g4 + i * 32 + lane);
        const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w}, dw[4] = {dv.x, dv.y, dv.z, dv.w};
        const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w}, gw[4] = {gv.x, gv.y, gv.z, gv.w};
        uint32_t o[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            float lo = __uint_as_float(xw[q] << 16) + __uint_as_float(dw[q] << 16);
            float hi = __uint_as_float(xw[q] & 0xFFFF0000u) + __uint_as_float(dw[q] & 0xFFFF0000u);
            if constexpr (BIAS) {
                float blo = __uint_as_float(bw[q] << 16), bhi = __uint_as_float(bw[q] & 0xFFFF0000u);
                if constexpr (GATE) {
                    blo *= __uint_as_float(gw[q] << 16);
                    bhi *= __uint_as_float(gw[q] & 0xFFFF0000u);
                }
                lo += blo;
                hi += bhi;
            }
            o[q] = pack_bf16x2_rn(lo, hi);
            sum += __uint_as_float(o[q] << 16) + __uint_as_float(o[q] & 0xFFFF0000u);
        }
        v[i] = make_uint4(o[0], o[1], o[2], o[3]);
        xr[i * 32 + lane] = v[i];
    }
    if constexpr (NORM) {
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
        const float mean = sum * (1.0f / H);
        float sq = 0.0f;
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
            const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float a = __uint_as_float(w[q] << 16) - mean, b = __uint_as_float(w[q] & 0xFFFF0000u) - mean;
                sq = fmaf(a, a, fmaf(b, b, sq));
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, off);
        const float rstd = rsqrtf(sq * (1.0f / H) + eps);
        uint4 *orow = reinterpret_cast<uint4 *>(out + row * H);
        const uint4 *sh4 = reinterpret_cast<const uint4 *>(shift), *sc4 = reinterpret_cast<const uint4 *>(scale);
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
            const uint4 s4 = __ldg(sc4 + i * 32 + lane), h4 = __ldg(sh4 + i * 32 + lane);
            const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
            const uint32_t sw[4] = {s4.x, s4.y, s4.z, s4.w}, hw[4] = {h4.x, h4.y, h4.z, h4.w};
            uint32_t o[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float a = (__uint_as_float(w[q] << 16) - mean) * rstd;
                const float b = (__uint_as_float(w[q] & 0xFFFF0000u) - mean) * rstd;
                const float ra = fmaf(a, 1.0f + __uint_as_float(sw[q] << 16), __uint_as_float(hw[q] << 16));
                const float rb = fmaf(b, 1.0f + __uint_as_float(sw[q] & 0xFFFF0000u), __uint_as_float(hw[q] & 0xFFFF0000u));
                o[q] = pack_bf16x2_rn(ra, rb);
            }
            orow[i * 32 + lane] = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
}

template <int VPL>
void launch_residual_ln(unsigned grid, cudaStream_t st, uint16_t *x, int64_t rows, const uint16_t *delta,
                        const uint16_t *bias, const uint16_t *gate, const uint16_t *shift, const uint16_t *scale,
                        float eps, uint16_t *out) {
    constexpr int kT = kNormWarps * 32;
    const bool b = bias != nullptr, g = gate != nullptr, nrm = out != nullptr;
    if (b && g && nrm) residual_layernorm_modulate_kernel<VPL, true, true, true><<<grid, kT, 0, st>>>(x, rows, delta, bias, gate, shift, scale, eps, out);
    else if (b && g) residual_layernorm_modulate_kernel<VPL, true, true, false><<<grid, kT, 0, st>>>(x, rows, delta, bias, gate, shift, scale, eps, out);
    else if (b && nrm) residual_layernorm_modulate_kernel<VPL, true, false, true><<<grid, kT, 0, st>>>(x, rows, delta, bias, gate, shift, scale, eps, out);
    else if (b) residual_layernorm_modulate_kernel<VPL, true, false, false><<<grid, kT, 0, st>>>(x, rows, delta, bias, gate, shift, scale, eps, out);
    else if (nrm) residual_layernorm_modulate_kernel<VPL, false, false, true><<<grid, kT, 0, st>>>(x, rows, delta, bias, gate, shift, scale, eps, out);
    else residual_layernorm_modulate_kernel<VPL, false, false, false><<<grid, kT, 0, st>>>(x, rows, delta, bias, gate, shift, scale, eps, out);
}

}  // namespace
}  // namespace qmm

extern "C" {

qmm_status qmm_residual_layernorm_modulate(uint16_t *x, int64_t rows, int64_t hidden, const uint16_t *delta,
                                           const uint16_t *bias, const uint16_t *gate, const uint16_t *shift,
                                           const uint16_t *scale, float eps, uint16_t *out, void *stream) {
    using qmm::fail;
    if (rows < 0 || hidden <= 0)
        return fail(QMM_ERR_BAD_SHAPE, "residual layernorm: %lld rows of %lld", (long long)rows, (long long)hidden);
    if (rows == 0) return QMM_OK;
    if (!x || !delta) return fail(QMM_ERR_INVALID_ARGUMENT, "residual layernorm: null x or delta");
    if (gate && !bias) return fail(QMM_ERR_INVALID_ARGUMENT, "residual layernorm: a gate multiplies the bias; no bias given");
    if (out && (!shift || !scale))
        return fail(QMM_ERR_INVALID_ARGUMENT, "residual layernorm: the normalised output needs shift and scale");
    if (hidden % 256 != 0 || hidden > 4096)
        return fail(QMM_ERR_UNSUPPORTED, "residual layernorm: hidden %lld is not a multiple of 256 up to 4096",
                    (long long)hidden);
    const uintptr_t a = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(delta) |
                        reinterpret_cast<uintptr_t>(bias) | reinterpret_cast<uintptr_t>(gate) |
                        reinterpret_cast<uintptr_t>(shift) | reinterpret_cast<uintptr_t>(scale) |
                        reinterpret_cast<uintptr_t>(out);
    if (a & 15u) return fail(QMM_ERR_MISALIGNED, "residual layernorm: pointers must be 16-byte aligned");
    {
        const uintptr_t xb = reinterpret_cast<uintptr_t>(x), xe = xb + (uintptr_t)(rows * hidden * 2);
        const uintptr_t db = reinterpret_cast<uintptr_t>(delta), de = db + (uintptr_t)(rows * hidden * 2);
        if (xb < de && db < xe) return fail(QMM_ERR_INVALID_ARGUMENT, "residual layernorm: delta overlaps x");
        if (out) {
            const uintptr_t ob = reinterpret_cast<uintptr_t>(out), oe = ob + (uintptr_t)(rows * hidden * 2);
            if ((ob < xe && xb < oe) || (ob < de && db < oe))
                return fail(QMM_ERR_INVALID_ARGUMENT, "residual layernorm: out overlaps x or delta");
        }
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return qmm::cuda_fail(e, "no CUDA device");
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const unsigned grid = (unsigned)((rows + qmm::kNormWarps - 1) / qmm::kNormWarps);
    switch ((int)(hidden / 256)) {
#define QMM_RLN_CASE(V) \
    case V: qmm::launch_residual_ln<V>(grid, st, x, rows, delta, bias, gate, shift, scale, eps, out); break;
        QMM_RLN_CASE(1) QMM_RLN_CASE(2) QMM_RLN_CASE(3) QMM_RLN_CASE(4) QMM_RLN_CASE(6) QMM_RLN_CASE(8)
        QMM_RLN_CASE(12) QMM_RLN_CASE(16)
#undef QMM_RLN_CASE
        default:
            return fail(QMM_ERR_UNSUPPORTED, "residual layernorm: hidden %lld is not 256/512/768/1024/1536/2048/3072/4096",
                        (long long)hidden);
    }
    qmm::count_launch();
    e = cudaGetLastError();
    return e == cudaSuccess ? QMM_OK : qmm::cuda_fail(e, "residual layernorm launch");
}

qmm_status qmm_layernorm_modulate(const uint16_t *x, int64_t rows, int64_t hidden, const uint16_t *shift,
                                  const uint16_t *scale, float eps, uint16_t *out, void *stream) {
    using qmm::fail;
    if (rows < 0 || hidden <= 0) return fail(QMM_ERR_BAD_SHAPE, "layernorm: %lld rows of %lld", (long long)rows, (long long)hidden);
    if (rows == 0) return QMM_OK;
    if (!x || !shift || !scale || !out) return fail(QMM_ERR_INVALID_ARGUMENT, "layernorm: null pointer");
    if (hidden % 256 != 0 || hidden > 4096)
        return fail(QMM_ERR_UNSUPPORTED, "layernorm: hidden %lld is not a multiple of 256 up to 4096", (long long)hidden);
    const uintptr_t a = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(shift) |
                        reinterpret_cast<uintptr_t>(scale) | reinterpret_cast<uintptr_t>(out);
    if (a & 15u) return fail(QMM_ERR_MISALIGNED, "layernorm: pointers must be 16-byte aligned");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return qmm::cuda_fail(e, "no CUDA device");
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const unsigned grid = (unsigned)((rows + qmm::kNormWarps - 1) / qmm::kNormWarps);
    const int vpl = (int)(hidden / 256);
    switch (vpl) {
#define QMM_LN_CASE(V) \
    case V: qmm::layernorm_modulate_kernel<V><<<grid, qmm::kNormWarps * 32, 0, st>>>(x, rows, shift, scale, eps, out); break;
        QMM_LN_CASE(1) QMM_LN_CASE(2) QMM_LN_CASE(3) QMM_LN_CASE(4) QMM_LN_CASE(5) QMM_LN_CASE(6) QMM_LN_CASE(7)
        QMM_LN_CASE(8) QMM_LN_CASE(9) QMM_LN_CASE(10) QMM_LN_CASE(11) QMM_LN_CASE(12) QMM_LN_CASE(13)
        QMM_LN_CASE(14) QMM_LN_CASE(15) QMM_LN_CASE(16)
#undef QMM_LN_CASE
        default: return fail(QMM_ERR_UNSUPPORTED, "layernorm: hidden %lld", (long long)hidden);
    }
    qmm::count_launch();
    e = cudaGetLastError();
    return e == cudaSuccess ? QMM_OK : qmm::cuda_fail(e, "layernorm launch");
}

}  // extern "C"
