// Fused epilogue: y = residual + gate * act(acc + bias), f32, one bf16 rounding;
// with res_mul the residual operand multiplies instead, y = residual * (gate *
// act(acc + bias)) (a SwiGLU up projection times the SiLU-activated gate
// projection, src/ops.rs:203).
// The reference applies these as separate bf16 tensor ops after the linear
// (image-forger src/quant.rs:157-160 bias; src/dit.rs:88-93 gate and residual).
#pragma once

#include "qmm.h"
#include "qmm_common.cuh"

namespace qmm {

__device__ __forceinline__ float apply_activation(float t, int act) {
    if (act == 1) {  // GELU, tanh approximation
        const float c = 0.7978845608028654f;
        return 0.5f * t * (1.0f + tanhf(c * (t + 0.044715f * t * t * t)));
    }
    if (act == 2) return t / (1.0f + expf(-t));  // SiLU
    return t;
}

struct EpilogueArgs {
    const uint16_t *bias;      // [n] or null
    const uint16_t *gate;      // [n] or null
    const uint16_t *residual;  // [m, n] or null
    int32_t act;               // qmm_activation
    int32_t res_mul;           // 1: the residual multiplies (QMM_EPILOGUE_RESIDUAL_MUL)
};

// The kernels' form of a qmm_epilogue: activation and residual mode decoded
// once on the host.
inline EpilogueArgs epilogue_args(const qmm_epilogue &ep) {
    return EpilogueArgs{ep.bias, ep.gate, ep.residual, ep.activation & 0xFF,
                        (ep.activation & QMM_EPILOGUE_RESIDUAL_MUL) ? 1 : 0};
}

// Per-output-feature constants of the epilogue.
struct FeatureConsts {
    float bias;
    float gate;
};

__device__ __forceinline__ FeatureConsts load_feature_consts(const EpilogueArgs &e, int64_t n,
                                                             bool valid) {
    FeatureConsts c{0.0f, 1.0f};
    if (valid) {
        if (e.bias) c.bias = bf16_bits_to_f32(__ldg(e.bias + n));
        if (e.gate) c.gate = bf16_bits_to_f32(__ldg(e.gate + n));
    }
    return c;
}

__device__ __forceinline__ float epilogue_value(const EpilogueArgs &e, const FeatureConsts &c,
                                                float acc, const uint16_t *residual_elem) {
    float t = apply_activation(acc + c.bias, e.act);
    if (e.gate) t = t * c.gate;
    if (residual_elem) {
        const float r = bf16_bits_to_f32(*residual_elem);
        t = e.res_mul ? r * t : r + t;
    }
    return t;
}

// Same as epilogue_value with the residual element already loaded (`resid`
// is ignored when the epilogue has no residual).
__device__ __forceinline__ float epilogue_value_rv(const EpilogueArgs &e, const FeatureConsts &c,
                                                   float acc, float resid) {
    float t = apply_activation(acc + c.bias, e.act);
    if (e.gate) t = t * c.gate;
    if (e.residual) t = e.res_mul ? resid * t : resid + t;
    return t;
}

__device__ __forceinline__ uint16_t f32_to_bf16_bits(float v) {
    __nv_bfloat16 b = __float2bfloat16_rn(v);
    return *reinterpret_cast<uint16_t *>(&b);
}

}  // namespace qmm
