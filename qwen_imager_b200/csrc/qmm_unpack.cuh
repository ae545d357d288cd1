// Unpacking of MLX affine codes into exact f32 integers, and the dequantized
// value f32(scale) * q + f32(offset) with the rounding of the reference
// (image-forger src/quant.rs:564-567: the product of a bf16 and an integer
// below 256 is exact in f32, so fmaf(q, s, o) == s*q + o rounded once).
//
// Codes are `bits` wide, packed little-end-first: code j of a word is
// (word >> (bits * j)) & (2^bits - 1).  An integer q < 256 placed in the low
// byte of the f32 bit pattern 0x4B000000 is the float 2^23 + q, so one byte
// permute plus one exact subtraction turns a code into a float.
#pragma once

#include <cuda_fp16.h>

#include "qmm_common.cuh"

namespace qmm {

constexpr float kMagic23 = 8388608.0f;  // 2^23

// Float 2^23 + (byte `i` of v).  Selector nibbles: byte0 <- v.b[i],
// bytes 1-2 <- 0x00 (byte 0 of 0x4B000000), byte3 <- 0x4B.
template <int I>
__device__ __forceinline__ float magic_byte(uint32_t v) {
    return __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7440u + I));
}

// The codes of one 32-bit word as exact floats, in k order.
template <int BITS>
struct WordCodes;

template <>
struct WordCodes<4> {
    static constexpr int kCount = 8;
    __device__ __forceinline__ static void unpack(uint32_t w, float (&q)[8]) {
        const uint32_t lo = w & 0x0F0F0F0Fu;         // codes 0, 2, 4, 6
        const uint32_t hi = (w >> 4) & 0x0F0F0F0Fu;  // codes 1, 3, 5, 7
        q[0] = magic_byte<0>(lo) - kMagic23;
        q[1] = magic_byte<0>(hi) - kMagic23;
        q[2] = magic_byte<1>(lo) - kMagic23;
        q[3] = magic_byte<1>(hi) - kMagic23;
        q[4] = magic_byte<2>(lo) - kMagic23;
        q[5] = magic_byte<2>(hi) - kMagic23;
        q[6] = magic_byte<3>(lo) - kMagic23;
        q[7] = magic_byte<3>(hi) - kMagic23;
    }
};

template <>
struct WordCodes<8> {
    static constexpr int kCount = 4;
    __device__ __forceinline__ static void unpack(uint32_t w, float (&q)[4]) {
        q[0] = magic_byte<0>(w) - kMagic23;
        q[1] = magic_byte<1>(w) - kMagic23;
        q[2] = magic_byte<2>(w) - kMagic23;
        q[3] = magic_byte<3>(w) - kMagic23;
    }
};

template <>
struct WordCodes<2> {
    static constexpr int kCount = 16;
    __device__ __forceinline__ static void unpack(uint32_t w, float (&q)[16]) {
        const uint32_t c0 = w & 0x03030303u;         // codes 0, 4, 8, 12
        const uint32_t c1 = (w >> 2) & 0x03030303u;  // codes 1, 5, 9, 13
        const uint32_t c2 = (w >> 4) & 0x03030303u;  // codes 2, 6, 10, 14
        const uint32_t c3 = (w >> 6) & 0x03030303u;  // codes 3, 7, 11, 15
        q[0] = magic_byte<0>(c0) - kMagic23;
        q[1] = magic_byte<0>(c1) - kMagic23;
        q[2] = magic_byte<0>(c2) - kMagic23;
        q[3] = magic_byte<0>(c3) - kMagic23;
        q[4] = magic_byte<1>(c0) - kMagic23;
        q[5] = magic_byte<1>(c1) - kMagic23;
        q[6] = magic_byte<1>(c2) - kMagic23;
        q[7] = magic_byte<1>(c3) - kMagic23;
        q[8] = magic_byte<2>(c0) - kMagic23;
        q[9] = magic_byte<2>(c1) - kMagic23;
        q[10] = magic_byte<2>(c2) - kMagic23;
        q[11] = magic_byte<2>(c3) - kMagic23;
        q[12] = magic_byte<3>(c0) - kMagic23;
        q[13] = magic_byte<3>(c1) - kMagic23;
        q[14] = magic_byte<3>(c2) - kMagic23;
        q[15] = magic_byte<3>(c3) - kMagic23;
    }
};

// Dequantizes one word into bf16 pairs: out[i] holds codes 2i (low half) and
// 2i+1 (high half) as bf16(fmaf(q, s, o)), i.e. bit-exact with the reference.
template <int BITS>
__device__ __forceinline__ void dequant_word_bf16x2(uint32_t w, float s, float o,
                                                    uint32_t (&out)[WordCodes<BITS>::kCount / 2]) {
    constexpr int C = WordCodes<BITS>::kCount;
    float q[C];
    WordCodes<BITS>::unpack(w, q);
#pragma unroll
    for (int i = 0; i < C / 2; ++i)
        out[i] = pack_bf16x2_rn(fmaf(q[2 * i], s, o), fmaf(q[2 * i + 1], s, o));
}

// Same result as dequant_word_bf16x2 with the subtraction of 2^23 and the
// multiply-add done as packed f32x2 operations (half the FMA-pipe instructions).
template <int I>
__device__ __forceinline__ uint32_t magic_byte_bits(uint32_t v) {
    return __byte_perm(v, 0x4B000000u, 0x7440u + I);
}

// F16: the same values rounded to fp16 pairs instead (the GEMM's fp16-operand
// instantiation; 11 significant bits instead of 8).
template <int BITS, bool F16 = false>
__device__ __forceinline__ void dequant_word_bf16x2_packed(uint32_t w, float2 s2, float2 o2,
                                                           uint32_t (&out)[WordCodes<BITS>::kCount / 2]) {
    constexpr int C = WordCodes<BITS>::kCount;
    const float2 neg_magic = make_float2(-kMagic23, -kMagic23);
    uint32_t m[C];
    if constexpr (BITS == 8) {
        m[0] = magic_byte_bits<0>(w);
        m[1] = magic_byte_bits<1>(w);
        m[2] = magic_byte_bits<2>(w);
        m[3] = magic_byte_bits<3>(w);
    } else if constexpr (BITS == 4) {
        const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
        m[0] = magic_byte_bits<0>(lo);
        m[1] = magic_byte_bits<0>(hi);
        m[2] = magic_byte_bits<1>(lo);
        m[3] = magic_byte_bits<1>(hi);
        m[4] = magic_byte_bits<2>(lo);
        m[5] = magic_byte_bits<2>(hi);
        m[6] = magic_byte_bits<3>(lo);
        m[7] = magic_byte_bits<3>(hi);
    } else {
        static_assert(BITS == 4 || BITS == 8, "packed path covers 4- and 8-bit codes");
    }
#pragma unroll
    for (int i = 0; i < C / 2; ++i) {
        const float2 f = make_float2(__uint_as_float(m[2 * i]), __uint_as_float(m[2 * i + 1]));
        const float2 q = add_f32x2(f, neg_magic);
        const float2 v = fma_f32x2(q, s2, o2);
        if constexpr (F16) {
            const __half2 h = __floats2half2_rn(v.x, v.y);
            out[i] = *reinterpret_cast<const uint32_t *>(&h);
        } else {
            out[i] = pack_bf16x2_rn(v.x, v.y);
        }
    }
}

}  // namespace qmm
