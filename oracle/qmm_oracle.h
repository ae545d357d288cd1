/* ORACLE -- test infrastructure, not product code.  See qmm_oracle.c. */
#ifndef QMM_ORACLE_H
#define QMM_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

void oracle_set_threads(int32_t n);
int32_t oracle_get_threads(void);
float oracle_bf16_to_f32(uint16_t b);
uint16_t oracle_f32_to_bf16(float f);
void oracle_bf16_from_f32_array(const float *src, uint16_t *dst, int64_t count);
void oracle_f32_from_bf16_array(const uint16_t *src, float *dst, int64_t count);

void oracle_dequantize_f32(const uint32_t *packed, const uint16_t *scales,
                           const uint16_t *offsets, int64_t output, int64_t input,
                           int32_t bits, int32_t group, float *dst);
void oracle_dequantize_bf16(const uint32_t *packed, const uint16_t *scales,
                            const uint16_t *offsets, int64_t output, int64_t input,
                            int32_t bits, int32_t group, uint16_t *dst);
void oracle_matmul_f32(const float *x, const float *w, const uint16_t *bias,
                       int64_t m, int64_t n, int64_t k, float *y);
void oracle_linear_f32(const uint16_t *x, int64_t m, const uint32_t *packed,
                       const uint16_t *scales, const uint16_t *offsets,
                       const uint16_t *bias, int64_t n, int64_t k, int32_t bits,
                       int32_t group, float *w_scratch, float *x_scratch, float *y);
void oracle_epilogue_bf16(const float *y_f32, const uint16_t *gate,
                          const uint16_t *residual, int32_t activation, int64_t m,
                          int64_t n, uint16_t *out);

#ifdef __cplusplus
}
#endif

#endif
