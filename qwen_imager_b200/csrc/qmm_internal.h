// Host-side internals shared by the translation units of libqmm.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "qmm.h"

namespace qmm {

// Records a failure message for qmm_last_error() and returns `status`.
qmm_status fail(qmm_status status, const char *fmt, ...) __attribute__((format(printf, 2, 3)));

// Converts a CUDA runtime error into QMM_ERR_CUDA with a message.
qmm_status cuda_fail(cudaError_t e, const char *what);

// Device address of the library's device error word on the current device.
uint32_t *device_error_word();

// Streaming multiprocessors of the current device.
int sm_count();

// Counts kernel launches (exported through qmm_launch_count()).
void count_launch(uint64_t n = 1);

// Whether the streaming GEMV is launched as a programmatic dependent of the
// previous kernel of its stream (on unless QMM_GEMV_PDL=0; read once).
bool gemv_pdl_enabled();

// Whether the caller declared that no kernel writes packed weights, scales or
// offsets while the library uses them (qmm_set_weights_immutable).
bool weights_immutable();

// Test support (qmm_debug_gemm_stall): GEMM launches made after the call on
// the current device withhold k-block `withhold` (-1: none) and wait at most
// wait_ns (0: the default limit); (-1, 0) restores normal launches.
qmm_status gemm_set_stall(int32_t withhold, uint64_t wait_ns);

// Launchers.  Arguments are validated by the caller (qmm_api.cu).
qmm_status launch_dequantize(const qmm_weight &w, void *dst, int32_t dtype, cudaStream_t st);

// True when the GEMV kernel supports this layout and token count.
bool gemv_supported(const qmm_weight &w, int64_t m);
qmm_status launch_gemv(const qmm_weight &w, const uint16_t *x, int64_t m, const qmm_epilogue &ep,
                       uint16_t *y, cudaStream_t st);

// Tensor-core (mma.sync) streaming GEMV: 4-bit, m <= 16, group a multiple of 64.
bool gemv_mma_supported(const qmm_weight &w, int64_t m);
qmm_status launch_gemv_mma(const qmm_weight &w, const uint16_t *x, int64_t m, const qmm_epilogue &ep,
                           uint16_t *y, cudaStream_t st);

// Streaming (bulk-copy) GEMV for m <= 16.
bool gemv_tma_supported(const qmm_weight &w, int64_t m);
qmm_status launch_gemv_tma(const qmm_weight &w, const uint16_t *x, int64_t m, const qmm_epilogue &ep,
                           uint16_t *y, cudaStream_t st);

// True when the tcgen05 GEMM supports this layout.
bool gemm_supported(const qmm_weight &w);
// Split-K factor worth using for this shape (1 = none).
int gemm_recommended_splits(const qmm_weight &w, int64_t m);
// splits > 1: ws holds splits * m * n floats (16-byte aligned); k / 64 % splits == 0; n % 4 == 0.
// f16: x is fp16 and the weights are dequantized to fp16 (QMM_PATH_GEMM_F16).
qmm_status launch_gemm(const qmm_weight &w, const uint16_t *x, int64_t m, const qmm_epilogue &ep,
                       uint16_t *y, bool pair, int splits, float *ws, cudaStream_t st, bool f16 = false);

}  // namespace qmm
