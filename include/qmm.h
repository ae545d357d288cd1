/*
 * qmm.h -- C ABI of the B200 (sm_100a) MLX affine group-quantized linear.
 *
 * The operator is the one image-forger's `quant::Linear` implements
 * (src/quant.rs): a weight matrix W [n, k] stored as `bits`-wide unsigned
 * codes packed little-end-first into uint32 words along k (first code in the
 * lowest bits), one bf16 scale and one bf16 offset ("biases" in MLX naming)
 * per group of `group` consecutive k, w = scale * q + offset, and an optional
 * per-output additive bias.  y [m, n] = x [m, k] . W^T (+ bias).
 *
 * Conventions of every entry point:
 *   - plain pointers to device memory, element counts as int64_t, the CUDA
 *     stream as an opaque `void *` (a cudaStream_t; NULL = legacy stream);
 *   - nothing is allocated; outputs are written into caller buffers;
 *   - launches are asynchronous on the given stream;
 *   - the return value is a qmm_status; the message of the last failure on the
 *     calling thread is available from qmm_last_error();
 *   - bf16 tensors are passed as uint16_t (raw bf16 bits), row-major and
 *     contiguous.
 * There is no CPU implementation behind this header: a process without a
 * usable CUDA device gets QMM_ERR_CUDA.
 */
#ifndef QMM_H
#define QMM_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QMM_ABI_VERSION 2

#if defined(__GNUC__)
#define QMM_API __attribute__((visibility("default")))
#else
#define QMM_API
#endif

/* Status codes.  Replaces the `candle_core::Error` results of quant.rs. */
typedef enum qmm_status {
    QMM_OK = 0,
    QMM_ERR_INVALID_ARGUMENT = 1, /* null pointer where one is required, bad enum */
    QMM_ERR_BAD_SHAPE = 2,        /* shapes inconsistent (quant.rs:50-67, 438-445, 506-513) */
    QMM_ERR_UNSUPPORTED = 3,      /* valid layout the fused kernels do not cover: the caller
                                     dequantizes and runs a dense GEMM (quant.rs:121, 783-790) */
    QMM_ERR_MISALIGNED = 4,       /* a pointer is not 16-byte aligned */
    QMM_ERR_CUDA = 5,             /* a CUDA runtime/driver call failed */
    QMM_ERR_TIMEOUT = 6           /* a bounded device-side wait expired (see qmm_device_error) */
} qmm_status;

/* Element type of qmm_dequantize's output (quant.rs:570-575: bf16 or f32). */
typedef enum qmm_dtype {
    QMM_DTYPE_BF16 = 0,
    QMM_DTYPE_F32 = 1
} qmm_dtype;

/*
 * A packed quantized weight: the `Affine` state of quant.rs:31-39.
 *   packed : uint32 [n, k * bits / 32]   (MLX "weight")
 *   scales : bf16   [n, k / group]       (MLX "scales")
 *   biases : bf16   [n, k / group]       (MLX "biases", quant.rs `offsets`)
 * The struct only borrows the pointers; weights are never modified.
 */
typedef struct qmm_weight {
    const uint32_t *packed;
    const uint16_t *scales;
    const uint16_t *biases;
    int64_t n;      /* output features (rows of W) */
    int64_t k;      /* input features */
    int32_t bits;   /* 2, 4 or 8 */
    int32_t group;  /* inputs per scale/offset group */
} qmm_weight;

/* Activation applied in the fused epilogue. */
typedef enum qmm_activation {
    QMM_ACT_NONE = 0,
    QMM_ACT_GELU_TANH = 1,   /* 0.5 t (1 + tanh(sqrt(2/pi) (t + 0.044715 t^3))) */
    QMM_ACT_SILU = 2         /* t / (1 + exp(-t)) */
} qmm_activation;

/*
 * Flag ORed into qmm_epilogue.activation: the residual operand multiplies
 * instead of adding, y = residual * (gate * act(acc + bias)).  With the
 * SiLU-activated gate projection of a SwiGLU MLP as the residual, the up
 * projection's epilogue forms silu(x Wg^T) * (x Wu^T) (src/ops.rs:196-207).
 */
#define QMM_EPILOGUE_RESIDUAL_MUL 0x100

/*
 * Fused epilogue, evaluated in f32 on the accumulator before one rounding to
 * bf16:  y = residual + gate * act(acc + bias)  (or residual * (...), see
 * QMM_EPILOGUE_RESIDUAL_MUL).
 * Every pointer may be NULL (term omitted).  bias and gate are bf16 [n]
 * (quant.rs:157-160 adds `bias`; src/dit.rs:88-93 multiplies by a per-feature
 * gate and adds the residual stream); residual is bf16 [m, n] and may alias y.
 */
typedef struct qmm_epilogue {
    const uint16_t *bias;
    const uint16_t *gate;
    const uint16_t *residual;
    int32_t activation;     /* qmm_activation, optionally | QMM_EPILOGUE_RESIDUAL_MUL */
} qmm_epilogue;

/* Kernel selection for qmm_linear_ex (tests and benchmarks). */
typedef enum qmm_path {
    QMM_PATH_AUTO = 0,   /* m <= 16: GEMV, otherwise the tcgen05 GEMM */
    QMM_PATH_GEMV = 1,   /* streaming GEMVs: tensor-core (4-bit, m <= 16), FMA (m <= 16),
                            warp-per-row (any m, slow for large m), first that fits */
    QMM_PATH_GEMM = 2,   /* tcgen05/TMEM GEMM, any m >= 1 */
    QMM_PATH_GEMM_PAIR = 3, /* the GEMM on CTA pairs (cta_group::2, MMA M = 256) */
    QMM_PATH_GEMM_F16 = 4   /* the GEMM with fp16 operands: x is fp16 (not bf16) and the
                               dequantized weights are rounded to fp16 (11 significant bits
                               instead of bf16's 8; closer to the reference's f32 weights,
                               src/quant.rs:105-113); y and the epilogue operands stay bf16 */
} qmm_path;

/* ABI version of the loaded library (QMM_ABI_VERSION at build time). */
QMM_API int32_t qmm_abi_version(void);

/* Message of the last non-OK status returned on the calling thread ("" if none). */
QMM_API const char *qmm_last_error(void);

/*
 * Infers bits and group from tensor shapes exactly as `Linear::load` does
 * (quant.rs:43-77): scales [scales_rows, scales_cols] must be [output, groups]
 * with groups > 0 dividing input; packed [packed_rows, packed_words] must have
 * packed_rows == output and packed_words * 32 == bits * input for bits in
 * {2, 4, 8}.  Host-only; touches no device memory.
 */
QMM_API qmm_status qmm_infer_layout(int64_t input, int64_t output,
                            int64_t scales_rows, int64_t scales_cols,
                            int64_t packed_rows, int64_t packed_words,
                            int32_t *bits_out, int32_t *group_out);

/* Checks a qmm_weight for internal consistency (host-only, no device access). */
QMM_API qmm_status qmm_validate(const qmm_weight *w);

/*
 * Dense W [n, k] = T(f32(scale) * q + f32(offset)), T = bf16 (round to
 * nearest even) or f32.  Bit-exact with `Dequantize::cpu_fwd`
 * (quant.rs:528-577) and the Metal `dequantize` kernel (quant.rs:186-206).
 * Replaces CustomOp3 "mlx-dequantize" (quant.rs:523-643).
 */
QMM_API qmm_status qmm_dequantize(const qmm_weight *w, void *dst, int32_t dtype, void *stream);

/*
 * y [m, n] = epilogue(x [m, k] . W^T).  Replaces CustomOp2 "mlx-qmm"
 * (quant.rs:411-503) plus the bias add of `Affine::forward` (quant.rs:157-160).
 * x, y, residual: 16-byte aligned; y must not overlap x.  m == 0 is a no-op.
 * ep may be NULL (no bias, no gate, no residual, no activation).
 */
QMM_API qmm_status qmm_linear(const qmm_weight *w, const uint16_t *x, int64_t m,
                      const qmm_epilogue *ep, uint16_t *y, void *stream);

/* qmm_linear with an explicit kernel choice (qmm_path). */
QMM_API qmm_status qmm_linear_ex(const qmm_weight *w, const uint16_t *x, int64_t m,
                         const qmm_epilogue *ep, uint16_t *y, int32_t path,
                         void *stream);

/*
 * Split-K factor worth using for a GEMM of m tokens with this weight (1 = none):
 * > 1 only when the output tiles fill less than half of the SMs (the DiT text
 * stream, tensor-parallel shards).  Host-only.  No counterpart in quant.rs
 * (the Metal qmm kernel has one fixed 128x64 tiling, quant.rs:486-489).
 */
QMM_API int32_t qmm_gemm_splits(const qmm_weight *w, int64_t m);

/* Bytes of f32 workspace qmm_linear_splitk needs: splits * m * n * 4 (0 for splits <= 1). */
QMM_API uint64_t qmm_splitk_workspace_bytes(const qmm_weight *w, int64_t m, int32_t splits);

/*
 * qmm_linear on the tcgen05 GEMM with K split `splits` ways (k / 64 divisible
 * by splits, n % 4 == 0 when splits > 1): each split writes f32 partial tiles
 * into `workspace` (caller-owned, 16-byte aligned, qmm_splitk_workspace_bytes
 * long, not overlapping x or y; no zero-initialisation needed), and a second
 * kernel sums them and applies the epilogue with one bf16 rounding.  Same
 * result contract as qmm_linear.  Calls sharing a workspace must be ordered
 * (one stream).  Replaces, for small-m shapes, the same CustomOp2 "mlx-qmm"
 * (quant.rs:411-503).
 */
QMM_API qmm_status qmm_linear_splitk(const qmm_weight *w, const uint16_t *x, int64_t m,
                             const qmm_epilogue *ep, uint16_t *y, int32_t splits,
                             void *workspace, uint64_t workspace_bytes, void *stream);

/*
 * Fused LayerNorm (no affine, f32 statistics) and adaLN modulation of a DiT
 * block input: out = bf16((x - mean) / sqrt(var + eps) * (1 + scale) + shift),
 * x and out bf16 [rows, hidden], shift and scale bf16 [hidden]; hidden a
 * multiple of 256 up to 4096; 16-byte aligned pointers; out may alias x.
 * Replaces the separate norm and modulation tensor ops around every DiT linear
 * input (src/dit.rs:50, 91).
 */
QMM_API qmm_status qmm_layernorm_modulate(const uint16_t *x, int64_t rows, int64_t hidden,
                                  const uint16_t *shift, const uint16_t *scale, float eps,
                                  uint16_t *out, void *stream);

/*
 * Residual update of a DiT hidden state and the next block input's LayerNorm
 * + modulation, one pass per row (the sequence-parallel tensor-parallel
 * stack, where `delta` is the reduce-scattered sum of the ranks' gated
 * row-parallel partial outputs for this rank's rows):
 *   x   = bf16(x + delta + gate * bias)                      f32, one rounding
 *   out = bf16((x - mean) / sqrt(var + eps) * (1 + scale) + shift)   if out != NULL
 * x, delta, out bf16 [rows, hidden]; bias, gate, shift, scale bf16 [hidden];
 * bias (and gate, which multiplies only the bias) may be NULL; hidden one of
 * 256, 512, 768, 1024, 1536, 2048, 3072, 4096; 16-byte aligned pointers;
 * delta and out must not overlap x.  Replaces the residual add after the
 * gated out/MLP projections and the norm before the next linear
 * (src/dit.rs:88-93, src/dit.rs:50).
 */
QMM_API qmm_status qmm_residual_layernorm_modulate(uint16_t *x, int64_t rows, int64_t hidden,
                                           const uint16_t *delta, const uint16_t *bias,
                                           const uint16_t *gate, const uint16_t *shift,
                                           const uint16_t *scale, float eps, uint16_t *out,
                                           void *stream);

/*
 * Tensor-parallel collectives of the sequence-parallel DiT stack over peer
 * memory (NVLink), fused with the residual update and the next LayerNorm +
 * modulation.  No counterpart in quant.rs (the reference runs on one device);
 * they replace, per row-parallel layer, an NCCL reduce-scatter, the
 * residual + norm kernel and an NCCL all-gather.
 *
 * Every rank holds three symmetric buffers (allocated so that every rank can
 * address every rank's copy, e.g. a symmetric allocation or CUDA IPC):
 *   part     bf16 [world * rows, hidden]  this rank's gated row-parallel partials
 *   gathered bf16 [world * rows, hidden]  the normalised input of the next
 *                                         column-parallel linear, whole
 *   counters uint64 [4], zero at first use
 * Rank r owns tokens [r * rows, (r + 1) * rows).  Per layer, on every rank and
 * in the same order: qmm_tp_signal_ready (this rank's `part` is complete),
 * qmm_tp_reduce_norm_gather with the layer's epoch (1, 2, ... counting these
 * calls), qmm_tp_wait_gathered with the same epoch.  Every wait inside is
 * bounded (4 s); on expiry the kernels skip their work and qmm_device_error
 * reports QMM_ERR_TIMEOUT.
 */
#define QMM_TP_MAX_RANKS 8

typedef struct qmm_tp_peers {
    int32_t world;
    int32_t rank;
    uint16_t *part[QMM_TP_MAX_RANKS];
    uint16_t *gathered[QMM_TP_MAX_RANKS];
    uint64_t *counters[QMM_TP_MAX_RANKS];
} qmm_tp_peers;

/* Per-stream vectors of the residual update and the next norm (index 0: the
 * rows before `split`, 1: from `split` on), bf16 [hidden] each; bias and gate
 * may be NULL (the gate multiplies only the bias). */
typedef struct qmm_tp_norm {
    const uint16_t *bias[2];
    const uint16_t *gate[2];
    const uint16_t *shift[2];
    const uint16_t *scale[2];
    int64_t split;
    float eps;
} qmm_tp_norm;

/* This rank's `part` is complete: tells every rank (one tiny kernel on `stream`). */
QMM_API qmm_status qmm_tp_signal_ready(const qmm_tp_peers *peers, void *stream);

/*
 * For this rank's `rows` tokens (x: bf16 [rows, hidden], hidden 256, 512, 1024,
 * 3072 or 4096): with `reduce`, waits for every rank's signal of this epoch and
 * sets x = bf16(x + sum over ranks of part + gate * bias) (f32 sum, one
 * rounding); with `normalize`, stores bf16(LayerNorm(x) * (1 + scale) + shift)
 * into every rank's `gathered` at the tokens' rows.
 */
QMM_API qmm_status qmm_tp_reduce_norm_gather(const qmm_tp_peers *peers, uint64_t epoch, int64_t rows,
                                     int64_t hidden, uint16_t *x, const qmm_tp_norm *norm,
                                     int32_t reduce, int32_t normalize, void *stream);

/* Waits (one tiny kernel on `stream`) until every rank has finished the
 * epoch's qmm_tp_reduce_norm_gather: `gathered` is complete and no rank still
 * reads this rank's `part`. */
QMM_API qmm_status qmm_tp_wait_gathered(const qmm_tp_peers *peers, uint64_t epoch, void *stream);

/*
 * qmm_linear_splitk with the f32 scratch in a static device array of the
 * library (qmm_static_scratch_bytes() = 16 MiB, held by every GPU that loads
 * the library until exit) instead of a caller workspace: allocates nothing.
 * For callers that cannot call cudaMalloc: plug-ins whose host owns all
 * device memory and offers them no allocator, and paths that must not pay
 * the device-wide synchronization of cudaMalloc/cudaFree.  No counterpart in
 * quant.rs.
 *   - splits * m * n * 4 bytes must fit the scratch; larger requests return
 *     QMM_ERR_UNSUPPORTED before any launch;
 *   - the scratch keeps the last call's contents; nothing in it must start
 *     at zero;
 *   - every call on a device uses the same scratch: calls that may overlap on
 *     the GPU (other streams, threads) race, so order them on one stream;
 *   - the first call on a device resolves the scratch address with a runtime
 *     call; make it before any stream capture;
 *   - the address is kept for the life of the process: after cudaDeviceReset
 *     (or anything else that destroys the device's primary context) do not
 *     call this entry point again in that process.
 */
QMM_API qmm_status qmm_linear_splitk_static(const qmm_weight *w, const uint16_t *x, int64_t m,
                                    const qmm_epilogue *ep, uint16_t *y, int32_t splits, void *stream);

/* Size in bytes of the static scratch behind qmm_linear_splitk_static. */
QMM_API uint64_t qmm_static_scratch_bytes(void);

/*
 * Reads and clears the device-side error word that bounded waits inside the
 * kernels set when they expire (0 = none).  Synchronizes `stream`.  No
 * counterpart in quant.rs (Metal has no bounded waits to report).
 */
QMM_API qmm_status qmm_device_error(void *stream, uint32_t *code_out);

/*
 * Test support for the bounded waits (no counterpart in quant.rs): GEMM
 * launches made after the call, on the current device, use a test
 * instantiation of the kernel in which every CTA's copy producer stops before
 * its `withhold_block`-th k-block (-1: never) and every wait gives up after
 * `wait_limit_ns` (1 ms .. 4 s; 0: the default 4 s).  The waits for the
 * withheld block then run out: the launch ends early with its output
 * incomplete, having drained its own copies and MMAs and freed its tensor
 * memory, and qmm_device_error reports QMM_ERR_TIMEOUT.  Synchronous (it
 * writes a device variable).  qmm_debug_gemm_stall(-1, 0) restores normal
 * launches.
 */
QMM_API qmm_status qmm_debug_gemm_stall(int32_t withhold_block, uint64_t wait_limit_ns);

/*
 * Declares (on != 0) that no kernel writes the packed codes, scales or offsets
 * of the weights this process passes to the library while launches that use
 * them may run: weights are loaded once and then only read, as the
 * reference's immutable shared weight buffers (src/shared.rs:148-184).  The
 * tensor-core GEMV then streams its weights without waiting for the kernel
 * before it on the stream (programmatic dependent launch), so they arrive
 * while that kernel drains; x, bias, gate and residual are still read, and y
 * written, only after it has completed.  Off by default.  Applies to launches
 * made after the call, in this process; returns the previous setting.  No
 * counterpart in quant.rs.
 */
QMM_API int32_t qmm_set_weights_immutable(int32_t on);

/*
 * Caps the persistent kernels' grids at `sms` CTAs (0 = every SM) for launches
 * made after the call, in this process; returns the previous cap.  Leaves SMs
 * free for kernels that run concurrently on other streams (e.g. a collective
 * overlapping a row-parallel GEMM).  No counterpart in quant.rs.
 */
QMM_API int32_t qmm_set_sm_budget(int32_t sms);

/*
 * Architecture of the library's device code, as the CUDA runtime reports it
 * for one of its kernels (cudaFuncGetAttributes: binaryVersion and
 * ptxVersion, major * 10 + minor; 100 for sm_100a).  Needs a CUDA device.
 * No counterpart in quant.rs.
 */
QMM_API qmm_status qmm_binary_version(int32_t *binary_version, int32_t *ptx_version);

/* Number of kernels this library has launched in the calling process (kernels
 * captured into a CUDA graph count once, at capture).  No counterpart in quant.rs. */
QMM_API uint64_t qmm_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* QMM_H */
