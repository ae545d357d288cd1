//! Raw bindings to libqmm (`include/qmm.h`): the B200 (sm_100a) MLX affine
//! group-quantized linear that image-forger's `quant::Linear`
//! (src/quant.rs) calls instead of its Metal `mlx-qmm` / `mlx-dequantize`
//! custom ops.
//!
//! Every declaration mirrors the header one for one (names, argument order,
//! C types); `tests/test_rust_binding.py` checks that on every change.
//! Conventions, as in the header:
//!   - device pointers are plain pointers; bf16 values travel as raw `u16`
//!     bits, packed codes as `u32` words;
//!   - the CUDA stream is the caller's `cudaStream_t`, passed as `*mut c_void`
//!     (null = legacy stream);
//!   - nothing is allocated inside; launches are asynchronous;
//!   - every call returns a `qmm_status`; `qmm_last_error` holds the message
//!     of the last failure on the calling thread.
#![allow(non_camel_case_types)]
#![no_std]

use core::ffi::{c_char, c_void};

pub const QMM_ABI_VERSION: i32 = 2;

/// Status codes (replace the `candle_core::Error` results of quant.rs).
pub type qmm_status = i32;
pub const QMM_OK: qmm_status = 0;
pub const QMM_ERR_INVALID_ARGUMENT: qmm_status = 1;
pub const QMM_ERR_BAD_SHAPE: qmm_status = 2;
/// Valid layout the fused kernels do not cover: dequantize and run a dense
/// GEMM, as `Module::forward` does for unfused layouts (src/quant.rs:121).
pub const QMM_ERR_UNSUPPORTED: qmm_status = 3;
pub const QMM_ERR_MISALIGNED: qmm_status = 4;
pub const QMM_ERR_CUDA: qmm_status = 5;
pub const QMM_ERR_TIMEOUT: qmm_status = 6;

/// Output element type of `qmm_dequantize`.
pub type qmm_dtype = i32;
pub const QMM_DTYPE_BF16: qmm_dtype = 0;
pub const QMM_DTYPE_F32: qmm_dtype = 1;

/// Activation of the fused epilogue (`qmm_epilogue::activation`).
pub type qmm_activation = i32;
pub const QMM_ACT_NONE: qmm_activation = 0;
pub const QMM_ACT_GELU_TANH: qmm_activation = 1;
pub const QMM_ACT_SILU: qmm_activation = 2;
/// ORed into `qmm_epilogue::activation`: the residual multiplies.
pub const QMM_EPILOGUE_RESIDUAL_MUL: i32 = 0x100;

/// Kernel choice of `qmm_linear_ex`.
pub type qmm_path = i32;
pub const QMM_PATH_AUTO: qmm_path = 0;
pub const QMM_PATH_GEMV: qmm_path = 1;
pub const QMM_PATH_GEMM: qmm_path = 2;
pub const QMM_PATH_GEMM_PAIR: qmm_path = 3;
/// The GEMM with fp16 operands (x fp16, weights rounded to fp16); y stays bf16.
pub const QMM_PATH_GEMM_F16: qmm_path = 4;

/// A packed quantized weight: the `Affine` state of src/quant.rs:31-39.
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct qmm_weight {
    pub packed: *const u32,
    pub scales: *const u16,
    pub biases: *const u16,
    pub n: i64,
    pub k: i64,
    pub bits: i32,
    pub group: i32,
}

/// Fused epilogue: y = residual + gate * act(acc + bias), one bf16 rounding.
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct qmm_epilogue {
    pub bias: *const u16,
    pub gate: *const u16,
    pub residual: *const u16,
    pub activation: i32,
}

pub const QMM_TP_MAX_RANKS: i32 = 8;

/// The symmetric buffers of a tensor-parallel group as every rank sees them.
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct qmm_tp_peers {
    pub world: i32,
    pub rank: i32,
    pub part: [*mut u16; 8],
    pub gathered: [*mut u16; 8],
    pub counters: [*mut u64; 8],
}

/// Per-stream vectors of the residual update and the next norm.
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct qmm_tp_norm {
    pub bias: [*const u16; 2],
    pub gate: [*const u16; 2],
    pub shift: [*const u16; 2],
    pub scale: [*const u16; 2],
    pub split: i64,
    pub eps: f32,
}

#[link(name = "qmm")]
extern "C" {
    pub fn qmm_abi_version() -> i32;
    pub fn qmm_last_error() -> *const c_char;
    /// Shape inference of `Linear::load` (src/quant.rs:43-77).
    pub fn qmm_infer_layout(input: i64, output: i64, scales_rows: i64, scales_cols: i64, packed_rows: i64,
                            packed_words: i64, bits_out: *mut i32, group_out: *mut i32) -> qmm_status;
    pub fn qmm_validate(w: *const qmm_weight) -> qmm_status;
    /// CustomOp3 "mlx-dequantize" (src/quant.rs:523-643).
    pub fn qmm_dequantize(w: *const qmm_weight, dst: *mut c_void, dtype: i32, stream: *mut c_void) -> qmm_status;
    /// CustomOp2 "mlx-qmm" (src/quant.rs:411-503) plus the bias add (src/quant.rs:157-160).
    pub fn qmm_linear(w: *const qmm_weight, x: *const u16, m: i64, ep: *const qmm_epilogue, y: *mut u16,
                      stream: *mut c_void) -> qmm_status;
    pub fn qmm_linear_ex(w: *const qmm_weight, x: *const u16, m: i64, ep: *const qmm_epilogue, y: *mut u16,
                         path: i32, stream: *mut c_void) -> qmm_status;
    pub fn qmm_gemm_splits(w: *const qmm_weight, m: i64) -> i32;
    pub fn qmm_splitk_workspace_bytes(w: *const qmm_weight, m: i64, splits: i32) -> u64;
    pub fn qmm_linear_splitk(w: *const qmm_weight, x: *const u16, m: i64, ep: *const qmm_epilogue, y: *mut u16,
                             splits: i32, workspace: *mut c_void, workspace_bytes: u64,
                             stream: *mut c_void) -> qmm_status;
    pub fn qmm_layernorm_modulate(x: *const u16, rows: i64, hidden: i64, shift: *const u16, scale: *const u16,
                                  eps: f32, out: *mut u16, stream: *mut c_void) -> qmm_status;
    pub fn qmm_residual_layernorm_modulate(x: *mut u16, rows: i64, hidden: i64, delta: *const u16,
                                           bias: *const u16, gate: *const u16, shift: *const u16,
                                           scale: *const u16, eps: f32, out: *mut u16,
                                           stream: *mut c_void) -> qmm_status;
    pub fn qmm_tp_signal_ready(peers: *const qmm_tp_peers, stream: *mut c_void) -> qmm_status;
    pub fn qmm_tp_reduce_norm_gather(peers: *const qmm_tp_peers, epoch: u64, rows: i64, hidden: i64, x: *mut u16,
                                     norm: *const qmm_tp_norm, reduce: i32, normalize: i32,
                                     stream: *mut c_void) -> qmm_status;
    pub fn qmm_tp_wait_gathered(peers: *const qmm_tp_peers, epoch: u64, stream: *mut c_void) -> qmm_status;
    pub fn qmm_linear_splitk_static(w: *const qmm_weight, x: *const u16, m: i64, ep: *const qmm_epilogue,
                                    y: *mut u16, splits: i32, stream: *mut c_void) -> qmm_status;
    pub fn qmm_static_scratch_bytes() -> u64;
    pub fn qmm_device_error(stream: *mut c_void, code_out: *mut u32) -> qmm_status;
    pub fn qmm_debug_gemm_stall(withhold_block: i32, wait_limit_ns: u64) -> qmm_status;
    pub fn qmm_set_weights_immutable(on: i32) -> i32;
    pub fn qmm_set_sm_budget(sms: i32) -> i32;
    pub fn qmm_binary_version(binary_version: *mut i32, ptx_version: *mut i32) -> qmm_status;
    pub fn qmm_launch_count() -> u64;
}

/// `Ok(())` for `QMM_OK`, otherwise the status (read `qmm_last_error` on the
/// same thread for the message), the shape a `candle_core::bail!` wants.
pub fn check(status: qmm_status) -> Result<(), qmm_status> {
    if status == QMM_OK {
        Ok(())
    } else {
        Err(status)
    }
}
