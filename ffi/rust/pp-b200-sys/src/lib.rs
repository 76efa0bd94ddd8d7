//! Bindings to `libpp_b200.so`, the B200 (sm_100a) int8 historical-KV decode
//! engine, declared in `include/pp_b200.h`.
//!
//! The library replaces the CUDA branches of the model's `int8_kv_ops` module
//! (app/src/model/int8_kv_ops.rs:11-55, Candle CustomOps over NVRTC kernels);
//! with the `candle` feature, [`int8_kv_ops`] holds those branches written
//! against this crate.  Conventions follow the app's own C ABI
//! (app/native/aten_hip/cpp/painter_ffi.h:20-25): an `i32` status per call,
//! a thread-local last-error string whose text keeps the tokens the app's
//! error classifier reads (app/src/inference.rs:34-92), `struct_size`
//! versioned option structs and caller-owned device memory.  `stream` is the
//! `cudaStream_t` of the caller's device (null = legacy default stream).
//!
//! Every declaration below mirrors the header one for one; the repository's
//! test suite parses both and compares names, argument types and struct
//! layouts.
#![allow(non_camel_case_types)]

use std::ffi::CStr;
use std::fmt;
use std::os::raw::{c_char, c_void};

pub const PP_B200_ABI_VERSION: u32 = 1;

pub const PP_STATUS_OK: i32 = 0;
pub const PP_STATUS_PRECONDITION: i32 = 1;
pub const PP_STATUS_INVALID_OUTPUT: i32 = 2;
pub const PP_STATUS_UNCERTAIN: i32 = 3;

pub const PP_DTYPE_F32: i32 = 0;
pub const PP_DTYPE_BF16: i32 = 1;

pub const PP_DEV_NONFINITE_INPUT: u32 = 0x1;
pub const PP_DEV_OFFSET_RANGE: u32 = 0x2;
pub const PP_DEV_LENGTH_RANGE: u32 = 0x4;
pub const PP_DEV_WAIT_TIMEOUT: u32 = 0x8;
pub const PP_DEV_POSITION_RANGE: u32 = 0x10;

pub const PP_ATTN_PLAN_READY: u32 = 0x1;
pub const PP_ATTN_PREFETCH_HISTORY: u32 = 0x2;

/// A caller-owned int8 KV arena of one layer: codes `u8 [rows, capacity,
/// head_dim]`, scales `f32 [rows, capacity]`, row = branch * heads + head.
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct PpKvArena {
    pub struct_size: u32,
    pub rows: u32,
    pub heads: u32,
    pub head_dim: u32,
    pub capacity: u32,
    pub reserved: u32,
    pub k: *mut u8,
    pub v: *mut u8,
    pub k_scale: *mut f32,
    pub v_scale: *mut f32,
}

/// Attention options (`split_tokens` 0 = stream-K balance over the SMs).
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct PpAttnParams {
    pub struct_size: u32,
    pub split_tokens: u32,
    pub q_dtype: i32,
    pub out_dtype: i32,
    pub softmax_scale: f32,
    pub flags: u32,
    pub max_ctas: u32,
    pub reserved: u32,
}

impl Default for PpAttnParams {
    fn default() -> Self {
        PpAttnParams {
            struct_size: std::mem::size_of::<PpAttnParams>() as u32,
            split_tokens: 0,
            q_dtype: PP_DTYPE_F32,
            out_dtype: PP_DTYPE_F32,
            softmax_scale: 0.0,
            flags: 0,
            max_ctas: 0,
            reserved: 0,
        }
    }
}

/// Float K/V rows `[rows, tokens, head_dim]` for the float-KV attention.
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct PpFloatKv {
    pub struct_size: u32,
    pub rows: u32,
    pub heads: u32,
    pub head_dim: u32,
    pub tokens: u32,
    pub dtype: i32,
    pub k_row_stride: u64,
    pub v_row_stride: u64,
    pub k: *const c_void,
    pub v: *const c_void,
}

/// Geometry of a QKV projection output for the q/k norm + RoPE epilogue.
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct PpQkvRope {
    pub struct_size: u32,
    pub rows: u32,
    pub heads: u32,
    pub head_dim: u32,
    pub max_context: u32,
    pub dtype: i32,
    pub reserved: [u32; 2],
}

extern "C" {
    pub fn pp_b200_abi_version() -> u32;
    pub fn pp_b200_last_error() -> *const c_char;
    pub fn pp_b200_quantize(x: *const c_void, x_dtype: i32, rows: u64, head_dim: u32, packed: *mut u8,
                            scales: *mut f32, status: *mut u32, stream: *mut c_void) -> i32;
    pub fn pp_b200_dequantize(packed: *const u8, scales: *const f32, rows: u64, head_dim: u32, round_bf16: i32,
                              out_dtype: i32, out: *mut c_void, stream: *mut c_void) -> i32;
    pub fn pp_b200_quant_append(arena: *const PpKvArena, k_new: *const c_void, v_new: *const c_void, dtype: i32,
                                offsets: *const u32, commit: u32, status: *mut u32, stream: *mut c_void) -> i32;
    pub fn pp_b200_copy_prefix(src: *const PpKvArena, dst: *const PpKvArena, lengths: *const u32,
                               stream: *mut c_void) -> i32;
    pub fn pp_b200_attention_workspace_size(arena: *const PpKvArena, params: *const PpAttnParams) -> usize;
    pub fn pp_b200_plan_ragged(arena: *const PpKvArena, params: *const PpAttnParams, lengths: *const u32,
                               scratch_token: u32, workspace: *mut c_void, workspace_bytes: usize,
                               stream: *mut c_void) -> i32;
    pub fn pp_b200_decode_attention(arena: *const PpKvArena, params: *const PpAttnParams, q: *const c_void,
                                    scratch_k: *const f32, scratch_v: *const f32, lengths: *const u32,
                                    out: *mut c_void, workspace: *mut c_void, workspace_bytes: usize,
                                    status: *mut u32, stream: *mut c_void) -> i32;
    /// Attention for callers that cannot allocate device memory at the call:
    /// a 4 MiB scratch array inside the library stands in for the workspace
    /// (larger geometries and plan reuse are refused; overlapping calls race).
    pub fn pp_b200_decode_attention_static(arena: *const PpKvArena, params: *const PpAttnParams, q: *const c_void,
                                           scratch_k: *const f32, scratch_v: *const f32, lengths: *const u32,
                                           out: *mut c_void, status: *mut u32, stream: *mut c_void) -> i32;
    pub fn pp_b200_float_attention_workspace_size(kv: *const PpFloatKv, params: *const PpAttnParams) -> usize;
    pub fn pp_b200_plan_ragged_float(kv: *const PpFloatKv, params: *const PpAttnParams, lengths: *const u32,
                                     workspace: *mut c_void, workspace_bytes: usize, stream: *mut c_void) -> i32;
    pub fn pp_b200_decode_attention_float(kv: *const PpFloatKv, params: *const PpAttnParams, q: *const c_void,
                                          q_row_stride: u64, lengths: *const u32, out: *mut c_void,
                                          workspace: *mut c_void, workspace_bytes: usize, status: *mut u32,
                                          stream: *mut c_void) -> i32;
    pub fn pp_b200_diag_bounded_wait(status: *mut u32, limit_us: u32, stream: *mut c_void) -> i32;
    pub fn pp_b200_status_message(status_bits: u32) -> *const c_char;
    pub fn pp_b200_checked_batch_rows(logical_rows: u64, guidance: u32, physical_rows: *mut u64) -> i32;
    pub fn pp_b200_check_write_offsets(past_lens: *const u64, count: u64, heads: u32, head_dim: u32,
                                       capacity: u32) -> i32;
    pub fn pp_b200_sched_partition(cost: *const u64, n_branches: u32, n_shards: u32, shard_of_branch: *mut u32,
                                   shard_cost: *mut u64) -> i32;
    pub fn pp_b200_sched_lane_seed(base: u64, lane: u64) -> u64;
    pub fn pp_b200_sched_uniform(lane_seed: u64, draw: u64) -> f32;
    pub fn pp_b200_sched_uniforms(lane_seeds: *const u64, draws: *mut u64, active: *const u32, rows: u32,
                                  out: *mut f32, stream: *mut c_void) -> i32;
    pub fn pp_b200_qkv_rope(geometry: *const PpQkvRope, qkv: *const c_void, params: *const c_void,
                            positions: *const u32, out: *mut c_void, status: *mut u32, stream: *mut c_void) -> i32;
    pub fn pp_b200_qkv_rope_append(geometry: *const PpQkvRope, qkv: *const c_void, params: *const c_void,
                                   positions: *const u32, arena: *const PpKvArena, offsets: *const u32, commit: u32,
                                   q_out: *mut c_void, scratch_k: *mut f32, scratch_v: *mut f32, status: *mut u32,
                                   stream: *mut c_void) -> i32;
    pub fn pp_b200_swiglu(input: *const c_void, out: *mut c_void, rows: u64, hidden: u32, dtype: i32,
                          stream: *mut c_void) -> i32;
    pub fn pp_b200_rmsnorm(x: *const c_void, residual: *const c_void, x_sum: *mut c_void, weight: *const c_void,
                           out: *mut c_void, rows: u64, width: u32, eps: f32, dtype: i32, stream: *mut c_void) -> i32;
    pub fn pp_b200_renyi_sample(raw: *const f32, uniforms: *const f32, bounds: *const u32, out: *mut u32, batch: u32,
                                choices: u32, guidance: u32, alpha: f32, cfg: f32, token_offset: u32,
                                stream: *mut c_void) -> i32;
    pub fn pp_b200_prepare(device: i32) -> i32;
    pub fn pp_b200_prepare_optional(device: i32, fusion: u32, split_k: u32, model_dtype: i32, head_width: u32,
                                    ffn_hidden: u32) -> i32;
}

/// The class of a non-OK status, with the library's message.
#[derive(Clone, Debug, PartialEq, Eq)]
pub enum PpError {
    /// Status 1: invalid geometry or argument; nothing was launched.
    Precondition(String),
    /// Status 2: a device status word reported invalid data.
    InvalidOutput(String),
    /// Status 3: a CUDA failure; the device state is uncertain and the KV
    /// state must be discarded.
    Uncertain(String),
}

impl fmt::Display for PpError {
    fn fmt(&self, f: &mut fmt::Formatter<'_>) -> fmt::Result {
        match self {
            PpError::Precondition(m) | PpError::InvalidOutput(m) | PpError::Uncertain(m) => f.write_str(m),
        }
    }
}

impl std::error::Error for PpError {}

/// The calling thread's last error message.
pub fn last_error() -> String {
    // SAFETY: the library returns a valid, NUL-terminated thread-local string.
    unsafe { CStr::from_ptr(pp_b200_last_error()) }.to_string_lossy().into_owned()
}

/// Text of device status bits (PP_DEV_*).
pub fn status_message(bits: u32) -> String {
    // SAFETY: the library returns a NUL-terminated string in static storage.
    unsafe { CStr::from_ptr(pp_b200_status_message(bits)) }.to_string_lossy().into_owned()
}

/// Turns a status into `Result`, carrying the library's message; its text
/// keeps the tokens the app's classifier reads (inference.rs:34-92).
pub fn check(status: i32) -> Result<(), PpError> {
    match status {
        PP_STATUS_OK => Ok(()),
        PP_STATUS_PRECONDITION => Err(PpError::Precondition(last_error())),
        PP_STATUS_INVALID_OUTPUT => Err(PpError::InvalidOutput(last_error())),
        _ => Err(PpError::Uncertain(last_error())),
    }
}

#[cfg(feature = "candle")]
pub mod int8_kv_ops;
