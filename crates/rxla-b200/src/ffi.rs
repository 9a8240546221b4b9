//! Raw declarations of `include/rxla_b200.h` (librxla_b200.so), one item per
//! header item and in the header's order.  Every function returns an `i32`
//! status (0 = OK, negative = a negated absl status class) unless noted.
#![allow(non_camel_case_types)]

use std::ffi::{c_char, c_void};

pub const RXLA_B200_ABI_VERSION: i32 = 1;

// status codes (rxla_b200_status)
pub const RXLA_B200_OK: i32 = 0;
pub const RXLA_B200_INVALID_ARGUMENT: i32 = -3;
pub const RXLA_B200_DEADLINE_EXCEEDED: i32 = -4;
pub const RXLA_B200_NOT_FOUND: i32 = -5;
pub const RXLA_B200_RESOURCE_EXHAUSTED: i32 = -8;
pub const RXLA_B200_FAILED_PRECONDITION: i32 = -9;
pub const RXLA_B200_OUT_OF_RANGE: i32 = -11;
pub const RXLA_B200_UNIMPLEMENTED: i32 = -12;
pub const RXLA_B200_INTERNAL: i32 = -13;
pub const RXLA_B200_UNAVAILABLE: i32 = -14;

// element types (rxla_b200_dtype)
pub const RXLA_B200_F32: i32 = 0;
pub const RXLA_B200_BF16: i32 = 1;
pub const RXLA_B200_U8: i32 = 2;
pub const RXLA_B200_I32: i32 = 3;
pub const RXLA_B200_F16: i32 = 4;

// linear epilogues (rxla_b200_epilogue)
pub const RXLA_B200_EPI_STORE: i32 = 0;
pub const RXLA_B200_EPI_RESIDUAL_ADD: i32 = 1;
pub const RXLA_B200_EPI_SWIGLU: i32 = 2;

// KV update policies (rxla_b200_kv_update)
pub const RXLA_B200_KV_CLAMP: i32 = 0;
pub const RXLA_B200_KV_CHECKED: i32 = 1;

pub const RXLA_B200_NOALLOC_SCRATCH_BYTES: u32 = 16 * 1024 * 1024;
pub const RXLA_B200_COMM_ID_BYTES: usize = 128;
pub const RXLA_B200_XLA_LINEAR_MAGIC: u32 = 0x4E4C_3852;
pub const RXLA_B200_XLA_ATTENTION_MAGIC: u32 = 0x5441_3852;

/// `rxla_b200_paged_decode_args`
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct rxla_b200_paged_decode_args {
    pub struct_size: u32,
    pub batch: i32,
    pub q_heads: i32,
    pub kv_heads: i32,
    pub head_dim: i32,
    pub q: *const u16,
    pub k_new: *const u16,
    pub v_new: *const u16,
    pub q_row_stride: i64,
    pub kv_row_stride: i64,
    pub q_norm_weight: *const f32,
    pub k_norm_weight: *const f32,
    pub norm_eps: f32,
    pub inv_freq: *const f32,
    pub rotary_dim: i32,
    pub scale: f32,
    pub k_pages: *mut u16,
    pub v_pages: *mut u16,
    pub num_pages: i64,
    pub page_size: i32,
    pub max_pages_per_seq: i32,
    pub page_table: *const i32,
    pub pages_per_seq: *const i32,
    pub ctx_lens: *const i32,
    pub kv_update: i32,
    pub advance_ctx: i32,
    pub accepted: *mut i32,
    pub out: *mut u16,
    pub workspace: *mut c_void,
    pub workspace_bytes: usize,
    pub max_context: i32,
}

/// `rxla_b200_gated_delta_args`
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct rxla_b200_gated_delta_args {
    pub struct_size: u32,
    pub batch: i32,
    pub tokens: i32,
    pub heads: i32,
    pub head_dim: i32,
    pub conv_kernel: i32,
    pub mixed: *const u16,
    pub z: *const u16,
    pub beta_logits: *const u16,
    pub a: *const u16,
    pub mixed_row_stride: i64,
    pub z_row_stride: i64,
    pub b_row_stride: i64,
    pub a_row_stride: i64,
    pub conv_weight: *const f32,
    pub a_log: *const f32,
    pub dt_bias: *const f32,
    pub norm_weight: *const f32,
    pub eps: f32,
    pub has_state: i32,
    pub conv_state: *mut u16,
    pub state: *mut f32,
    pub out: *mut u16,
    pub workspace: *mut c_void,
    pub workspace_bytes: usize,
}

/// `rxla_b200_decoder_config`
#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct rxla_b200_decoder_config {
    pub struct_size: u32,
    pub layers: i32,
    pub hidden: i32,
    pub q_heads: i32,
    pub kv_heads: i32,
    pub head_dim: i32,
    pub intermediate: i32,
    pub vocab: i32,
    pub rms_eps: f32,
    pub rope_theta: f32,
    pub embedding_dtype: i32,
    pub group_size: i32,
    pub max_batch: i32,
    pub max_context: i32,
    pub tp_rank: i32,
    pub tp_size: i32,
}

/// `rxla_b200_xla_linear_config`: a custom call's backend_config bytes (64).
#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct rxla_b200_xla_linear_config {
    pub magic: u32,
    pub version: u32,
    pub m: i64,
    pub n: i64,
    pub k: i64,
    pub group_size: i64,
    pub x_dtype: i32,
    pub y_dtype: i32,
    pub epilogue: i32,
    pub fused_norm: i32,
    pub eps: f32,
    pub reserved: i32,
}

/// `rxla_b200_xla_attention_config`: a custom call's backend_config bytes (64).
#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct rxla_b200_xla_attention_config {
    pub magic: u32,
    pub version: u32,
    pub batch: i32,
    pub q_heads: i32,
    pub kv_heads: i32,
    pub head_dim: i32,
    pub page_size: i32,
    pub max_pages_per_seq: i32,
    pub num_pages: i64,
    pub max_context: i32,
    pub has_qk_norm: i32,
    pub rotary_dim: i32,
    pub kv_update: i32,
    pub norm_eps: f32,
    pub scale: f32,
}

/// Opaque handles.
#[repr(C)]
pub struct rxla_b200_decoder {
    _private: [u8; 0],
}
#[repr(C)]
pub struct rxla_b200_comm {
    _private: [u8; 0],
}
#[repr(C)]
pub struct rxla_b200_safetensors {
    _private: [u8; 0],
}

extern "C" {
    pub fn rxla_b200_abi_version() -> i32;
    pub fn rxla_b200_last_error_message() -> *const c_char;
    pub fn rxla_b200_device_info(device: i32, sm_count: *mut i32, cc_major: *mut i32, cc_minor: *mut i32) -> i32;
    pub fn rxla_b200_device_status(reset: i32) -> i32;
    pub fn rxla_b200_set_wait_timeout(ns: i64) -> i32;
    pub fn rxla_b200_get_wait_timeout(ns: *mut i64) -> i32;
    pub fn rxla_b200_bounded_wait_check(kind: i32, flag: *const u64, target: u64,
                                        stream: *mut c_void) -> i32;

    pub fn rxla_b200_w8a16_linear(
        x: *const c_void, x_dtype: i32, weight: *const u8, scale: *const f32, group_size: i64,
        m: i64, n: i64, k: i64, y: *mut c_void, y_dtype: i32, epilogue: i32, stream: *mut c_void,
    ) -> i32;
    pub fn rxla_b200_w8a16_linear_workspace_size(
        m: i64, n: i64, k: i64, group_size: i64, epilogue: i32, bytes: *mut usize,
    ) -> i32;
    pub fn rxla_b200_w8a16_linear_ws(
        x: *const c_void, x_dtype: i32, weight: *const u8, scale: *const f32, group_size: i64,
        m: i64, n: i64, k: i64, y: *mut c_void, y_dtype: i32, epilogue: i32,
        workspace: *mut c_void, workspace_bytes: usize, stream: *mut c_void,
    ) -> i32;
    pub fn rxla_b200_w8a16_norm_linear(
        h: *const f32, norm_weight: *const f32, eps: f32, weight: *const u8, scale: *const f32,
        group_size: i64, m: i64, n: i64, k: i64, y: *mut c_void, y_dtype: i32, epilogue: i32,
        stream: *mut c_void,
    ) -> i32;
    pub fn rxla_b200_bf16_linear(
        x: *const c_void, x_dtype: i32, weight: *const u16, m: i64, n: i64, k: i64,
        y: *mut c_void, y_dtype: i32, epilogue: i32, stream: *mut c_void,
    ) -> i32;

    pub fn rxla_b200_paged_decode_workspace_size(
        batch: i32, q_heads: i32, kv_heads: i32, head_dim: i32, max_context: i32, bytes: *mut usize,
    ) -> i32;
    pub fn rxla_b200_paged_decode_attention(args: *const rxla_b200_paged_decode_args, stream: *mut c_void) -> i32;
    pub fn rxla_b200_paged_decode_attention_noalloc(
        args: *const rxla_b200_paged_decode_args, stream: *mut c_void,
    ) -> i32;

    pub fn rxla_b200_rms_norm_bf16(
        x: *const f32, weight: *const f32, rows: i64, width: i64, eps: f32, y: *mut u16,
        stream: *mut c_void,
    ) -> i32;
    pub fn rxla_b200_argmax(logits: *const f32, rows: i64, vocab: i64, out: *mut i32, stream: *mut c_void) -> i32;

    pub fn rxla_b200_w8_embedding(
        ids: *const i32, rows: i64, weight: *const u8, scale: *const f32, vocab: i64, hidden: i64,
        group_size: i64, out: *mut f32, stream: *mut c_void,
    ) -> i32;
    pub fn rxla_b200_sigmoid_gate(
        x: *const u16, x_row_stride: i64, gate: *const u16, gate_row_stride: i64, rows: i64,
        width: i64, y: *mut u16, y_row_stride: i64, stream: *mut c_void,
    ) -> i32;
    pub fn rxla_b200_gated_delta_workspace_size(
        batch: i32, tokens: i32, heads: i32, head_dim: i32, bytes: *mut usize,
    ) -> i32;
    pub fn rxla_b200_gated_delta(args: *const rxla_b200_gated_delta_args, stream: *mut c_void) -> i32;

    pub fn rxla_b200_decoder_create(
        config: *const rxla_b200_decoder_config, device: i32, comm: *mut rxla_b200_comm,
        out: *mut *mut rxla_b200_decoder,
    ) -> i32;
    pub fn rxla_b200_decoder_destroy(decoder: *mut rxla_b200_decoder) -> i32;
    pub fn rxla_b200_decoder_parameter(
        decoder: *mut rxla_b200_decoder, name: *const c_char, device_ptr: *mut *mut c_void,
        bytes: *mut i64, dtype: *mut i32,
    ) -> i32;
    pub fn rxla_b200_decoder_set_parameter(
        decoder: *mut rxla_b200_decoder, name: *const c_char, host: *const c_void, bytes: i64,
    ) -> i32;
    pub fn rxla_b200_decoder_init_synthetic(decoder: *mut rxla_b200_decoder, seed: u64) -> i32;
    pub fn rxla_b200_decoder_reset(decoder: *mut rxla_b200_decoder, stream: *mut c_void) -> i32;
    pub fn rxla_b200_decoder_step(
        decoder: *mut rxla_b200_decoder, tokens: *const i32, batch: i32, next_tokens: *mut i32,
        logits: *mut f32, stream: *mut c_void,
    ) -> i32;
    pub fn rxla_b200_decoder_prefill(
        decoder: *mut rxla_b200_decoder, seq: i32, tokens: *const i32, count: i32,
        next_token: *mut i32, logits: *mut f32, stream: *mut c_void,
    ) -> i32;

    pub fn rxla_b200_safetensors_open(path: *const c_char, out: *mut *mut rxla_b200_safetensors) -> i32;
    pub fn rxla_b200_safetensors_close(reader: *mut rxla_b200_safetensors) -> i32;
    pub fn rxla_b200_safetensors_count(reader: *const rxla_b200_safetensors, count: *mut i32) -> i32;
    pub fn rxla_b200_safetensors_info(
        reader: *const rxla_b200_safetensors, index: i32, name: *mut *const c_char,
        dtype: *mut i32, ndim: *mut i32, shape: *mut i64, bytes: *mut i64,
    ) -> i32;
    pub fn rxla_b200_safetensors_find(
        reader: *const rxla_b200_safetensors, name: *const c_char, index: *mut i32,
    ) -> i32;
    pub fn rxla_b200_safetensors_metadata(
        reader: *const rxla_b200_safetensors, key: *const c_char, value: *mut *const c_char,
    ) -> i32;
    pub fn rxla_b200_safetensors_read(
        reader: *const rxla_b200_safetensors, index: i32, row0: i64, rows: i64, col0: i64,
        cols: i64, dst: *mut c_void, dst_bytes: i64,
    ) -> i32;
    pub fn rxla_b200_decoder_load_safetensors(
        decoder: *mut rxla_b200_decoder, path: *const c_char, prefix: *const c_char,
        loaded: *mut i32, skipped: *mut i32,
    ) -> i32;
    pub fn rxla_b200_decoder_step_host(
        decoder: *mut rxla_b200_decoder, tokens_host: *const i32, batch: i32,
        next_tokens_host: *mut i32, stream: *mut c_void,
    ) -> i32;
    pub fn rxla_b200_decoder_io(
        decoder: *mut rxla_b200_decoder, tokens_in: *mut *mut i32, tokens_out: *mut *mut i32,
        logits: *mut *mut f32,
    ) -> i32;
    pub fn rxla_b200_decoder_kv_cache(
        decoder: *mut rxla_b200_decoder, layer: i32, k_pages: *mut *mut c_void,
        v_pages: *mut *mut c_void, bytes: *mut i64,
    ) -> i32;
    pub fn rxla_b200_decoder_context_lengths(decoder: *mut rxla_b200_decoder, lens: *mut *const i32) -> i32;
    pub fn rxla_b200_decoder_set_context_lengths(
        decoder: *mut rxla_b200_decoder, lens_host: *const i32, count: i32, stream: *mut c_void,
    ) -> i32;

    pub fn rxla_b200_comm_unique_id(id: *mut u8) -> i32;
    pub fn rxla_b200_comm_init(
        id: *const u8, rank: i32, world_size: i32, device: i32, out: *mut *mut rxla_b200_comm,
    ) -> i32;
    pub fn rxla_b200_comm_destroy(comm: *mut rxla_b200_comm) -> i32;
    pub fn rxla_b200_allreduce(
        comm: *mut rxla_b200_comm, buffer: *mut c_void, count: i64, dtype: i32, stream: *mut c_void,
    ) -> i32;
    pub fn rxla_b200_comm_p2p_enable(comm: *mut rxla_b200_comm, max_count: i64) -> i32;
    pub fn rxla_b200_p2p_allreduce_f32(
        comm: *mut rxla_b200_comm, partial: *mut f32, residual: *mut f32, count: i64,
        stream: *mut c_void,
    ) -> i32;

    // XLA legacy GPU custom-call handlers (no status return)
    pub fn rxla_b200_xla_w8a16_linear(
        stream: *mut c_void, buffers: *mut *mut c_void, opaque: *const c_char, opaque_len: usize,
    );
    pub fn rxla_b200_xla_w8a16_linear_status(
        stream: *mut c_void, buffers: *mut *mut c_void, opaque: *const c_char, opaque_len: usize,
        status: *mut c_void,
    );
    pub fn rxla_b200_xla_paged_decode_attention(
        stream: *mut c_void, buffers: *mut *mut c_void, opaque: *const c_char, opaque_len: usize,
    );
    pub fn rxla_b200_xla_paged_decode_attention_status(
        stream: *mut c_void, buffers: *mut *mut c_void, opaque: *const c_char, opaque_len: usize,
        status: *mut c_void,
    );
    pub fn rxla_b200_xla_check_config(target: *const c_char, opaque: *const c_void, opaque_len: usize) -> i32;
}
