//! Raw declarations of include/marian_cuda.h, one per entry point, in the
//! header's order.  Layouts are `#[repr(C)]` mirrors of the header's structs.
#![allow(non_camel_case_types, dead_code)]

use std::os::raw::{c_char, c_void};

pub type mc_status = i32;
pub const MC_OK: mc_status = 0;
pub const MC_INVALID_INPUT: mc_status = 1;
pub const MC_MODEL: mc_status = 2;
pub const MC_INFERENCE: mc_status = 3;
pub const MC_DEVICE_TIMEOUT: mc_status = 4;
pub const MC_CUDA: mc_status = 5;

#[repr(C)]
pub struct mc_engine {
    _opaque: [u8; 0],
}

#[repr(C)]
#[derive(Clone, Copy, Default, Debug)]
pub struct mc_config {
    pub device: i32,
    pub max_inflight: u32,
    pub max_encode_tokens: u32,
    pub page_tokens: u32,
    pub kv_pages: u32,
    pub max_length_factor: u32,
    pub lanes: u32,
}

#[repr(C)]
#[derive(Clone, Copy, Default, Debug)]
pub struct mc_model_info {
    pub dim: i32,
    pub heads: i32,
    pub ffn_dim: i32,
    pub encoder_layers: i32,
    pub decoder_layers: i32,
    pub decoder_kind: i32,
    pub source_vocab: i32,
    pub target_vocab: i32,
    pub weight_bytes: u64,
}

#[repr(C)]
#[derive(Clone, Copy, Default, Debug)]
pub struct mc_model_report {
    pub tensors: u64,
    pub dense_linears: u64,
    pub embeddings: u64,
    pub activation_scales: u64,
    pub row_scaled_linears: u64,
    pub decoder_output_alpha: f32,
    pub engine_graph: i32,
    pub decoder_kind: i32,
    pub dim: i32,
    pub heads: i32,
    pub encoder_layers: i32,
    pub decoder_layers: i32,
}

#[repr(C)]
#[derive(Clone, Copy, Default, Debug)]
pub struct mc_text_segment {
    pub content_start: u64,
    pub content_end: u64,
    pub separator_start: u64,
    pub separator_end: u64,
    pub source_pieces: u64,
}

#[repr(C)]
pub struct mc_segment_error {
    pub kind: i32,
    pub start: u64,
    pub end: u64,
    pub pieces: u64,
    pub maximum: u64,
    pub message: [c_char; 256],
}

pub type mc_piece_count_fn = unsafe extern "C" fn(
    ctx: *mut c_void,
    text: *const c_char,
    len: usize,
    pieces: *mut u64,
    message: *mut c_char,
    message_capacity: usize,
) -> i32;

pub const MC_Q8_LINEAR_NOALLOC_MAX_ACTIVATIONS: u32 = 8 * 1024 * 1024;

// Kernel classes of mc_profile_read.
pub const MC_KERNEL_KINDS: i32 = 14;

unsafe extern "C" {
    pub fn mc_config_default(cfg: *mut mc_config);
    pub fn mc_create(cfg: *const mc_config, out: *mut *mut mc_engine) -> mc_status;
    pub fn mc_load_marian_bin(e: *mut mc_engine, bytes: *const u8, len: usize) -> mc_status;
    pub fn mc_model_info_get(e: *const mc_engine, info: *mut mc_model_info) -> mc_status;
    pub fn mc_inspect_marian_bin(
        bytes: *const u8,
        len: usize,
        report: *mut mc_model_report,
        message: *mut c_char,
        message_capacity: usize,
    ) -> mc_status;
    pub fn mc_load_shortlist(e: *mut mc_engine, bytes: *const u8, len: usize) -> mc_status;
    pub fn mc_destroy(e: *mut mc_engine);
    pub fn mc_last_error(e: *const mc_engine, buf: *mut c_char, cap: usize) -> usize;
    pub fn mc_is_ready(e: *const mc_engine) -> i32;
    pub fn mc_translate_token_ids(
        e: *mut mc_engine,
        tokens: *const i32,
        n_tokens: usize,
        offsets: *const u32,
        batch: u32,
        max_output_tokens: *const u32,
        force_len: *const u32,
        out_tokens: *mut i32,
        out_capacity: usize,
        out_offsets: *mut u32,
    ) -> mc_status;
    pub fn mc_submit(
        e: *mut mc_engine,
        request_id: u64,
        tokens: *const i32,
        n_tokens: u32,
        max_output_tokens: u32,
        force_len: u32,
    ) -> mc_status;
    pub fn mc_step(e: *mut mc_engine, active_after: *mut u32, queued_after: *mut u32) -> mc_status;
    pub fn mc_poll(
        e: *mut mc_engine,
        ids: *mut u64,
        lengths: *mut u32,
        max_results: u32,
        tokens: *mut i32,
        token_capacity: usize,
        n_results: *mut u32,
    ) -> mc_status;
    pub fn mc_trace_first_step(
        e: *mut mc_engine,
        tokens: *const i32,
        n_tokens: usize,
        offsets: *const u32,
        batch: u32,
        encoder_output: *mut f32,
        cross_key: *mut f32,
        cross_value: *mut f32,
        decoder_state: *mut f32,
    ) -> mc_status;
    pub fn mc_encode_token_ids(
        e: *mut mc_engine,
        tokens: *const i32,
        n_tokens: usize,
        offsets: *const u32,
        batch: u32,
        encoder_output: *mut f32,
    ) -> mc_status;
    pub fn mc_replay(
        e: *mut mc_engine,
        tokens: *const i32,
        n_tokens: usize,
        offsets: *const u32,
        batch: u32,
        max_output_tokens: *const u32,
        force_len: *const u32,
        arrival_s: *const f64,
        latency_s: *mut f64,
    ) -> mc_status;
    pub fn mc_stream(e: *const mc_engine) -> *mut c_void;
    pub fn mc_profile(e: *mut mc_engine, enable: i32) -> mc_status;
    pub fn mc_profile_read(
        e: *const mc_engine,
        kind: i32,
        launches: *mut u64,
        ms: *mut f64,
        flops: *mut f64,
        bytes: *mut f64,
    ) -> mc_status;
    pub fn mc_launch_count(e: *const mc_engine) -> u64;
    pub fn mc_timeline(e: *mut mc_engine, enable: i32) -> mc_status;
    pub fn mc_timeline_read(
        e: *const mc_engine,
        steps: *mut u64,
        busy_ms: *mut f64,
        idle_ms: *mut f64,
    ) -> mc_status;
    pub fn mc_q8_gemm(
        a: *const i8,
        w: *const i8,
        m: i32,
        n: i32,
        k: i32,
        row_scale: *const f32,
        col_scale: *const f32,
        bias: *const f32,
        residual: *const f32,
        relu: i32,
        mode: i32,
        out: *mut c_void,
        stream: *mut c_void,
    ) -> mc_status;
    pub fn mc_q8_linear(
        x: *const f32,
        m: i32,
        k: i32,
        w: *const i8,
        n: i32,
        activation_mult: f32,
        weight_mult: f32,
        bias: *const f32,
        y: *mut f32,
        stream: *mut c_void,
    ) -> mc_status;
    pub fn mc_q8_linear_ln(
        x: *const f32,
        m: i32,
        k: i32,
        w: *const i8,
        d: i32,
        activation_mult: f32,
        weight_mult: f32,
        bias: *const f32,
        residual: *const f32,
        gamma: *const f32,
        beta: *const f32,
        y: *mut f32,
        y_q: *mut i8,
        y_alpha: f32,
        stream: *mut c_void,
    ) -> mc_status;
    pub fn mc_q8_linear_noalloc(
        x: *const f32,
        m: i32,
        k: i32,
        w: *const i8,
        n: i32,
        activation_mult: f32,
        weight_mult: f32,
        bias: *const f32,
        y: *mut f32,
        stream: *mut c_void,
        status_bits: *mut u32,
    ) -> mc_status;
    pub fn mc_op_status(status_bits: *mut u32) -> mc_status;
    pub fn mc_segment_text(
        text: *const c_char,
        len: usize,
        max_pieces: u64,
        count_pieces: mc_piece_count_fn,
        ctx: *mut c_void,
        segments: *mut mc_text_segment,
        capacity: usize,
        n_segments: *mut usize,
        error: *mut mc_segment_error,
    ) -> mc_status;
}
