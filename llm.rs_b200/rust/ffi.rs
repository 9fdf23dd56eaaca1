//! Raw bindings of `include/llmrs_cuda.h` for the reference crate
//! (`src/backend/cuda/ffi.rs` in the maintainer's tree).
//!
//! UNVERIFIED: written against the C header; this image has no Rust toolchain,
//! so it has never been compiled.  Every function returns 0 (`LLMRS_OK`) or an
//! `LLMRS_E*` code; `check` turns a nonzero code into a panic, which is how the
//! reference reports errors (`assert_eq!` at src/backend/cpu.rs:37, `.unwrap()`
//! on every OpenCL call in src/backend/opencl.rs).
#![allow(non_camel_case_types)]

use std::os::raw::{c_char, c_int, c_uint, c_ulonglong, c_void};

pub const LLMRS_OK: c_int = 0;
pub const LLMRS_F16: c_int = 0;
pub const LLMRS_F32: c_int = 1;
pub const LLMRS_BF16: c_int = 2;
pub const LLMRS_WFMT_Q4_0: c_int = 0;
pub const LLMRS_WFMT_Q8_0: c_int = 1;

// `which` codes of llmrs_model_set_weight / llmrs_model_load_weight
pub const LLMRS_W_Q: c_int = 0;
pub const LLMRS_W_K: c_int = 1;
pub const LLMRS_W_V: c_int = 2;
pub const LLMRS_W_O: c_int = 3;
pub const LLMRS_W_GATE_UP: c_int = 4;
pub const LLMRS_W_DOWN: c_int = 5;
pub const LLMRS_W_ATTN_NORM: c_int = 6;
pub const LLMRS_W_MLP_NORM: c_int = 7;
pub const LLMRS_W_EMBED: c_int = 8;
pub const LLMRS_W_FINAL_NORM: c_int = 9;
pub const LLMRS_W_LM_HEAD: c_int = 10;
pub const LLMRS_W_GATE: c_int = 11;
pub const LLMRS_W_UP: c_int = 12;

#[repr(C)]
pub struct llmrs_ctx {
    _opaque: [u8; 0],
}
#[repr(C)]
pub struct llmrs_model {
    _opaque: [u8; 0],
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct llmrs_config {
    pub n_layers: c_int,
    pub hidden: c_int,
    pub n_heads: c_int,
    pub n_kv_heads: c_int,
    pub head_dim: c_int,
    pub ffn: c_int,
    pub vocab: c_int,
    pub max_seq: c_int,
    pub rms_eps: f32,
    pub rope_theta: f32,
    pub weight_format: c_int,
    pub tied_embeddings: c_int,
    pub scale_dtype: c_int,
    pub tp_rank: c_int,
    pub tp_size: c_int,
}

#[link(name = "llmrs_cuda")]
extern "C" {
    pub fn llmrs_last_error() -> *const c_char;
    pub fn llmrs_version() -> *const c_char;
    pub fn llmrs_device_count(count: *mut c_int) -> c_int;
    pub fn llmrs_ctx_create(device: c_int, out: *mut *mut llmrs_ctx) -> c_int;
    pub fn llmrs_ctx_destroy(ctx: *mut llmrs_ctx) -> c_int;
    pub fn llmrs_ctx_set_stream(ctx: *mut llmrs_ctx, cuda_stream: *mut c_void) -> c_int;
    pub fn llmrs_malloc(ctx: *mut llmrs_ctx, bytes: usize, d_ptr: *mut *mut c_void) -> c_int;
    pub fn llmrs_free(ctx: *mut llmrs_ctx, d_ptr: *mut c_void) -> c_int;
    pub fn llmrs_h2d(ctx: *mut llmrs_ctx, d_dst: *mut c_void, h_src: *const c_void, bytes: usize) -> c_int;
    pub fn llmrs_d2h(ctx: *mut llmrs_ctx, h_dst: *mut c_void, d_src: *const c_void, bytes: usize) -> c_int;
    pub fn llmrs_d2d(ctx: *mut llmrs_ctx, d_dst: *mut c_void, d_src: *const c_void, bytes: usize) -> c_int;
    pub fn llmrs_memset(ctx: *mut llmrs_ctx, d_dst: *mut c_void, value: c_int, bytes: usize) -> c_int;
    pub fn llmrs_sync(ctx: *mut llmrs_ctx) -> c_int;
    pub fn llmrs_backend_name() -> *const c_char;

    // ---- one entry per `trait Backend` method (src/backend.rs:15-40) ----
    pub fn llmrs_matmul_transposed_q4(ctx: *mut llmrs_ctx, d_a: *const f32, d_qs: *const u8,
                                      d_scales: *const c_void, scale_dtype: c_int, d_c: *mut f32,
                                      m: c_int, k: c_int, n: c_int) -> c_int;
    pub fn llmrs_matmul_transposed_q8(ctx: *mut llmrs_ctx, d_a: *const f32, d_qw: *const i8,
                                      d_scales: *const c_void, scale_dtype: c_int, d_c: *mut f32,
                                      m: c_int, k: c_int, n: c_int) -> c_int;
    pub fn llmrs_matmul_transposed_f32(ctx: *mut llmrs_ctx, d_a: *const f32, d_b: *const f32, d_c: *mut f32,
                                       m: c_int, k: c_int, n: c_int) -> c_int;
    pub fn llmrs_matmul(ctx: *mut llmrs_ctx, d_a: *const f32, d_b: *const f32, d_c: *mut f32,
                        m: c_int, k: c_int, n: c_int) -> c_int;
    pub fn llmrs_matmul_slice(ctx: *mut llmrs_ctx, d_a: *const f32, d_other: *const f32, d_c: *mut f32,
                              m: c_int, rows: c_int, cols: c_int) -> c_int;
    pub fn llmrs_add_assign(ctx: *mut llmrs_ctx, d_a: *mut f32, d_b: *const f32, n: usize) -> c_int;
    pub fn llmrs_silu_mul(ctx: *mut llmrs_ctx, d_gate: *mut f32, d_up: *const f32, n: usize) -> c_int;
    pub fn llmrs_rope_inplace(ctx: *mut llmrs_ctx, d_x: *mut f32, rows: c_int, head_dim: c_int,
                              start_pos: c_int, theta_base: f32) -> c_int;
    pub fn llmrs_rms_norm(ctx: *mut llmrs_ctx, d_x: *const f32, d_w: *const f32, d_y: *mut f32,
                          rows: c_int, cols: c_int, eps: f32) -> c_int;
    pub fn llmrs_softmax(ctx: *mut llmrs_ctx, d_x: *const f32, d_y: *mut f32, rows: c_int, cols: c_int) -> c_int;
    pub fn llmrs_scale(ctx: *mut llmrs_ctx, d_x: *const f32, d_y: *mut f32, n: usize, value: f32) -> c_int;
    pub fn llmrs_copy_from(ctx: *mut llmrs_ctx, d_src: *const f32, d_dst: *mut f32, n: usize) -> c_int;
    pub fn llmrs_quantize_row_q8_0(ctx: *mut llmrs_ctx, d_x: *const f32, d_q: *mut i8, d_s: *mut f32,
                                   rows: c_int, k: c_int) -> c_int;
    pub fn llmrs_quantize_q4(ctx: *mut llmrs_ctx, d_w: *const f32, n: usize, d_qs: *mut u8,
                             d_scales: *mut f32) -> c_int;
    pub fn llmrs_sample(ctx: *mut llmrs_ctx, d_logits: *const f32, vocab: c_int, h_recent: *const c_int,
                        n_recent: c_int, repeat_penalty: f32, temperature: f32, top_p: f32, u: f32,
                        h_token: *mut c_int) -> c_int;

    // ---- fused attention ops ----
    pub fn llmrs_rope_table(head_dim: c_int, n_pos: c_int, theta_base: f32, h_cos: *mut f32,
                            h_sin: *mut f32) -> c_int;
    pub fn llmrs_attention_decode(ctx: *mut llmrs_ctx, d_qkv: *const f32, d_kcache: *mut f32, d_vcache: *mut f32,
                                  d_rope_cos: *const f32, d_rope_sin: *const f32, d_out: *mut f32,
                                  n_heads: c_int, n_kv_heads: c_int, head_dim: c_int, max_seq: c_int,
                                  pos: c_int) -> c_int;
    pub fn llmrs_attention_decode_noalloc(cuda_stream: *mut c_void, d_qkv: *const f32, d_kcache: *mut f32,
                                          d_vcache: *mut f32, d_rope_cos: *const f32, d_rope_sin: *const f32,
                                          d_out: *mut f32, n_heads: c_int, n_kv_heads: c_int, head_dim: c_int,
                                          max_seq: c_int, pos: c_int, d_err: *mut c_uint) -> c_int;
    pub fn llmrs_attention_prefill(ctx: *mut llmrs_ctx, d_qkv: *mut f32, d_kcache: *mut f32, d_vcache: *mut f32,
                                   d_rope_cos: *const f32, d_rope_sin: *const f32, d_out: *mut f32,
                                   n_rows: c_int, n_heads: c_int, n_kv_heads: c_int, head_dim: c_int,
                                   max_seq: c_int, start_pos: c_int) -> c_int;

    // ---- model: device-resident weights + KV cache, fused token loop ----
    pub fn llmrs_model_create(ctx: *mut llmrs_ctx, cfg: *const llmrs_config, out: *mut *mut llmrs_model) -> c_int;
    pub fn llmrs_model_destroy(model: *mut llmrs_model) -> c_int;
    pub fn llmrs_model_init_synthetic(model: *mut llmrs_model, seed: u64) -> c_int;
    pub fn llmrs_model_set_weight(model: *mut llmrs_model, layer: c_int, which: c_int, h_codes: *const c_void,
                                  h_scales: *const f32) -> c_int;
    pub fn llmrs_model_load_weight(model: *mut llmrs_model, layer: c_int, which: c_int, h_data: *const c_void,
                                   dtype: c_int) -> c_int;
    pub fn llmrs_kv_fill(model: *mut llmrs_model, layer: c_int, h_k: *const f32, h_v: *const f32,
                         n_pos: c_int) -> c_int;
    pub fn llmrs_kv_read(model: *mut llmrs_model, layer: c_int, h_k: *mut f32, h_v: *mut f32,
                         n_pos: c_int) -> c_int;
    pub fn llmrs_decode_step(model: *mut llmrs_model, token: c_int, pos: c_int, h_logits: *mut f32,
                             h_argmax: *mut c_int) -> c_int;
    pub fn llmrs_generate(model: *mut llmrs_model, token: c_int, pos: c_int, n_steps: c_int,
                          h_tokens_out: *mut c_int) -> c_int;
    pub fn llmrs_prefill(model: *mut llmrs_model, h_ids: *const c_int, n: c_int, start_pos: c_int,
                         h_logits: *mut f32, h_argmax: *mut c_int) -> c_int;
    pub fn llmrs_model_sample(model: *mut llmrs_model, h_recent: *const c_int, n_recent: c_int,
                              repeat_penalty: f32, temperature: f32, top_p: f32, u: f32,
                              h_token: *mut c_int) -> c_int;
    pub fn llmrs_model_logits(model: *mut llmrs_model, h_logits: *mut f32) -> c_int;

    // ---- tensor parallel (no counterpart in the reference) ----
    pub fn llmrs_model_tp_region(model: *mut llmrs_model, d_region: *mut *mut c_void, bytes: *mut usize) -> c_int;
    pub fn llmrs_model_tp_connect(model: *mut llmrs_model, regions: *const *mut c_void) -> c_int;
    pub fn llmrs_ipc_get_handle(d_ptr: *const c_void, handle_out: *mut c_void) -> c_int;
    pub fn llmrs_ipc_open_handle(device: c_int, handle: *const c_void, d_ptr_out: *mut *mut c_void) -> c_int;
    pub fn llmrs_ipc_close_handle(device: c_int, d_ptr: *mut c_void) -> c_int;
    pub fn llmrs_model_set_peer_timeout(model: *mut llmrs_model, timeout_ms: c_int) -> c_int;
    pub fn llmrs_model_tp_epoch(model: *mut llmrs_model, epoch: *mut c_ulonglong) -> c_int;
    pub fn llmrs_model_tp_resync(model: *mut llmrs_model, epoch: c_ulonglong) -> c_int;
}

/// Panic with the library's message on a nonzero status (the reference's
/// error convention: it panics, it never returns a `Result`).
pub fn check(rc: c_int) {
    if rc != LLMRS_OK {
        let msg = unsafe { std::ffi::CStr::from_ptr(llmrs_last_error()) };
        panic!("llmrs-cuda error {}: {}", rc, msg.to_string_lossy());
    }
}
