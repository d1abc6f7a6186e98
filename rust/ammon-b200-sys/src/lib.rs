//! Raw `extern "C"` declarations of libammon_b200 (`include/ammon_b200.h`), one per header
//! declaration, with the header's types as `#[repr(C)]` structs and opaque handles. Every
//! function returns an `AB_*` status except the accessors noted in the header; on failure
//! `ab_last_error()` holds the message for the calling thread. The safe wrappers with the
//! reference crate's names live in the `ammon-b200` crate.
#![allow(non_camel_case_types)]
#![allow(clippy::missing_safety_doc)]

use std::os::raw::{c_char, c_int, c_void};

pub const AB_OK: c_int = 0;
pub const AB_ERR_VALIDATION: c_int = 1;
pub const AB_ERR_CUDA: c_int = 2;
pub const AB_ERR_ARGUMENT: c_int = 3;
pub const AB_ERR_DEVICE: c_int = 4;
pub const AB_ERR_NCCL: c_int = 5;

pub const AB_F32: i32 = 0;
pub const AB_BF16: i32 = 1;
pub const AB_U32: i32 = 2;

pub const AB_COMM_ID_BYTES: usize = 128;

/// Contiguous row-major device tensor view (rank 1..4).
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct ab_tensor {
    pub data: *mut c_void,
    pub dtype: i32,
    pub rank: i32,
    pub dims: [u32; 4],
}

/// DecodeStep { token, position }.
#[repr(C)]
#[derive(Clone, Copy, Debug, Default, PartialEq, Eq)]
pub struct ab_decode_step {
    pub token: u32,
    pub position: u32,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct ab_attention_weights {
    pub norm: ab_tensor,
    pub query: ab_tensor,
    pub key: ab_tensor,
    pub value: ab_tensor,
    pub output: ab_tensor,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct ab_swiglu_weights {
    pub norm: ab_tensor,
    pub gate: ab_tensor,
    pub up: ab_tensor,
    pub down: ab_tensor,
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct ab_llama_config {
    pub dim: u32,
    pub layers: u32,
    pub heads: u32,
    pub kv_heads: u32,
    pub head_dim: u32,
    pub hidden: u32,
    pub vocab: u32,
    pub seq: u32,
    pub batch: u32,
    pub rope_theta: f32,
    pub norm_eps: f32,
    pub dtype: i32,
}

/// AutoregressiveModel as a C vtable (`step` returns a host pointer to vocab_size logits,
/// valid until the next step).
#[repr(C)]
#[derive(Clone, Copy)]
pub struct ab_autoregressive_model {
    pub self_: *mut c_void,
    pub vocab_size: Option<unsafe extern "C" fn(*mut c_void) -> u32>,
    pub max_seq_len: Option<unsafe extern "C" fn(*mut c_void) -> u32>,
    pub step: Option<unsafe extern "C" fn(*mut c_void, u32, u32, *mut *const f32) -> c_int>,
}

macro_rules! opaque {
    ($($name:ident),*) => { $( #[repr(C)] pub struct $name { _private: [u8; 0] } )* };
}
opaque!(ab_runtime, ab_scheme, ab_kvcache, ab_attention_block, ab_swiglu_block, ab_llama,
        ab_comm, ab_bpe);

extern "C" {
    pub fn ab_last_error() -> *const c_char;
    pub fn ab_runtime_create(device: i32, out_: *mut *mut ab_runtime) -> c_int;
    pub fn ab_runtime_destroy(rt: *mut ab_runtime) -> c_int;
    pub fn ab_runtime_synchronize(rt: *mut ab_runtime) -> c_int;
    pub fn ab_runtime_stream(rt: *mut ab_runtime) -> *mut c_void;
    pub fn ab_runtime_sm_count(rt: *mut ab_runtime, out_: *mut i32) -> c_int;
    pub fn ab_runtime_set_wait_limit(rt: *mut ab_runtime, ms: u32) -> c_int;
    pub fn ab_runtime_wait_limit(rt: *mut ab_runtime, ms: *mut u32) -> c_int;
    pub fn ab_host_register(ptr: *mut c_void, bytes: u64) -> c_int;
    pub fn ab_host_unregister(ptr: *mut c_void) -> c_int;
    pub fn ab_tensor_zeros(rt: *mut ab_runtime, dtype: i32, rank: i32, dims: *const u32, out_: *mut ab_tensor) -> c_int;
    pub fn ab_tensor_free(rt: *mut ab_runtime, t: *mut ab_tensor) -> c_int;
    pub fn ab_tensor_write(rt: *mut ab_runtime, t: ab_tensor, host: *const c_void, bytes: u64) -> c_int;
    pub fn ab_tensor_read(rt: *mut ab_runtime, t: ab_tensor, host: *mut c_void, bytes: u64) -> c_int;
    pub fn ab_tensor_fill_normal(rt: *mut ab_runtime, t: ab_tensor, seed: u64, stream: u64, mean: f32, std: f32) -> c_int;
    pub fn ab_tensor_narrow(t: ab_tensor, start: u32, len: u32, out_: *mut ab_tensor) -> c_int;
    pub fn ab_tensor_reshape(t: ab_tensor, rank: i32, dims: *const u32, out_: *mut ab_tensor) -> c_int;
    pub fn ab_step_parcel(rt: *mut ab_runtime, n: u32, out_: *mut ab_tensor) -> c_int;
    pub fn ab_step_deposit(rt: *mut ab_runtime, parcel: ab_tensor, steps: *const ab_decode_step, n: u32) -> c_int;
    pub fn ab_scheme_create(rt: *mut ab_runtime, out_: *mut *mut ab_scheme) -> c_int;
    pub fn ab_scheme_destroy(s: *mut ab_scheme) -> c_int;
    pub fn ab_scheme_submit(s: *mut ab_scheme) -> c_int;
    pub fn ab_scheme_node_count(s: *const ab_scheme, out_: *mut u32) -> c_int;
    pub fn ab_scheme_replay_stats(s: *const ab_scheme, records: *mut u32, replays: *mut u32) -> c_int;
    pub fn ab_scheme_use_graph(s: *mut ab_scheme, enable: i32) -> c_int;
    pub fn ab_scheme_time_nodes(s: *mut ab_scheme, iters: u32, ms: *mut f32, n: u32) -> c_int;
    pub fn ab_scheme_node_label(s: *const ab_scheme, i: u32, buf: *mut c_char, cap: u32) -> c_int;
    pub fn ab_kernel_embed(s: *mut ab_scheme, table: ab_tensor, step: ab_tensor, x: ab_tensor) -> c_int;
    pub fn ab_kernel_gemv(s: *mut ab_scheme, x: ab_tensor, w: ab_tensor, xout: ab_tensor, step: ab_tensor) -> c_int;
    pub fn ab_kernel_rmsnorm(s: *mut ab_scheme, x: ab_tensor, weight: ab_tensor, o: ab_tensor) -> c_int;
    pub fn ab_kernel_rmsnorm_inplace(s: *mut ab_scheme, x: ab_tensor, weight: ab_tensor) -> c_int;
    pub fn ab_kernel_rope(s: *mut ab_scheme, q: ab_tensor, k: ab_tensor, step: ab_tensor, theta: f32) -> c_int;
    pub fn ab_kernel_rope_store(s: *mut ab_scheme, q: ab_tensor, k_proj: ab_tensor, k: ab_tensor, step: ab_tensor, theta: f32) -> c_int;
    pub fn ab_kernel_cache_store(s: *mut ab_scheme, src: ab_tensor, dst: ab_tensor, step: ab_tensor) -> c_int;
    pub fn ab_kernel_attention_partial(s: *mut ab_scheme, q: ab_tensor, key_cache: ab_tensor, value_cache: ab_tensor, partial: ab_tensor, step: ab_tensor) -> c_int;
    pub fn ab_kernel_attention_combine(s: *mut ab_scheme, partial: ab_tensor, xb: ab_tensor, step: ab_tensor) -> c_int;
    pub fn ab_kernel_attention_decode(s: *mut ab_scheme, q: ab_tensor, key_cache: ab_tensor, value_cache: ab_tensor, out_: ab_tensor, step: ab_tensor) -> c_int;
    pub fn ab_kernel_attention(s: *mut ab_scheme, q: ab_tensor, att: ab_tensor, xb: ab_tensor, key_cache: ab_tensor, value_cache: ab_tensor, step: ab_tensor) -> c_int;
    pub fn ab_kernel_swiglu(s: *mut ab_scheme, hb: ab_tensor, hb2: ab_tensor) -> c_int;
    pub fn ab_tensor_add_into(s: *mut ab_scheme, a: ab_tensor, b: ab_tensor, out_: ab_tensor) -> c_int;
    pub fn ab_tensor_matmul_into(s: *mut ab_scheme, a: ab_tensor, b: ab_tensor, out_: ab_tensor) -> c_int;
    pub fn ab_embedding_record(s: *mut ab_scheme, table: ab_tensor, step: ab_tensor, x: ab_tensor) -> c_int;
    pub fn ab_rmsnorm_record(s: *mut ab_scheme, x: ab_tensor, weight: ab_tensor, out_: ab_tensor) -> c_int;
    pub fn ab_rmsnorm_record_inplace(s: *mut ab_scheme, x: ab_tensor, weight: ab_tensor) -> c_int;
    pub fn ab_linear_record(s: *mut ab_scheme, weight: ab_tensor, x: ab_tensor, out_: ab_tensor) -> c_int;
    pub fn ab_kvcache_create(rt: *mut ab_runtime, layers: u32, seq_len: u32, kv_heads: u32, head_size: u32, dtype: i32, batch: u32, out_: *mut *mut ab_kvcache) -> c_int;
    pub fn ab_kvcache_layer(c: *const ab_kvcache, layer: u32, key: *mut ab_tensor, value: *mut ab_tensor) -> c_int;
    pub fn ab_kvcache_zero(c: *mut ab_kvcache) -> c_int;
    pub fn ab_kvcache_destroy(c: *mut ab_kvcache) -> c_int;
    pub fn ab_attention_block_create(rt: *mut ab_runtime, hidden: u32, query_heads: u32, seq_len: u32, max_batch: u32, rope_theta: f32, out_: *mut *mut ab_attention_block) -> c_int;
    pub fn ab_attention_block_record(b: *mut ab_attention_block, s: *mut ab_scheme, x: ab_tensor, w: *const ab_attention_weights, key: ab_tensor, value: ab_tensor, step: ab_tensor) -> c_int;
    pub fn ab_attention_block_destroy(b: *mut ab_attention_block) -> c_int;
    pub fn ab_swiglu_block_create(rt: *mut ab_runtime, hidden: u32, intermediate: u32, max_batch: u32, out_: *mut *mut ab_swiglu_block) -> c_int;
    pub fn ab_swiglu_block_record(b: *mut ab_swiglu_block, s: *mut ab_scheme, x: ab_tensor, w: *const ab_swiglu_weights) -> c_int;
    pub fn ab_swiglu_block_destroy(b: *mut ab_swiglu_block) -> c_int;
    pub fn ab_attention_decode_noalloc(stream: *mut c_void, q: ab_tensor, key_cache: ab_tensor, value_cache: ab_tensor, out_: ab_tensor, step: ab_tensor) -> c_int;
    pub fn ab_attention_decode_noalloc_status(stream: *mut c_void, flags: *mut u32) -> c_int;
    pub fn ab_sample_argmax(logits: *const f32, n: u32) -> i32;
    pub fn ab_generate_tokens(m: *const ab_autoregressive_model, prompt: *const i32, prompt_len: u32, max_new_tokens: u32, has_stop: i32, stop_on: i32, out_tokens: *mut i32, cap: u32, out_len: *mut u32, tokens_per_second: *mut f64) -> c_int;
    pub fn ab_bpe_from_path(path: *const c_char, vocab_size: u32, out_: *mut *mut ab_bpe) -> c_int;
    pub fn ab_bpe_from_parts(pieces: *const *const c_char, lengths: *const u32, scores: *const f32, n: u32, max_token_length: u32, out_: *mut *mut ab_bpe) -> c_int;
    pub fn ab_bpe_info(t: *const ab_bpe, vocab_size: *mut u32, max_token_length: *mut u32) -> c_int;
    pub fn ab_bpe_encode(t: *const ab_bpe, text: *const c_char, len: usize, bos: i32, eos: i32, out_: *mut i32, cap: u32, n_out: *mut u32) -> c_int;
    pub fn ab_bpe_decode(t: *const ab_bpe, prev_token: i32, token: i32, out_: *mut c_char, cap: u32, n_out: *mut u32) -> c_int;
    pub fn ab_bpe_destroy(t: *mut ab_bpe) -> c_int;
    pub fn ab_llama_create(rt: *mut ab_runtime, cfg: *const ab_llama_config, out_: *mut *mut ab_llama) -> c_int;
    pub fn ab_llama_init_synthetic(m: *mut ab_llama, seed: u64, std: f32) -> c_int;
    pub fn ab_llama_weight(m: *mut ab_llama, which: i32, layer: u32, out_: *mut ab_tensor) -> c_int;
    pub fn ab_llama_cache(m: *mut ab_llama, out_: *mut *mut ab_kvcache) -> c_int;
    pub fn ab_llama_step(m: *mut ab_llama, steps: *const ab_decode_step, n: u32, logits_host: *mut f32, argmax_host: *mut i32) -> c_int;
    pub fn ab_llama_decode_device(m: *mut ab_llama, start: *const ab_decode_step, n: u32, steps: u32, tokens_out: *mut i32) -> c_int;
    pub fn ab_llama_prefill(m: *mut ab_llama, stream: u32, tokens: *const i32, n: u32, pos0: u32, logits_host: *mut f32, argmax_host: *mut i32) -> c_int;
    pub fn ab_llama_prefill_rows(m: *mut ab_llama, rows: u32) -> c_int;
    pub fn ab_llama_prefill_scheme(m: *mut ab_llama, stream: u32, rows: u32, head: i32, out_: *mut *mut ab_scheme) -> c_int;
    pub fn ab_llama_prefill_launches(m: *const ab_llama, out_: *mut u32) -> c_int;
    pub fn ab_llama_generate_tokens(m: *mut ab_llama, prompt: *const i32, prompt_len: u32, max_new_tokens: u32, has_stop: i32, stop_on: i32, out_tokens: *mut i32, cap: u32, out_len: *mut u32, tokens_per_second: *mut f64) -> c_int;
    pub fn ab_llama_step_trace(m: *mut ab_llama, out_: *mut u64, cap: u32, barriers: *mut u32, grid: *mut u32) -> c_int;
    pub fn ab_llama_scheme(m: *mut ab_llama, out_: *mut *mut ab_scheme) -> c_int;
    pub fn ab_llama_logits(m: *mut ab_llama, out_: *mut ab_tensor) -> c_int;
    pub fn ab_llama_reset(m: *mut ab_llama) -> c_int;
    pub fn ab_llama_as_model(m: *mut ab_llama, out_: *mut ab_autoregressive_model) -> c_int;
    pub fn ab_llama_destroy(m: *mut ab_llama) -> c_int;
    pub fn ab_comm_unique_id(id: *mut u8) -> c_int;
    pub fn ab_comm_create_timeout(rt: *mut ab_runtime, id: *const u8, rank: i32, world: i32, timeout_ms: u32, out_: *mut *mut ab_comm) -> c_int;
    pub fn ab_comm_create(rt: *mut ab_runtime, id: *const u8, rank: i32, world: i32, out_: *mut *mut ab_comm) -> c_int;
    pub fn ab_comm_rank(c: *const ab_comm, rank: *mut i32, world: *mut i32) -> c_int;
    pub fn ab_comm_loopback_reduce(rt: *mut ab_runtime, world: u32, ready: u32, n: u32, out_: *mut f32) -> c_int;
    pub fn ab_comm_abort(c: *mut ab_comm) -> c_int;
    pub fn ab_comm_destroy(c: *mut ab_comm) -> c_int;
    pub fn ab_comm_last_error() -> *const c_char;
    pub fn ab_llama_create_tp(rt: *mut ab_runtime, cfg: *const ab_llama_config, comm: *mut ab_comm, out_: *mut *mut ab_llama) -> c_int;
    pub fn ab_llama2c_config(path: *const c_char, batch: u32, dtype: i32, rope_theta: f32, cfg: *mut ab_llama_config) -> c_int;
    pub fn ab_llama_load_llama2c(rt: *mut ab_runtime, path: *const c_char, dtype: i32, batch: u32, rope_theta: f32, comm: *mut ab_comm, cfg_out: *mut ab_llama_config, out_: *mut *mut ab_llama) -> c_int;
}
