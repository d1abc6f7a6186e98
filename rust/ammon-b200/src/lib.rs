//! The decode-path API of the Ammon crate (`src/lib.rs` re-exports: `Embedding`, `RmsNorm`,
//! `Linear`, `CausalAttentionBlock`, `SwiGluBlock`, `KvCache`, `KvLayer`, `DecodeStep`,
//! `AutoregressiveModel`, `generate_tokens`, `sample_argmax`, `BpeTokenizer`) with its bodies on
//! libammon_b200: every `record` validates, then appends the B200 kernels to the scheme, and
//! `Scheme::submit` replays them as one CUDA graph. Host logic (the greedy loop, the tokenizer
//! trait) stays in Rust, as the crate has it.
//!
//! Differences from the Goldy-typed original: tensors are [`Tensor`] device views instead of
//! `goldy::TensorView`, errors are [`AmmonError`] (status code + the library's message), and
//! `AutoregressiveModel::step` returns a borrowed host slice of logits.
use ammon_b200_sys as sys;
use std::ffi::{CStr, CString};
use std::os::raw::c_int;
use std::time::Instant;

pub use sys::{AB_BF16, AB_F32, AB_U32};

/// A failed library call: the `AB_ERR_*` status and `ab_last_error()`'s text.
#[derive(Debug, Clone)]
pub struct AmmonError {
    pub code: i32,
    pub message: String,
}

impl std::fmt::Display for AmmonError {
    fn fmt(&self, f: &mut std::fmt::Formatter<'_>) -> std::fmt::Result {
        write!(f, "ammon_b200 error {}: {}", self.code, self.message)
    }
}

impl std::error::Error for AmmonError {}

pub type Result<T> = std::result::Result<T, AmmonError>;

fn check(status: c_int) -> Result<()> {
    if status == sys::AB_OK {
        return Ok(());
    }
    let message = unsafe {
        let p = sys::ab_last_error();
        if p.is_null() { String::new() } else { CStr::from_ptr(p).to_string_lossy().into_owned() }
    };
    Err(AmmonError { code: status, message })
}

fn argument(message: &str) -> AmmonError {
    AmmonError { code: sys::AB_ERR_ARGUMENT, message: message.to_string() }
}

// ---- runtime, tensors, schemes -----------------------------------------------------------

/// One GPU and its stream (`gpu::create_runtime`, src/gpu.rs:5-13).
pub struct Runtime {
    raw: *mut sys::ab_runtime,
}

impl Runtime {
    pub fn new(device: i32) -> Result<Self> {
        let mut raw = std::ptr::null_mut();
        check(unsafe { sys::ab_runtime_create(device, &mut raw) })?;
        Ok(Runtime { raw })
    }

    pub fn synchronize(&self) -> Result<()> {
        check(unsafe { sys::ab_runtime_synchronize(self.raw) })
    }

    /// Uploads DecodeSteps into a retained parcel, ordered before later submits
    /// (`MemoryExchange::bind_deposit`).
    pub fn deposit(&self, parcel: &Tensor, steps: &[DecodeStep]) -> Result<()> {
        let raw: Vec<sys::ab_decode_step> = steps
            .iter()
            .map(|s| sys::ab_decode_step { token: s.token, position: s.position })
            .collect();
        check(unsafe { sys::ab_step_deposit(self.raw, parcel.raw, raw.as_ptr(), raw.len() as u32) })
    }

    pub fn as_raw(&self) -> *mut sys::ab_runtime {
        self.raw
    }
}

impl Drop for Runtime {
    fn drop(&mut self) {
        unsafe { sys::ab_runtime_destroy(self.raw) };
    }
}

/// A contiguous row-major device tensor: owned (freed on drop) or a view of another one.
pub struct Tensor {
    raw: sys::ab_tensor,
    owner: Option<*mut sys::ab_runtime>,
}

impl Tensor {
    pub fn zeros(rt: &Runtime, dims: &[u32], dtype: i32) -> Result<Self> {
        let mut raw = empty_tensor();
        check(unsafe {
            sys::ab_tensor_zeros(rt.raw, dtype, dims.len() as i32, dims.as_ptr(), &mut raw)
        })?;
        Ok(Tensor { raw, owner: Some(rt.raw) })
    }

    /// A non-owning view of `raw` (the caller keeps the memory alive).
    pub fn view_of(raw: sys::ab_tensor) -> Self {
        Tensor { raw, owner: None }
    }

    pub fn dims(&self) -> &[u32] {
        &self.raw.dims[..self.raw.rank as usize]
    }

    pub fn numel(&self) -> usize {
        self.dims().iter().map(|&d| d as usize).product()
    }

    /// `TensorView::narrow(0, start, len)`.
    pub fn narrow(&self, start: u32, len: u32) -> Result<Tensor> {
        let mut out = empty_tensor();
        check(unsafe { sys::ab_tensor_narrow(self.raw, start, len, &mut out) })?;
        Ok(Tensor::view_of(out))
    }

    pub fn reshape(&self, dims: &[u32]) -> Result<Tensor> {
        let mut out = empty_tensor();
        check(unsafe { sys::ab_tensor_reshape(self.raw, dims.len() as i32, dims.as_ptr(), &mut out) })?;
        Ok(Tensor::view_of(out))
    }

    /// Synchronous host -> device copy of exactly the tensor's bytes (f32 / u32 elements, or
    /// u16 bf16 bits for a bf16 tensor).
    pub fn write<T: Copy>(&self, rt: &Runtime, host: &[T]) -> Result<()> {
        let bytes = std::mem::size_of_val(host) as u64;
        check(unsafe { sys::ab_tensor_write(rt.raw, self.raw, host.as_ptr() as *const _, bytes) })
    }

    /// Waits for the stream, then device -> host.
    pub fn read<T: Copy + Default>(&self, rt: &Runtime) -> Result<Vec<T>> {
        let elem = if self.raw.dtype == AB_BF16 { 2 } else { 4 };
        if std::mem::size_of::<T>() != elem {
            return Err(argument("host element size does not match the tensor's dtype"));
        }
        let mut out = vec![T::default(); self.numel()];
        let bytes = (out.len() * elem) as u64;
        check(unsafe { sys::ab_tensor_read(rt.raw, self.raw, out.as_mut_ptr() as *mut _, bytes) })?;
        Ok(out)
    }

    /// Seeded synthetic values (the CPU oracle's generator).
    pub fn fill_normal(&self, rt: &Runtime, seed: u64, stream: u64, mean: f32, std: f32) -> Result<()> {
        check(unsafe { sys::ab_tensor_fill_normal(rt.raw, self.raw, seed, stream, mean, std) })
    }

    pub fn as_raw(&self) -> sys::ab_tensor {
        self.raw
    }
}

impl Drop for Tensor {
    fn drop(&mut self) {
        if let Some(rt) = self.owner {
            unsafe { sys::ab_tensor_free(rt, &mut self.raw) };
        }
    }
}

fn empty_tensor() -> sys::ab_tensor {
    sys::ab_tensor { data: std::ptr::null_mut(), dtype: 0, rank: 0, dims: [0; 4] }
}

/// Record-then-replay list of dispatches (`goldy::Scheme`).
pub struct Scheme {
    raw: *mut sys::ab_scheme,
}

impl Scheme {
    pub fn new(rt: &Runtime) -> Result<Self> {
        let mut raw = std::ptr::null_mut();
        check(unsafe { sys::ab_scheme_create(rt.raw, &mut raw) })?;
        Ok(Scheme { raw })
    }

    pub fn submit(&mut self) -> Result<()> {
        check(unsafe { sys::ab_scheme_submit(self.raw) })
    }

    pub fn ir_node_count(&self) -> Result<u32> {
        let mut n = 0;
        check(unsafe { sys::ab_scheme_node_count(self.raw, &mut n) })?;
        Ok(n)
    }

    /// (graph instantiations, submits).
    pub fn replay_stats(&self) -> Result<(u32, u32)> {
        let (mut rec, mut rep) = (0, 0);
        check(unsafe { sys::ab_scheme_replay_stats(self.raw, &mut rec, &mut rep) })?;
        Ok((rec, rep))
    }
}

impl Drop for Scheme {
    fn drop(&mut self) {
        unsafe { sys::ab_scheme_destroy(self.raw) };
    }
}

// ---- DecodeStep (src/kernels.rs:10-33) ---------------------------------------------------

#[derive(Clone, Copy, Debug, Default, PartialEq, Eq)]
pub struct DecodeStep {
    pub token: u32,
    pub position: u32,
}

impl DecodeStep {
    /// A retained device parcel of `n` zeroed DecodeSteps (`DecodeStep::parcel`).
    pub fn parcel(rt: &Runtime, n: u32) -> Result<Tensor> {
        let mut raw = empty_tensor();
        check(unsafe { sys::ab_step_parcel(rt.raw, n, &mut raw) })?;
        Ok(Tensor { raw, owner: Some(rt.raw) })
    }
}

// ---- modules (src/modules.rs) ------------------------------------------------------------

pub struct Embedding {
    _rt: *mut sys::ab_runtime,
}

impl Embedding {
    pub fn new(rt: &Runtime) -> Result<Self> {
        Ok(Embedding { _rt: rt.raw })
    }

    pub fn record(&self, scheme: &mut Scheme, table: &Tensor, step: &Tensor, x: &Tensor) -> Result<()> {
        check(unsafe { sys::ab_embedding_record(scheme.raw, table.raw, step.raw, x.raw) })
    }
}

pub struct RmsNorm {
    _rt: *mut sys::ab_runtime,
}

impl RmsNorm {
    pub fn new(rt: &Runtime) -> Result<Self> {
        Ok(RmsNorm { _rt: rt.raw })
    }

    pub fn record(&self, scheme: &mut Scheme, x: &Tensor, weight: &Tensor, out: &Tensor) -> Result<()> {
        check(unsafe { sys::ab_rmsnorm_record(scheme.raw, x.raw, weight.raw, out.raw) })
    }

    pub fn record_inplace(&self, scheme: &mut Scheme, x: &Tensor, weight: &Tensor) -> Result<()> {
        check(unsafe { sys::ab_rmsnorm_record_inplace(scheme.raw, x.raw, weight.raw) })
    }
}

pub struct Linear {
    _rt: *mut sys::ab_runtime,
}

impl Linear {
    pub fn new(rt: &Runtime) -> Result<Self> {
        Ok(Linear { _rt: rt.raw })
    }

    /// out = weight @ x.
    pub fn record(&self, scheme: &mut Scheme, weight: &Tensor, x: &Tensor, out: &Tensor) -> Result<()> {
        check(unsafe { sys::ab_linear_record(scheme.raw, weight.raw, x.raw, out.raw) })
    }
}

/// One layer's K and V cache views (`KvLayer`).
pub struct KvLayer {
    pub key: Tensor,
    pub value: Tensor,
}

/// Persistent `[layers, batch, seq, kv_heads, head]` cache (`KvCache`).
pub struct KvCache {
    raw: *mut sys::ab_kvcache,
}

impl KvCache {
    /// `KvCache::new(runtime, layers, seq, kv_heads, head)`: fp32, one stream.
    pub fn new(rt: &Runtime, layers: u32, seq_len: u32, kv_heads: u32, head_size: u32) -> Result<Self> {
        Self::with_options(rt, layers, seq_len, kv_heads, head_size, AB_F32, 1)
    }

    /// bf16 storage and more streams (`batch` caches) than the reference's one.
    pub fn with_options(rt: &Runtime, layers: u32, seq_len: u32, kv_heads: u32, head_size: u32,
                        dtype: i32, batch: u32) -> Result<Self> {
        let mut raw = std::ptr::null_mut();
        check(unsafe {
            sys::ab_kvcache_create(rt.raw, layers, seq_len, kv_heads, head_size, dtype, batch, &mut raw)
        })?;
        Ok(KvCache { raw })
    }

    pub fn layer(&self, layer: u32) -> Result<KvLayer> {
        let (mut k, mut v) = (empty_tensor(), empty_tensor());
        check(unsafe { sys::ab_kvcache_layer(self.raw, layer, &mut k, &mut v) })?;
        Ok(KvLayer { key: Tensor::view_of(k), value: Tensor::view_of(v) })
    }

    pub fn zero(&mut self) -> Result<()> {
        check(unsafe { sys::ab_kvcache_zero(self.raw) })
    }
}

impl Drop for KvCache {
    fn drop(&mut self) {
        unsafe { sys::ab_kvcache_destroy(self.raw) };
    }
}

pub struct CausalAttentionBlockWeights<'a> {
    pub norm: &'a Tensor,
    pub query: &'a Tensor,
    pub key: &'a Tensor,
    pub value: &'a Tensor,
    pub output: &'a Tensor,
}

pub struct SwiGluBlockWeights<'a> {
    pub norm: &'a Tensor,
    pub gate: &'a Tensor,
    pub up: &'a Tensor,
    pub down: &'a Tensor,
}

/// Pre-norm causal attention with RoPE and the K/V append (`CausalAttentionBlock`).
pub struct CausalAttentionBlock {
    raw: *mut sys::ab_attention_block,
}

impl CausalAttentionBlock {
    /// `CausalAttentionBlock::new(runtime, hidden, query_heads, seq_len)`: batch 1, RoPE theta
    /// 10000, as the reference has them.
    pub fn new(rt: &Runtime, hidden: u32, query_heads: u32, seq_len: u32) -> Result<Self> {
        Self::with_options(rt, hidden, query_heads, seq_len, 1, 10000.0)
    }

    pub fn with_options(rt: &Runtime, hidden: u32, query_heads: u32, seq_len: u32, max_batch: u32,
                        rope_theta: f32) -> Result<Self> {
        let mut raw = std::ptr::null_mut();
        check(unsafe {
            sys::ab_attention_block_create(rt.raw, hidden, query_heads, seq_len, max_batch,
                                           rope_theta, &mut raw)
        })?;
        Ok(CausalAttentionBlock { raw })
    }

    pub fn record(&self, scheme: &mut Scheme, x: &Tensor, weights: &CausalAttentionBlockWeights,
                  cache: &KvLayer, step: &Tensor) -> Result<()> {
        let w = sys::ab_attention_weights {
            norm: weights.norm.raw,
            query: weights.query.raw,
            key: weights.key.raw,
            value: weights.value.raw,
            output: weights.output.raw,
        };
        check(unsafe {
            sys::ab_attention_block_record(self.raw, scheme.raw, x.raw, &w, cache.key.raw,
                                           cache.value.raw, step.raw)
        })
    }
}

impl Drop for CausalAttentionBlock {
    fn drop(&mut self) {
        unsafe { sys::ab_attention_block_destroy(self.raw) };
    }
}

/// Pre-norm SwiGLU feed-forward block (`SwiGluBlock`).
pub struct SwiGluBlock {
    raw: *mut sys::ab_swiglu_block,
}

impl SwiGluBlock {
    pub fn new(rt: &Runtime, hidden: u32, intermediate: u32) -> Result<Self> {
        Self::with_batch(rt, hidden, intermediate, 1)
    }

    pub fn with_batch(rt: &Runtime, hidden: u32, intermediate: u32, max_batch: u32) -> Result<Self> {
        let mut raw = std::ptr::null_mut();
        check(unsafe { sys::ab_swiglu_block_create(rt.raw, hidden, intermediate, max_batch, &mut raw) })?;
        Ok(SwiGluBlock { raw })
    }

    pub fn record(&self, scheme: &mut Scheme, x: &Tensor, weights: &SwiGluBlockWeights) -> Result<()> {
        let w = sys::ab_swiglu_weights {
            norm: weights.norm.raw,
            gate: weights.gate.raw,
            up: weights.up.raw,
            down: weights.down.raw,
        };
        check(unsafe { sys::ab_swiglu_block_record(self.raw, scheme.raw, x.raw, &w) })
    }
}

impl Drop for SwiGluBlock {
    fn drop(&mut self) {
        unsafe { sys::ab_swiglu_block_destroy(self.raw) };
    }
}

// ---- model contract and the greedy loop (src/model.rs, src/generate.rs) -------------------

/// One-token-at-a-time generator: `step` gives the vocabulary logits of `(token, pos)`.
pub trait AutoregressiveModel {
    fn vocab_size(&self) -> usize;
    fn max_seq_len(&self) -> u32;
    fn step(&mut self, token: u32, pos: u32) -> Result<&[f32]>;
}

/// First index of the maximum logit (ties keep the lowest index).
pub fn sample_argmax(logits: &[f32]) -> i32 {
    let mut best = 0usize;
    for (i, &v) in logits.iter().enumerate().skip(1) {
        if v > logits[best] {
            best = i;
        }
    }
    best as i32
}

#[derive(Debug, Clone)]
pub struct GenerateTokenOutput {
    pub tokens: Vec<i32>,
    pub prompt_tokens: usize,
    pub tokens_per_second: f64,
}

/// Greedy decode with the reference loop's contract: the prompt is fed one position at a time
/// (its ids forced as the next tokens), then each next id is the logits' first maximum; steps run
/// while pos < min(max_new_tokens, max_seq_len) - 1, a next id equal to `stop_on` ends the loop
/// before it is emitted, and tokens/s counts positions after the first over the time from the
/// first emitted token.
pub fn generate_tokens<M: AutoregressiveModel>(model: &mut M, prompt_tokens: &[i32],
                                                max_new_tokens: u32, stop_on: Option<i32>)
                                                -> Result<GenerateTokenOutput> {
    if prompt_tokens.is_empty() {
        return Err(argument("expected at least one prompt token"));
    }
    let limit = max_new_tokens.min(model.max_seq_len()).saturating_sub(1);
    let mut tokens = Vec::new();
    let mut current = prompt_tokens[0] as u32;
    let mut pos = 0u32;
    let mut started: Option<Instant> = None;
    while pos < limit {
        let next = {
            let logits = model.step(current, pos)?;
            match prompt_tokens.get(pos as usize + 1) {
                Some(&forced) => forced,
                None => sample_argmax(logits),
            }
        };
        pos += 1;
        if stop_on == Some(next) {
            break;
        }
        tokens.push(next);
        current = next as u32;
        started.get_or_insert_with(Instant::now);
    }
    let secs = started.map(|t| t.elapsed().as_secs_f64()).unwrap_or(0.0);
    let tokens_per_second = if secs > 0.0 { pos.saturating_sub(1) as f64 / secs } else { 0.0 };
    Ok(GenerateTokenOutput { tokens, prompt_tokens: prompt_tokens.len(), tokens_per_second })
}

/// Llama-shaped model assembled by the library (llama2.c layout), batch 1 through the trait.
pub struct LlamaModel {
    raw: *mut sys::ab_llama,
    cfg: sys::ab_llama_config,
    logits: Vec<f32>,
}

impl LlamaModel {
    pub fn new(rt: &Runtime, cfg: sys::ab_llama_config) -> Result<Self> {
        let mut raw = std::ptr::null_mut();
        check(unsafe { sys::ab_llama_create(rt.raw, &cfg, &mut raw) })?;
        Ok(LlamaModel { raw, cfg, logits: vec![0.0; (cfg.batch * cfg.vocab) as usize] })
    }

    /// llama2.c checkpoint (`run.c` layout), converted to `dtype`.
    pub fn from_llama2c(rt: &Runtime, path: &str, dtype: i32, rope_theta: f32) -> Result<Self> {
        let c = CString::new(path).map_err(|_| argument("path contains a NUL byte"))?;
        let mut raw = std::ptr::null_mut();
        let mut cfg = sys::ab_llama_config::default();
        check(unsafe {
            sys::ab_llama_load_llama2c(rt.raw, c.as_ptr(), dtype, 1, rope_theta,
                                       std::ptr::null_mut(), &mut cfg, &mut raw)
        })?;
        Ok(LlamaModel { raw, cfg, logits: vec![0.0; cfg.vocab as usize] })
    }

    pub fn init_synthetic(&mut self, seed: u64, std: f32) -> Result<()> {
        check(unsafe { sys::ab_llama_init_synthetic(self.raw, seed, std) })
    }

    /// Greedy decode of `steps` tokens on the device (argmax and the next DecodeStep there).
    pub fn decode_device(&mut self, start: &[DecodeStep], steps: u32) -> Result<Vec<i32>> {
        let raw: Vec<sys::ab_decode_step> = start
            .iter()
            .map(|s| sys::ab_decode_step { token: s.token, position: s.position })
            .collect();
        let mut out = vec![0i32; steps as usize * raw.len()];
        check(unsafe {
            sys::ab_llama_decode_device(self.raw, raw.as_ptr(), raw.len() as u32, steps, out.as_mut_ptr())
        })?;
        Ok(out)
    }

    pub fn reset(&mut self) -> Result<()> {
        check(unsafe { sys::ab_llama_reset(self.raw) })
    }
}

impl AutoregressiveModel for LlamaModel {
    fn vocab_size(&self) -> usize {
        self.cfg.vocab as usize
    }

    fn max_seq_len(&self) -> u32 {
        self.cfg.seq
    }

    fn step(&mut self, token: u32, pos: u32) -> Result<&[f32]> {
        if self.cfg.batch != 1 {
            return Err(argument("AutoregressiveModel::step needs a batch-1 model"));
        }
        let s = sys::ab_decode_step { token, position: pos };
        check(unsafe {
            sys::ab_llama_step(self.raw, &s, 1, self.logits.as_mut_ptr(), std::ptr::null_mut())
        })?;
        Ok(&self.logits[..self.cfg.vocab as usize])
    }
}

impl Drop for LlamaModel {
    fn drop(&mut self) {
        unsafe { sys::ab_llama_destroy(self.raw) };
    }
}

// ---- tokenizer (src/tokenizer.rs) ---------------------------------------------------------

pub trait Tokenizer {
    fn vocab_size(&self) -> usize;
    fn encode(&self, text: &str, bos: bool, eos: bool) -> Vec<i32>;
    fn decode(&self, prev_token: i32, token: i32) -> String;
}

/// llama2.c `tokenizer.bin` BPE, run by the library's host code (`BpeTokenizer`).
pub struct BpeTokenizer {
    raw: *mut sys::ab_bpe,
    vocab: usize,
}

impl BpeTokenizer {
    pub fn from_path(path: &str, vocab_size: usize) -> Result<Self> {
        let c = CString::new(path).map_err(|_| argument("path contains a NUL byte"))?;
        let mut raw = std::ptr::null_mut();
        check(unsafe { sys::ab_bpe_from_path(c.as_ptr(), vocab_size as u32, &mut raw) })?;
        Ok(BpeTokenizer { raw, vocab: vocab_size })
    }
}

impl Tokenizer for BpeTokenizer {
    fn vocab_size(&self) -> usize {
        self.vocab
    }

    fn encode(&self, text: &str, bos: bool, eos: bool) -> Vec<i32> {
        let cap = text.len() as u32 + 3;
        let mut out = vec![0i32; cap as usize];
        let mut n = 0u32;
        let status = unsafe {
            sys::ab_bpe_encode(self.raw, text.as_ptr() as *const _, text.len(), bos as i32,
                               eos as i32, out.as_mut_ptr(), cap, &mut n)
        };
        if status != sys::AB_OK {
            return Vec::new();
        }
        out.truncate(n as usize);
        out
    }

    fn decode(&self, prev_token: i32, token: i32) -> String {
        let mut n = 0u32;
        unsafe { sys::ab_bpe_decode(self.raw, prev_token, token, std::ptr::null_mut(), 0, &mut n) };
        let mut buf = vec![0u8; n as usize];
        unsafe {
            sys::ab_bpe_decode(self.raw, prev_token, token, buf.as_mut_ptr() as *mut _, n, &mut n)
        };
        String::from_utf8_lossy(&buf).into_owned()
    }
}

impl Drop for BpeTokenizer {
    fn drop(&mut self) {
        unsafe { sys::ab_bpe_destroy(self.raw) };
    }
}
