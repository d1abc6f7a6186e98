/*
 * ammon_b200 — C ABI of the B200-native Ammon decode layer path.
 *
 * The entry points mirror the public API of the Ammon crate (src/lib.rs re-exports):
 * a runtime (src/gpu.rs), record-then-replay schemes (Goldy's Scheme, used by every
 * module's record()), the DecodeStep control parcel (src/kernels.rs:10-33), the
 * kernels of src/kernels.rs, the modules of src/modules.rs, and the host decode
 * loop (src/generate.rs, src/tokenizer.rs:179-189). Each declaration names the
 * reference item it replaces.
 *
 * Conventions
 *  - Every function returns an int status (AB_OK = 0). On failure ab_last_error()
 *    returns a message for the calling thread. No C++ exception crosses the ABI.
 *  - Record functions validate first. A rejected call adds no node to the scheme
 *    (the reference's "IR node count unchanged" contract, tests/kernels.rs:125-146).
 *  - Tensors are plain descriptors of contiguous row-major device memory. The caller
 *    owns weights, activations and caches; modules own their scratch.
 *  - Nothing runs at record time. ab_scheme_submit() replays the recorded work on the
 *    runtime's stream as one CUDA graph; per-step data changes through
 *    ab_step_deposit() without re-recording.
 */
#ifndef AMMON_B200_H
#define AMMON_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* ---- status ------------------------------------------------------------- */
#define AB_OK 0
#define AB_ERR_VALIDATION 1 /* shape / dtype contract violated (GoldyError::Validation) */
#define AB_ERR_CUDA 2       /* a CUDA runtime call failed */
#define AB_ERR_ARGUMENT 3   /* null handle, bad enum, size out of range */
#define AB_ERR_DEVICE 4     /* a kernel flagged an out-of-range token or position */
#define AB_ERR_NCCL 5       /* a collective failed */

/* Message of the last failed call on this thread ("" if none). */
const char* ab_last_error(void);

/* ---- data types ---------------------------------------------------------- */
typedef enum { AB_F32 = 0, AB_BF16 = 1, AB_U32 = 2 } ab_dtype;

/* Contiguous row-major device tensor view (goldy::TensorView). rank 1..4. */
typedef struct {
    void* data;
    int32_t dtype;
    int32_t rank;
    uint32_t dims[4];
} ab_tensor;

/* DecodeStep { token, position } (src/kernels.rs:10-15). A parcel of n of them is an
 * AB_U32 tensor of dims [n, 2]; entry b drives batch row (stream) b. */
typedef struct {
    uint32_t token;
    uint32_t position;
} ab_decode_step;

typedef struct ab_runtime ab_runtime;
typedef struct ab_scheme ab_scheme;
typedef struct ab_kvcache ab_kvcache;
typedef struct ab_attention_block ab_attention_block;
typedef struct ab_swiglu_block ab_swiglu_block;
typedef struct ab_llama ab_llama;

/* ---- runtime (src/gpu.rs:5-13 create_runtime) ---------------------------- */
int ab_runtime_create(int32_t device, ab_runtime** out);
int ab_runtime_destroy(ab_runtime* rt);
/* Waits for the runtime stream; reports AB_ERR_DEVICE if a kernel flagged a bad index. */
int ab_runtime_synchronize(ab_runtime* rt);
/* The runtime's cudaStream_t, for callers that interleave their own work. */
void* ab_runtime_stream(ab_runtime* rt);
/* Number of SMs of the runtime's device. */
int ab_runtime_sm_count(ab_runtime* rt, int32_t* out);
/* Limit of every bounded wait inside the runtime's kernels (mbarrier rings, grid barriers of
 * the persistent step, peer flags of the all-reduce), in milliseconds; at least 1 ms takes
 * effect. Default 2000, or AMMON_B200_WAIT_MS when the runtime is created. A wait that runs out
 * ends its kernel early and the next synchronising call reports AB_ERR_DEVICE ("bounded wait
 * timed out"); the device stays usable. Synchronises the runtime stream first. No reference
 * counterpart: Goldy has no device-side waits. */
int ab_runtime_set_wait_limit(ab_runtime* rt, uint32_t ms);
int ab_runtime_wait_limit(ab_runtime* rt, uint32_t* ms);
/* Page-locks `bytes` of caller host memory at `ptr` (cudaHostRegister) for as long as the caller
 * keeps it: when the whole logits copy of a step ([n, vocab] floats) lies inside one range
 * registered here, ab_llama_step copies the logits from the device straight into it, without
 * the staging copy; any other buffer still works through the staging copy.
 * ab_host_unregister(ptr), with the `ptr` given to ab_host_register, before the memory is
 * freed. No reference counterpart (the host side of AutoregressiveModel::step,
 * src/model.rs:10). */
int ab_host_register(void* ptr, uint64_t bytes);
int ab_host_unregister(void* ptr);

/* ---- tensors (goldy::Tensor::zeros / from_f32 / host take) ---------------- */
int ab_tensor_zeros(ab_runtime* rt, int32_t dtype, int32_t rank, const uint32_t* dims,
                    ab_tensor* out);
int ab_tensor_free(ab_runtime* rt, ab_tensor* t);
/* Synchronous host -> device copy of `bytes` (must equal the tensor's size). */
int ab_tensor_write(ab_runtime* rt, ab_tensor t, const void* host, uint64_t bytes);
/* Waits for the runtime stream, then device -> host copy. */
int ab_tensor_read(ab_runtime* rt, ab_tensor t, void* host, uint64_t bytes);
/* Seeded synthetic values: mean + std * z with z an Irwin-Hall(12) deviate of a
 * splitmix64 hash of (seed, stream, index). Bit-identical to the CPU generator used by
 * the test oracle. f32 and bf16 tensors. */
int ab_tensor_fill_normal(ab_runtime* rt, ab_tensor t, uint64_t seed, uint64_t stream,
                          float mean, float std);
/* goldy::TensorView::narrow(0, start, len) and reshape: host-side view arithmetic. */
int ab_tensor_narrow(ab_tensor t, uint32_t start, uint32_t len, ab_tensor* out);
int ab_tensor_reshape(ab_tensor t, int32_t rank, const uint32_t* dims, ab_tensor* out);

/* ---- DecodeStep parcel (src/kernels.rs:17-33 parcel / deposit_target) ------- */
/* Device parcel of n zeroed DecodeSteps (AB_U32, dims [n, 2]). Free with ab_tensor_free. */
int ab_step_parcel(ab_runtime* rt, uint32_t n, ab_tensor* out);
/* Deposit: upload n steps, ordered on the runtime stream before later submits
 * (MemoryExchange::bind_deposit + write_data, tests/kernels.rs:202-210). */
int ab_step_deposit(ab_runtime* rt, ab_tensor parcel, const ab_decode_step* steps, uint32_t n);

/* ---- schemes (goldy::Scheme: record, submit, ir_node_count, replay_stats) ---- */
int ab_scheme_create(ab_runtime* rt, ab_scheme** out);
int ab_scheme_destroy(ab_scheme* s);
/* Replays every recorded node on the runtime stream. The first submit after a record
 * captures and instantiates a CUDA graph; later submits relaunch it. */
int ab_scheme_submit(ab_scheme* s);
int ab_scheme_node_count(const ab_scheme* s, uint32_t* out);
/* records = graph instantiations, replays = submits. */
int ab_scheme_replay_stats(const ab_scheme* s, uint32_t* records, uint32_t* replays);
/* enable = 0 launches nodes directly on each submit (debugging); default 1 (graph). */
int ab_scheme_use_graph(ab_scheme* s, int32_t enable);
/* Profiling aid with no reference counterpart (the reference labels dispatches for
 * Goldy's tooling, src/blocks.rs:113-257): launches each recorded node on its own,
 * `iters` times, between CUDA events on the runtime stream, and writes the mean
 * milliseconds per launch of node i to ms[i] (n >= node count). */
int ab_scheme_time_nodes(ab_scheme* s, uint32_t iters, float* ms, uint32_t n);
/* Label of node i ("attn_qkv_rope", "ffn_gate_up_swiglu", ...), NUL-terminated. */
int ab_scheme_node_label(const ab_scheme* s, uint32_t i, char* buf, uint32_t cap);

/* ---- kernels (src/kernels.rs; each records one dispatch) ------------------- */
/* embed (src/kernels.rs:35-47): x[b, :] = table[step[b].token, :]. */
int ab_kernel_embed(ab_scheme* s, ab_tensor table, ab_tensor step, ab_tensor x);
/* gemv (src/kernels.rs:49-73): serial-order xout[pos, i] = sum_j w[i, j] x[j]. */
int ab_kernel_gemv(ab_scheme* s, ab_tensor x, ab_tensor w, ab_tensor xout, ab_tensor step);
/* rmsnorm / rmsnorm_inplace (src/kernels.rs:75-128): one row per block, eps 1e-5. x is
 * [dim] or [rows, dim], f32 or bf16; an in-place norm keeps x's dtype. */
int ab_kernel_rmsnorm(ab_scheme* s, ab_tensor x, ab_tensor weight, ab_tensor o);
int ab_kernel_rmsnorm_inplace(ab_scheme* s, ab_tensor x, ab_tensor weight);
/* rope (src/kernels.rs:130-172): rotates q [heads, head] and row pos of k [seq, kv, head].
 * Batched form: q [batch, heads, head] with one DecodeStep per row; k is shared
 * [seq, kv, head] or per row [>= batch, seq, kv, head]. */
int ab_kernel_rope(ab_scheme* s, ab_tensor q, ab_tensor k, ab_tensor step, float theta);
/* rope_store (src/kernels.rs:174-210). */
int ab_kernel_rope_store(ab_scheme* s, ab_tensor q, ab_tensor k_proj, ab_tensor k,
                         ab_tensor step, float theta);
/* cache_store (src/kernels.rs:212-226). */
int ab_kernel_cache_store(ab_scheme* s, ab_tensor src, ab_tensor dst, ab_tensor step);
/* attention_partial / attention_combine (src/kernels.rs:228-410): flash-decoding with the
 * reference's 8-position splits and partial layout [q_heads, splits, head + 2]. */
int ab_kernel_attention_partial(ab_scheme* s, ab_tensor q, ab_tensor key_cache,
                                ab_tensor value_cache, ab_tensor partial, ab_tensor step);
int ab_kernel_attention_combine(ab_scheme* s, ab_tensor partial, ab_tensor xb, ab_tensor step);
/* The fused replacement of attention_partial + attention_combine (src/kernels.rs:228-410):
 * flash-decoding over positions [0, step.position] in one kernel (TMA-staged K/V tiles, GQA
 * groups share their loads, the last split folds the partials). q f32 [heads, head] with
 * caches [seq, kv_heads, head], or q [batch, heads, head] with caches [>= batch, seq,
 * kv_heads, head] and one DecodeStep per row; out [batch, heads * head] f32 or bf16. Its
 * split scratch is allocated here and owned by the scheme (freed by ab_scheme_destroy),
 * so the scheme must have a runtime. */
int ab_kernel_attention_decode(ab_scheme* s, ab_tensor q, ab_tensor key_cache,
                               ab_tensor value_cache, ab_tensor out, ab_tensor step);
/* attention (src/kernels.rs:412-460): serial scores into att [q_heads, seq]. */
int ab_kernel_attention(ab_scheme* s, ab_tensor q, ab_tensor att, ab_tensor xb,
                        ab_tensor key_cache, ab_tensor value_cache, ab_tensor step);
/* swiglu (src/kernels.rs:462-476): hb = silu(hb) * hb2. */
int ab_kernel_swiglu(ab_scheme* s, ab_tensor hb, ab_tensor hb2);
/* TensorKernels::add_into / matmul_into (src/kernels.rs:506-528). matmul: a is the
 * weight [d_out, d_in], b is x [d_in] or [batch, d_in], out [d_out] or [batch, d_out]. */
int ab_tensor_add_into(ab_scheme* s, ab_tensor a, ab_tensor b, ab_tensor out);
int ab_tensor_matmul_into(ab_scheme* s, ab_tensor a, ab_tensor b, ab_tensor out);

/* ---- modules (src/modules.rs) --------------------------------------------- */
/* Embedding::record (src/modules.rs:111-119). x is [dim] or [batch, dim]. */
int ab_embedding_record(ab_scheme* s, ab_tensor table, ab_tensor step, ab_tensor x);
/* RmsNorm::record / record_inplace (src/modules.rs:146-163). */
int ab_rmsnorm_record(ab_scheme* s, ab_tensor x, ab_tensor weight, ab_tensor out);
int ab_rmsnorm_record_inplace(ab_scheme* s, ab_tensor x, ab_tensor weight);
/* Linear::record (src/modules.rs:178-186): out = weight @ x. */
int ab_linear_record(ab_scheme* s, ab_tensor weight, ab_tensor x, ab_tensor out);

/* KvCache::new / layer (src/modules.rs:38-64): [layers, batch, seq, kv_heads, head].
 * layer() returns [seq, kv_heads, head] views when batch == 1, else
 * [batch, seq, kv_heads, head]. dtype AB_F32 (the reference's) or AB_BF16. */
int ab_kvcache_create(ab_runtime* rt, uint32_t layers, uint32_t seq_len, uint32_t kv_heads,
                      uint32_t head_size, int32_t dtype, uint32_t batch, ab_kvcache** out);
int ab_kvcache_layer(const ab_kvcache* c, uint32_t layer, ab_tensor* key, ab_tensor* value);
int ab_kvcache_zero(ab_kvcache* c);
int ab_kvcache_destroy(ab_kvcache* c);

/* CausalAttentionBlockWeights (src/modules.rs:13-19). */
typedef struct {
    ab_tensor norm, query, key, value, output;
} ab_attention_weights;

/* CausalAttentionBlock::new (src/modules.rs:203-230). The reference signature is
 * (hidden, query_heads, seq_len) with batch 1 and RoPE theta 10000
 * (src/blocks.rs:234); max_batch and rope_theta extend it (pass 1 and 10000 for the
 * reference behaviour). */
int ab_attention_block_create(ab_runtime* rt, uint32_t hidden, uint32_t query_heads,
                              uint32_t seq_len, uint32_t max_batch, float rope_theta,
                              ab_attention_block** out);
/* CausalAttentionBlock::record (src/modules.rs:232-260; op order src/blocks.rs:178-259):
 * RMSNorm, Q/K/V, RoPE with the K/V append at step.position, split attention, output
 * projection and residual add into x. key/value are [B, seq, kv_heads, head] (a cache per
 * row of x) or [seq, kv_heads, head]: one cache that every row appends to and attends over,
 * so rows of x with distinct positions are consecutive tokens of one sequence (a prompt
 * prefilled in one pass; each row attends over positions 0 .. its own). */
int ab_attention_block_record(ab_attention_block* b, ab_scheme* s, ab_tensor x,
                              const ab_attention_weights* w, ab_tensor key, ab_tensor value,
                              ab_tensor step);
int ab_attention_block_destroy(ab_attention_block* b);

/* SwiGluBlockWeights (src/modules.rs:23-28): gate = w1, up = w3, down = w2. */
typedef struct {
    ab_tensor norm, gate, up, down;
} ab_swiglu_weights;

/* SwiGluBlock::new (src/modules.rs:289-298), with max_batch (1 = reference). */
int ab_swiglu_block_create(ab_runtime* rt, uint32_t hidden, uint32_t intermediate,
                           uint32_t max_batch, ab_swiglu_block** out);
/* SwiGluBlock::record (src/modules.rs:300-321; op order src/blocks.rs:262-278). */
int ab_swiglu_block_record(ab_swiglu_block* b, ab_scheme* s, ab_tensor x,
                           const ab_swiglu_weights* w);
int ab_swiglu_block_destroy(ab_swiglu_block* b);

/* ---- allocation-free attention ----------------------------------------------------
 * No counterpart in the reference. Runs the block path's flash-decoding attention
 * (q [heads, head] or [batch, heads, head] f32, caches [seq, kv_heads, head] or
 * [batch, seq, kv_heads, head], out [batch, heads * head], DecodeStep parcel) on `stream`
 * (a cudaStream_t of the current device; NULL = default stream) without allocating any
 * device memory: the split partials and tickets live in one static device array of the
 * library (4 MiB of partials = batch * heads * splits * (head + 2) floats, and 16384
 * tickets = batch * kv_heads). For callers that must not call cudaMalloc/cudaFree, such
 * as hosts whose device memory is owned by their own pooling allocator, or latency-bound
 * loops that cannot take cudaFree's device-wide synchronisation. A shape needing more
 * scratch than the array holds fails with AB_ERR_ARGUMENT before anything is launched.
 * Every call on a device shares the array and it keeps the last call's contents (the
 * tickets are cleared on the stream before each launch): calls that overlap on the GPU
 * race. The first call on each device looks up the array's address with
 * cudaGetSymbolAddress, with that device current; make that first call before any
 * stream capture begins. The looked-up address is kept for the life of the process: after
 * cudaDeviceReset it is stale, so do not call this entry (or its status call) again in a
 * process that reset the device. A row whose position is >= seq produces a zero row and
 * raises a flag, as does a bounded wait inside the kernel that ran out (its row is then
 * incomplete); read the flags with ab_attention_decode_noalloc_status. */
int ab_attention_decode_noalloc(void* stream, ab_tensor q, ab_tensor key_cache,
                                ab_tensor value_cache, ab_tensor out, ab_tensor step);
/* Companion of ab_attention_decode_noalloc (no counterpart in the reference): waits for
 * `stream`, reads and clears the device flag word the allocation-free calls on the current
 * device raise, and returns AB_ERR_DEVICE (message via ab_last_error) if any call since the
 * last status read flagged a position >= seq or a bounded wait that ran out. The raw bits go
 * to *flags (may be NULL). Allocates nothing. */
int ab_attention_decode_noalloc_status(void* stream, uint32_t* flags);

/* ---- host decode loop (src/model.rs, src/generate.rs, src/tokenizer.rs) ------ */
/* sample_argmax (src/tokenizer.rs:179-189): first index of the maximum. */
int32_t ab_sample_argmax(const float* logits, uint32_t n);

/* AutoregressiveModel (src/model.rs:7-11) as a C vtable. step() returns a host
 * pointer to vocab_size logits that stays valid until the next step. */
typedef struct {
    void* self;
    uint32_t (*vocab_size)(void* self);
    uint32_t (*max_seq_len)(void* self);
    int (*step)(void* self, uint32_t token, uint32_t pos, const float** logits);
} ab_autoregressive_model;

/* generate_tokens (src/generate.rs:43-91). Writes up to cap ids to out_tokens and the
 * full count to *out_len; tokens_per_second as the reference computes it. */
int ab_generate_tokens(const ab_autoregressive_model* m, const int32_t* prompt,
                       uint32_t prompt_len, uint32_t max_new_tokens, int32_t has_stop,
                       int32_t stop_on, int32_t* out_tokens, uint32_t cap, uint32_t* out_len,
                       double* tokens_per_second);

/* ---- BPE tokenizer (src/tokenizer.rs:18-178) ---------------------------------------
 * llama2.c tokenizer.bin pieces and scores; encode/decode as BpeTokenizer's Tokenizer impl.
 * Host-only (no GPU needed). */
typedef struct ab_bpe ab_bpe;
/* BpeTokenizer::from_path (src/tokenizer.rs:28-60): u32 max_token_length, then per piece
 * f32 score, i32 length, bytes; pieces are read as UTF-8 with ill-formed bytes replaced. */
int ab_bpe_from_path(const char* path, uint32_t vocab_size, ab_bpe** out);
/* BpeTokenizer::from_parts (src/tokenizer.rs:62-74): n pieces given as bytes + lengths. */
int ab_bpe_from_parts(const char* const* pieces, const uint32_t* lengths, const float* scores,
                      uint32_t n, uint32_t max_token_length, ab_bpe** out);
/* vocab_size / max_token_length (either pointer may be NULL). */
int ab_bpe_info(const ab_bpe* t, uint32_t* vocab_size, uint32_t* max_token_length);
/* Tokenizer::encode (src/tokenizer.rs:101-160) of len UTF-8 bytes: writes the first
 * min(n, cap) ids to out (may be NULL) and n to *n_out. */
int ab_bpe_encode(const ab_bpe* t, const char* text, size_t len, int32_t bos, int32_t eos,
                  int32_t* out, uint32_t cap, uint32_t* n_out);
/* Tokenizer::decode (src/tokenizer.rs:162-172): the UTF-8 bytes of the piece (first
 * min(n, cap) into out, not NUL-terminated) and n in *n_out. */
int ab_bpe_decode(const ab_bpe* t, int32_t prev_token, int32_t token, char* out, uint32_t cap,
                  uint32_t* n_out);
int ab_bpe_destroy(ab_bpe* t);

/* ---- Llama-shaped model assembly ----------------------------------------------
 * The reference leaves model assembly to architecture crates (README.md:5,21). This
 * is the llama2.c-layout composition the harness and benchmark use: Embedding,
 * layers x [CausalAttentionBlock, SwiGluBlock], final RmsNorm, classifier Linear. */
typedef struct {
    uint32_t dim, layers, heads, kv_heads, head_dim, hidden, vocab, seq, batch;
    float rope_theta, norm_eps;
    int32_t dtype; /* AB_F32: fp32 everywhere; AB_BF16: bf16 weights and KV cache */
} ab_llama_config;

int ab_llama_create(ab_runtime* rt, const ab_llama_config* cfg, ab_llama** out);
/* Seeded synthetic weights, the same streams the CPU oracle uses. */
int ab_llama_init_synthetic(ab_llama* m, uint64_t seed, float std);
/* Weight view: which = 0 embed, 1 wcls, 2 rms_final, 3 rms_att, 4 wq, 5 wk, 6 wv, 7 wo,
 * 8 rms_ffn, 9 w1, 10 w2, 11 w3. */
int ab_llama_weight(ab_llama* m, int32_t which, uint32_t layer, ab_tensor* out);
/* KV cache of the model (for inspection). */
int ab_llama_cache(ab_llama* m, ab_kvcache** out);
/* One batched decode step: deposits n = batch steps and replays the step graph.
 * logits_host (may be NULL) receives [batch, vocab] fp32; argmax_host (may be NULL)
 * receives [batch] ids from the device argmax (same tie rule as sample_argmax). */
int ab_llama_step(ab_llama* m, const ab_decode_step* steps, uint32_t n, float* logits_host,
                  int32_t* argmax_host);
/* Greedy decode of `steps` tokens with no host round-trip: the argmax of
 * src/tokenizer.rs:179-189 runs on the device and feeds the next step. Deposits the
 * n = batch `start` steps, then replays the step graph `steps` times, each replay
 * feeding its argmax back as the next DecodeStep {token, position + 1}. tokens_out
 * (may be NULL) receives [steps, batch] ids. A row whose position reaches seq_len stops
 * advancing and raises AB_ERR_DEVICE at the end. */
int ab_llama_decode_device(ab_llama* m, const ab_decode_step* start, uint32_t n, uint32_t steps,
                           int32_t* tokens_out);
/* Batched prefill of one cache stream (batch row `stream`): the n tokens at positions
 * pos0 .. pos0 + n - 1 run as the rows of passes of up to R rows, so each weight is read once
 * per pass instead of once per token, where generate_tokens feeds a prompt one DecodeStep at
 * a time (src/generate.rs:60-66). The K/V cache ends as that loop leaves it (within the
 * arithmetic's rounding). logits_host (may be NULL) receives the last token's [vocab] logits,
 * argmax_host (may be NULL) its greedy id. R is 256 unless set by ab_llama_prefill_rows (or
 * AMMON_B200_PREFILL_ROWS) and at most seq_len. Under tensor parallelism every rank makes the
 * same call. */
int ab_llama_prefill(ab_llama* m, uint32_t stream, const int32_t* tokens, uint32_t n,
                     uint32_t pos0, float* logits_host, int32_t* argmax_host);
/* Rows per prefill pass (1..256; 0 = the default); takes effect at the next prefill. */
int ab_llama_prefill_rows(ab_llama* m, uint32_t rows);
/* The recorded prefill pass of `rows` positions of `stream` (with the classifier when head
 * is non-zero), for profiling: it reads the DecodeSteps the last prefill deposited. Owned by
 * the model; a later prefill may drop it. */
int ab_llama_prefill_scheme(ab_llama* m, uint32_t stream, uint32_t rows, int32_t head,
                            ab_scheme** out);
/* Graph nodes (kernels and collectives) the last prefill launched over all its passes. */
int ab_llama_prefill_launches(const ab_llama* m, uint32_t* out);
/* generate_tokens (src/generate.rs:43-91) on a batch-1 model, same arguments and results as
 * ab_generate_tokens, with the prompt run by ab_llama_prefill and each generated token by one
 * step with the device argmax (4 bytes read back). tokens_per_second counts the generated
 * tokens after the first (the prompt's pick) over the time from that pick on. */
int ab_llama_generate_tokens(ab_llama* m, const int32_t* prompt, uint32_t prompt_len,
                             uint32_t max_new_tokens, int32_t has_stop, int32_t stop_on,
                             int32_t* out_tokens, uint32_t cap, uint32_t* out_len,
                             double* tokens_per_second);
/* Profiling aid with no reference counterpart: when the model runs its decode step as the
 * persistent single launch (batch 1, bf16; AMMON_B200_STEP_TRACE set at model creation),
 * %globaltimer nanoseconds of each CTA at each grid barrier of the last step,
 * [barriers][4][grid]: its arrival, its release, when it had staged the operand of the phase
 * that ends at that barrier (0 where no phase stages one), and at the barrier after a
 * tensor-parallel all-reduce site when it had pushed its partial rows to every rank and began
 * to wait for the other ranks' (0 at other barriers); the first min(cap, 4 * barriers * grid)
 * values. *barriers and *grid are 0 when no trace is kept. */
int ab_llama_step_trace(ab_llama* m, uint64_t* out, uint32_t cap, uint32_t* barriers,
                        uint32_t* grid);
/* The model's step scheme (recorded on first use), for profiling. */
int ab_llama_scheme(ab_llama* m, ab_scheme** out);
/* Device logits [batch, vocab] of the last step. */
int ab_llama_logits(ab_llama* m, ab_tensor* out);
/* Zero the KV cache (a new sequence). */
int ab_llama_reset(ab_llama* m);
/* AutoregressiveModel view of a batch-1 model (logits read back to the host). */
int ab_llama_as_model(ab_llama* m, ab_autoregressive_model* out);
int ab_llama_destroy(ab_llama* m);

/* ---- tensor parallelism over NVLink (NCCL) --------------------------------------
 * No counterpart in the reference (it runs on one device). One process per GPU; the
 * communicator wraps NCCL, loaded at run time (the process's already-loaded
 * libnccl.so.2 when there is one). Collectives are recorded into schemes and captured
 * into the step graph like kernels. */
typedef struct ab_comm ab_comm;
#define AB_COMM_ID_BYTES 128
/* A fresh communicator id (rank 0 makes it and shares it with the other ranks). */
int ab_comm_unique_id(uint8_t* id);
/* Joins the communicator of `world` ranks that `id` names. A rank that never joins ends the
 * call on the others with AB_ERR_NCCL after timeout_ms (the rendezvous communicator is
 * aborted with ncclCommAbort) instead of blocking it; ab_comm_create takes the timeout from
 * AMMON_B200_COMM_TIMEOUT_MS, default 300000. */
int ab_comm_create_timeout(ab_runtime* rt, const uint8_t* id, int32_t rank, int32_t world,
                           uint32_t timeout_ms, ab_comm** out);
int ab_comm_create(ab_runtime* rt, const uint8_t* id, int32_t rank, int32_t world,
                   ab_comm** out);
int ab_comm_rank(const ab_comm* c, int32_t* rank, int32_t* world);
/* Diagnostic of the all-reduce's bounded wait, on one GPU: runs the tensor-parallel
 * all-reduce kernel over `world` (1..8) ranks whose partials (rank r: r + 1 + 0.25*(i % 7))
 * and arrival words all sit in this GPU's memory. Rank 0 is this process; rank r > 0 has
 * arrived when bit r of `ready` is set and never arrives otherwise. out (n floats, host)
 * receives the rank-ordered sum; with a rank missing the kernel gives up after the
 * runtime's wait limit and the call returns AB_ERR_DEVICE ("bounded wait timed out"). */
int ab_comm_loopback_reduce(ab_runtime* rt, uint32_t world, uint32_t ready, uint32_t n,
                            float* out);
/* Aborts outstanding collectives (error paths); destroy still frees the handle. */
int ab_comm_abort(ab_comm* c);
int ab_comm_destroy(ab_comm* c);
/* NCCL's message for the last collective that failed inside a submit on this thread. */
const char* ab_comm_last_error(void);

/* Tensor-parallel Llama-shaped model: query heads, kv heads, SwiGLU columns and the
 * vocabulary are split evenly over the communicator's ranks (each must divide); wq, wk,
 * wv, w1, w3 and the classifier are row shards, wo and w2 column shards. The residual
 * stream is replicated: after wo and after w2 one all-reduce sums the ranks' partial
 * projections into it. The greedy pick takes every rank's best (value, id) and keeps
 * the first maximum, the sample_argmax rule. Every rank must make the same calls. */
int ab_llama_create_tp(ab_runtime* rt, const ab_llama_config* cfg, ab_comm* comm,
                       ab_llama** out);

/* llama2.c checkpoint (no counterpart in the reference, which leaves checkpoints to
 * architecture crates, README.md:5,21): seven int32 (dim, hidden_dim, n_layers, n_heads,
 * n_kv_heads, vocab_size -- negative for a classifier of its own --, seq_len) then the fp32
 * tensors of llama2.c's run.c layout. ab_llama2c_config reads and size-checks the header
 * only (no GPU needed); ab_llama_load_llama2c creates the model (this rank's shard when
 * comm is not NULL), converts the weights to `dtype` (AB_F32 or AB_BF16) and uploads them.
 * cfg_out may be NULL. */
int ab_llama2c_config(const char* path, uint32_t batch, int32_t dtype, float rope_theta,
                      ab_llama_config* cfg);
int ab_llama_load_llama2c(ab_runtime* rt, const char* path, int32_t dtype, uint32_t batch,
                          float rope_theta, ab_comm* comm, ab_llama_config* cfg_out,
                          ab_llama** out);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif
#endif /* AMMON_B200_H */
