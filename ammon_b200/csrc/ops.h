// Host-side interfaces of the fused decode kernels (gemv.cu, attention.cu).
#pragma once

#include <cuda.h>

#include "internal.h"

namespace ab {

struct Step;

// Encodes a 2-D tiled TMA descriptor over a row-major [rows, inner] tensor (row stride in
// bytes), box [box_rows, box_inner], with a 0/32/64/128-byte swizzle. dtype is AB_F32 or
// AB_BF16. Throws on failure.
void encode_tmap_2d(CUtensorMap* map, int32_t dtype, const void* base, uint64_t inner,
                    uint64_t rows, uint64_t row_stride_bytes, uint32_t box_inner,
                    uint32_t box_rows, int swizzle_bytes);

// Prologue applied to the activations a GEMV reads.
enum GemvPro : int {
    kProNone = 0,  // x is used as given (f32 or bf16, converted to the weight type)
    kProNorm = 1,  // x (f32) is RMS-normalised with a gain vector first
};

// Epilogue applied to each pair of output rows (2u, 2u + 1).
enum GemvEpi : int {
    kEpiStore = 0,     // out[b, r] = y
    kEpiQkv = 1,       // rows of [wq; wk; wv]: RoPE on q and k, K/V appended to the cache
    kEpiSwiglu = 2,    // rows (w1[u], w3[u]): out[b, u] = silu(y1) * y3
    kEpiResidual = 3,  // out[b, r] += y (f32 residual stream)
};

// Where a tensor-parallel projection leaves its partial for the row all-reduce of one
// site: this rank's send slot (f32, read by the peers over NVLink) (comm.cu).
constexpr uint32_t kTpMaxWorld = 8;
struct TpPush {
    float* out;
    uint32_t site;
};

// Value a rank's flag holds once site `site` of step `epoch` was pushed.
__host__ __device__ inline uint64_t tp_signal_value(uint64_t epoch, uint32_t site) {
    return epoch * 1024 + site + 1;
}

// Parameters of one fused GEMV launch (plain old data; passed by value to the kernel).
struct GemvParams {
    // Virtual weight matrix: up to three row-major [rows, K] segments stacked, or two
    // segments interleaved row by row (kEpiSwiglu).
    const void* seg[3];
    uint32_t seg_rows[3];
    uint32_t n_rows;  // total virtual rows
    uint32_t units;   // output pairs = ceil(n_rows / 2) (or rows of w1 for SwiGLU)
    uint32_t K;
    uint32_t nchunks;  // ceil(K / (32 * elements per 16 bytes))
    uint32_t prefetch_chunks;  // 512-byte chunks of each first weight row prefetched into L2
    uint32_t nb;       // live batch rows in this launch
    // activations [nb, K]
    const void* x;
    int32_t x_dtype;
    uint32_t x_stride;
    const void* norm_w;
    int32_t norm_dtype;
    float eps;
    // outputs
    void* out;
    int32_t out_dtype;
    uint32_t out_stride;
    const float* addend;  // kEpiStore: out = addend + y (f32, laid out like out); may be null
    // kEpiQkv
    float* q;
    uint32_t qd, kvd, head, seq;
    float theta;
    void* kcache;
    void* vcache;
    int32_t kv_dtype;
    uint64_t cache_stride;  // elements between consecutive batch rows of the cache
    const Step* step;
    uint32_t* flags;
    // scratch for the tensor-core path at batch > 4; null = GEMV only
    void* xn;        // the GEMM's activation operand: bf16 [batch, K] (normalised for
                     // kProNorm), or for fp32 weights the tf32 hi and lo halves [2][batch, K]
    uint64_t xn_bytes;
    float* ws;       // split-K partials
    uint64_t ws_floats;
    uint32_t* tickets;  // one per row tile, zero between launches
    uint32_t tickets_n;
};

// Largest batch the GEMV serves in one launch; above it the weights go to the tensor-core
// GEMM (gemm_tc.cu): bf16 on the f16 pipe, fp32 as 3xTF32 on the tf32 pipe.
constexpr uint32_t kGemvMaxBatch = 4;
// Rows (batch rows or prefill-pass rows) up to which a tensor-parallel block sums the ranks'
// partial projections with the NVLink peer all-reduce (tp_reduce); wider steps use NCCL.
constexpr uint32_t kTpPeerMaxRows = 64;

// Parameters of one tensor-core GEMM launch (gemm_tc.cu).
struct GemmTcParams {
    uint32_t K, nb, bn, tiles, kblocks, ksplit, stages, tmem_cols;
    uint32_t krot;  // tile t starts at k-block (t * krot) mod its k-blocks
    uint32_t seg_tiles[3];
    int32_t interleave;  // tile t = rows [64t, 64t + 64) of segment 0, then of segment 1
    float* ws;
    uint64_t ws_floats;
    uint32_t* tickets;
    uint32_t tickets_n;
    // epilogue (as GemvParams)
    void* out;
    int32_t out_dtype;
    uint32_t out_stride;
    const float* addend;
    uint32_t n_rows;
    float* q;
    uint32_t qd, kvd, head, seq;
    float theta;
    void* kcache;
    void* vcache;
    int32_t kv_dtype;
    uint64_t cache_stride;
    const Step* step;
    uint32_t* flags;
};

struct GemmTcPlan {
    uint32_t bn, tiles, kblocks, ksplit, stages, tmem_cols, krot;
    size_t smem;
    uint64_t ws_floats;
};

GemmTcPlan gemm_tc_plan(uint32_t rows, uint32_t K, uint32_t batch, int sms, bool interleave,
                        bool f32);
bool gemm_tc_fits(uint32_t rows, uint32_t K, uint32_t batch, bool interleave, bool f32);
// x: bf16 activation rows (wdtype bf16), or the tf32 hi rows with x_lo the lo rows (fp32).
void record_gemm_tc(ab_scheme* s, const char* label, GemmTcParams p, int32_t wdtype,
                    const void* const* segs, const uint32_t* seg_rows, int nseg, const void* x,
                    const void* x_lo, uint32_t x_stride, int epi);
// hi/lo [rows, dim] = exact tf32 split of x (RMS-normalised with norm_w when non-null).
void record_split_rows_tf32(ab_scheme* s, const char* label, const float* x, uint32_t x_stride,
                            const void* norm_w, int32_t w_dtype, float* hi, float* lo,
                            uint32_t rows, uint32_t dim, float eps);
void record_rmsnorm_rows_bf16(ab_scheme* s, const char* label, const float* x, const void* w,
                              int32_t w_dtype, void* out, uint32_t rows, uint32_t dim, float eps);
// Workspace floats and tickets that cover every tensor-core GEMM with up to `max_tiles`
// row tiles at batches up to `max_batch`.
void gemm_tc_scratch(uint32_t max_tiles, uint32_t max_batch, int sms, uint64_t* ws_floats,
                     uint32_t* tickets);

// Scratch of the tensor-core GEMM path owned by a module: the activation operand
// (8 bytes per element of [max_batch, max_k]: bf16 rows or fp32 hi/lo halves), the
// split-K partials and one ticket per row tile. Nothing is allocated when max_batch is
// within the GEMV's range.
struct GemmScratch {
    void* xn = nullptr;
    uint64_t xn_bytes = 0;
    float* ws = nullptr;
    uint64_t ws_floats = 0;
    uint32_t* tickets = nullptr;
    uint32_t tickets_n = 0;
};
void alloc_tc_scratch(Runtime* rt, GemmScratch* g, uint32_t max_batch, uint32_t max_k,
                      uint32_t max_tiles);
void free_tc_scratch(GemmScratch* g);
void attach_tc_scratch(GemvParams* p, const GemmScratch& g);

// Module constructors with an explicit head size and an optional tensor-parallel
// communicator (blocks.cu); the C entry points call them with tp = null.
ab_attention_block* attention_block_new(ab_runtime* rt, uint32_t hidden, uint32_t heads,
                                        uint32_t head, uint32_t seq_len, uint32_t max_batch,
                                        float rope_theta, ab_comm* tp);
ab_swiglu_block* swiglu_block_new(ab_runtime* rt, uint32_t hidden, uint32_t intermediate,
                                  uint32_t max_batch, ab_comm* tp);

// ---- tensor parallelism (comm.cu) ----
int comm_rank(const ab_comm* c);
int comm_world(const ab_comm* c);
// NVLink peer exchange for the row all-reduce of the decode projections: every rank's
// projection stores its partial in its own send slot; the reduce kernel that follows it
// raises this rank's flag in each peer's flag block (peer pointers opened through CUDA
// IPC), waits until every peer's flag for the site is up and sums the ranks' slots in rank
// order, reading the peers' over NVLink. Slots alternate by site parity, so a rank running
// ahead never overwrites a slot a peer has not read yet. comm_peers_setup is collective; it returns false (on
// every rank) when any peer cannot be opened, and the NCCL all-reduce stays in use.
bool comm_peers_setup(ab_comm* c, size_t max_elems);
void comm_peers_release(ab_comm* c);
bool comm_has_peers(const ab_comm* c);
// The persistent decode step's exchange block of `bytes` on every rank (collective): this
// rank's (zeroed) and every rank's as this rank addresses it through CUDA IPC. Kept until
// the communicator is destroyed (after a barrier of all ranks). False on every rank when a
// peer cannot be opened.
bool comm_fused_block(ab_comm* c, size_t bytes, unsigned char** local,
                      unsigned char* peers[kTpMaxWorld]);
void comm_begin_recording(ab_comm* c);
void record_tp_epoch(ab_scheme* s, ab_comm* c);
TpPush comm_push_target(ab_comm* c);
void record_tp_reduce(ab_scheme* s, const char* label, ab_comm* c, const TpPush& push,
                      float* x, uint32_t n);
void record_allreduce_f32(ab_scheme* s, const char* label, ab_comm* c, const float* send,
                          float* recv, size_t count);
void record_allgather_bytes(ab_scheme* s, const char* label, ab_comm* c, const void* send,
                            void* recv, size_t bytes);

// Seeded synthetic values of a [rows, cols] region of a larger [*, global_cols] tensor
// whose element (r, c) is element (row0 + r, col0 + c) of the global one (runtime.cu).
void fill_normal_region(Runtime* rt, ab_tensor t, uint64_t seed, uint64_t stream, float mean,
                        float std, uint64_t global_cols, uint64_t row0, uint64_t col0);

// Records one fused GEMV (weights of dtype wdtype) over batch rows [0, batch).
void record_gemv(ab_scheme* s, const char* label, GemvParams p, int32_t wdtype, uint32_t batch,
                 int pro, int epi);

// Whether the fused GEMV can run on these shapes (K vector-aligned, rows 16-byte aligned).
bool gemv_fusable(int32_t wdtype, uint32_t K, const void* const* segs, int nseg);

// Parameters of the fused flash-decoding attention launch.
struct AttnParams {
    const float* q;      // [B, H, hd] (rotated)
    const void* kcache;  // [B, S, KV, hd]
    const void* vcache;
    int32_t kv_dtype;
    uint64_t cache_stride;  // elements between batch rows of the cache (0: rows share one)
    uint32_t cache_rows;    // the same in positions (set by record_attention)
    void* out;              // [B, H * hd]
    int32_t out_dtype;
    uint32_t heads, kv_heads, head, seq, batch;
    uint32_t nsplit;
    uint32_t min_chunk;  // fewest positions per split (a multiple of 64; 0 = 64)
    float* part_o;   // [B, KV, nsplit, g, hd]
    float* part_ml;  // [B, KV, nsplit, g, 2]
    uint64_t part_cap;  // floats available from part_o on (0: unknown, no other layout used)
    uint32_t* counters;  // [B, KV], zero between launches
    const Step* step;
    uint32_t* flags;
};

// Scratch (floats for part_o + part_ml, counters) the fused attention needs.
void attention_scratch_size(uint32_t batch, uint32_t heads, uint32_t head, uint32_t nsplit,
                            uint64_t* floats, uint64_t* counters);
uint32_t attention_choose_splits(uint32_t batch, uint32_t kv_heads, uint32_t seq, int sm_count,
                                 uint32_t max_splits);
uint32_t attention_min_chunk();
uint32_t attention_max_splits(uint32_t max_groups, uint32_t seq, int sm_count,
                              uint32_t max_splits);
bool attention_fusable(uint32_t heads, uint32_t kv_heads, uint32_t head, int32_t kv_dtype);
void record_attention(ab_scheme* s, const char* label, AttnParams p);
// Prompt attention of a pass whose rows share one bf16 cache (cache_rows == 0), head 64 or
// 128, on the tcgen05 tensor cores (attention_prompt_tc.cu); false when it does not apply.
bool record_prompt_attention_tc(ab_scheme* s, const char* label, const AttnParams& p);

// ---- persistent decode step (step_fused.cu) ----------------------------------------------
// What the single-launch batch-1 decode step reads and writes (device pointers; per-layer
// K/V caches are [seq, kv_heads, head] views).
struct FusedStepModel {
    // tensor parallelism: this rank's shard sizes below (heads, kv_heads, hidden, vocab),
    // and every rank's exchange block (comm_fused_block); world 1 without
    uint32_t world = 1, rank = 0;
    unsigned char* xblock[kTpMaxWorld] = {};
    uint32_t batch, layers, dim, heads, kv_heads, head_dim, hidden, vocab, seq;
    int32_t dtype;
    float rope_theta, norm_eps;
    const void* embed;
    const void* wcls;
    const void* rms_final;
    std::vector<const void*> rms_att, wq, wk, wv, wo, rms_ffn, w1, w2, w3;
    std::vector<void*> kcache, vcache;
    float* x;
    float* logits;
    int32_t* argmax;
    void* step;
    int32_t* history;
};
struct FusedStep;
// AMMON_B200_FUSED_STEP=0 turns the persistent step off (the per-kernel step graph runs).
bool fused_step_enabled();
// "" when the persistent step can run the model, else the reason it cannot.
std::string fused_step_unsupported(const FusedStepModel& m, int sms);
FusedStep* fused_step_create(Runtime* rt, const FusedStepModel& m);
void fused_step_destroy(FusedStep* f);
// One node "decode_step" (a cooperative launch); with feedback the argmax becomes the next
// DecodeStep and the token history entry, as feedback_kernel does for the step graph.
void record_fused_step(ab_scheme* s, FusedStep* f, bool feedback);
bool fused_step_trace(FusedStep* f, std::vector<uint64_t>* out, uint32_t* barriers,
                      uint32_t* grid);
// Bytes of the exchange block a tensor-parallel persistent step over `world` ranks needs.
size_t fused_step_xblock_bytes(uint32_t world, uint32_t dim);

// Rejects batched shapes the single-row reference kernels cannot take.
void record_embed(ab_scheme* s, ab_tensor table, ab_tensor step, ab_tensor x);
void record_rmsnorm_ref(ab_scheme* s, ab_tensor x, ab_tensor weight, ab_tensor o, float eps);
void record_linear(ab_scheme* s, const char* label, ab_tensor weight, ab_tensor x, ab_tensor out);

}  // namespace ab
