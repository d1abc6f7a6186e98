// Host decode loop (src/generate.rs, src/tokenizer.rs:179-189) and the Llama-shaped
// model the harness decodes with. The reference leaves model assembly to architecture
// crates (README.md:5,21); this one composes the modules in the llama2.c order:
// Embedding, layers x [CausalAttentionBlock, SwiGluBlock], final RmsNorm, classifier.
//
// One decode step is one CUDA graph recorded once: the DecodeStep parcel is refreshed
// by a deposit before each replay, so nothing is re-recorded per token.
//
// Under tensor parallelism (ab_llama_create_tp) every rank holds a shard: its query and kv
// heads, its SwiGLU columns and its slice of the vocabulary; the residual stream and the
// embedding table are replicated. The greedy pick merges every rank's best (value, id).
#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "ops.h"

using namespace ab;

namespace ab {

// Candidate of a greedy pick: best logit and its vocabulary id.
struct ArgPair {
    float v;
    uint32_t i;
};

// (value, id) of the first maximum of a row of logits, ids offset by `offset`; NaNs never
// win. The reduction keeps the lowest id among equal values: the rule of sample_argmax
// (src/tokenizer.rs:179-189).
__device__ __forceinline__ ArgPair row_argmax(const float* __restrict__ row, uint32_t n,
                                              uint32_t offset) {
    __shared__ float bv[32];
    __shared__ uint32_t bi[32];
    float best = -INFINITY;
    uint32_t idx = 0xffffffffu;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = row[i];
        if (v > best || (idx == 0xffffffffu && v == best)) {
            best = v;
            idx = i;
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ov > best || (ov == best && oi < idx)) {
            best = ov;
            idx = oi;
        }
    }
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    if (lane == 0) {
        bv[warp] = best;
        bi[warp] = idx;
    }
    __syncthreads();
    ArgPair r = {-INFINITY, 0xffffffffu};
    if (warp == 0) {
        const uint32_t nw = blockDim.x / 32;
        best = lane < nw ? bv[lane] : -INFINITY;
        idx = lane < nw ? bi[lane] : 0xffffffffu;
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, idx, o);
            if (ov > best || (ov == best && oi < idx)) {
                best = ov;
                idx = oi;
            }
        }
        r.v = best;
        r.i = idx == 0xffffffffu ? 0xffffffffu : idx + offset;
    }
    return r;
}

// Device argmax with the row split over kArgmaxSplit CTAs: CTA (s, b) takes the first maximum
// of its slice of row b, and the last CTA of the row to finish (atomic ticket, reset for the
// next replay) keeps the first maximum of the slices' candidates (greater value, or the lower
// id among equal values: the sample_argmax rule). One 1024-thread CTA per row read a 128k-entry
// row at ~20 GB/s; the split takes the row in a few microseconds.
constexpr uint32_t kArgmaxSplit = 64;

__device__ __forceinline__ ArgPair first_max(ArgPair a, ArgPair b) {
    if (b.i == 0xffffffffu) return a;
    if (a.i == 0xffffffffu || b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
    return a;
}

__global__ void __launch_bounds__(256)
    argmax_split_kernel(const float* __restrict__ logits, uint32_t vocab, ArgPair* part,
                        uint32_t* tickets, int32_t* __restrict__ out) {
    pdl_wait();
    const uint32_t sl = blockIdx.x, b = blockIdx.y, ns = gridDim.x;
    const uint32_t chunk = (vocab + ns - 1) / ns;
    const uint32_t lo = min(vocab, sl * chunk), hi = min(vocab, lo + chunk);
    const ArgPair r = row_argmax(logits + (uint64_t)b * vocab + lo, hi - lo, lo);
    __shared__ int last;
    if (threadIdx.x == 0) {
        part[(uint64_t)b * ns + sl] = r;
        __threadfence();
        last = atomicAdd(&tickets[b], 1u) == ns - 1;
    }
    __syncthreads();
    if (last && threadIdx.x < 32) {
        __threadfence();
        ArgPair best = {-INFINITY, 0xffffffffu};
        for (uint32_t k = threadIdx.x; k < ns; k += 32) {
            const ArgPair* src = part + (uint64_t)b * ns + k;
            ArgPair c;
            c.v = __ldcg(&src->v);
            c.i = __ldcg(&src->i);
            best = first_max(best, c);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            ArgPair c;
            c.v = __shfl_xor_sync(0xffffffffu, best.v, o);
            c.i = __shfl_xor_sync(0xffffffffu, best.i, o);
            best = first_max(best, c);
        }
        if (threadIdx.x == 0) {
            out[b] = best.i == 0xffffffffu ? 0 : (int32_t)best.i;
            tickets[b] = 0;
        }
    }
    pdl_trigger();
}

// Best (value, global id) of this rank's vocabulary slice, per row.
__global__ void __launch_bounds__(1024)
    argmax_pair_kernel(const float* __restrict__ logits, uint32_t vocab_l, uint32_t offset,
                       ArgPair* __restrict__ out) {
    pdl_wait();
    const ArgPair r = row_argmax(logits + (uint64_t)blockIdx.x * vocab_l, vocab_l, offset);
    if (threadIdx.x == 0) out[blockIdx.x] = r;
    pdl_trigger();
}

// Merge the ranks' candidates [world, batch] into the first maximum per row.
__global__ void argmax_merge_kernel(const ArgPair* __restrict__ all, uint32_t world,
                                    uint32_t batch, int32_t* __restrict__ out) {
    pdl_wait();
    const uint32_t b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < batch) {
        ArgPair best = {-INFINITY, 0xffffffffu};
        for (uint32_t r = 0; r < world; r++) {
            const ArgPair c = all[(uint64_t)r * batch + b];
            if (c.i == 0xffffffffu) continue;
            if (c.v > best.v || (c.v == best.v && c.i < best.i) || best.i == 0xffffffffu) best = c;
        }
        out[b] = best.i == 0xffffffffu ? 0 : (int32_t)best.i;
    }
    pdl_trigger();
}

// Device-side sample feedback: the next DecodeStep of row b is {argmax[b], position + 1};
// the id is also kept in history[position + 1, b].
__global__ void feedback_kernel(const int32_t* __restrict__ argmax, Step* step,
                                int32_t* __restrict__ history, uint32_t batch, uint32_t seq,
                                uint32_t* flags) {
    pdl_wait();
    const uint32_t b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < batch) {
        const uint32_t next = step[b].position + 1;
        if (next >= seq) {
            atomicOr(flags, kFlagPositionRange);
        } else {
            const int32_t tok = argmax[b];
            history[(uint64_t)next * batch + b] = tok;
            step[b].token = (uint32_t)tok;
            step[b].position = next;
        }
    }
    pdl_trigger();
}

}  // namespace ab

struct ab_llama {
    Runtime* rt = nullptr;
    ab_llama_config c = {};
    ab_comm* comm = nullptr;  // tensor parallelism (null: one GPU)
    int32_t rank = 0, world = 1;
    uint32_t heads_l = 0, kv_l = 0, hidden_l = 0, vocab_l = 0;  // this rank's shard
    ab_tensor embed = {}, wcls = {}, rms_final = {};
    std::vector<ab_tensor> rms_att, wq, wk, wv, wo, rms_ffn, w1, w2, w3;
    ab_kvcache* cache = nullptr;
    ab_attention_block* attn = nullptr;
    ab_swiglu_block* ffn = nullptr;
    ab_tensor x = {}, logits = {}, step = {}, argmax = {}, history = {};
    ab_tensor logits_all = {}, pairs = {}, pairs_all = {};  // tensor parallelism
    ab_tensor amx_part = {}, amx_tickets = {};  // split argmax: [batch, split] pairs, [batch]
    ab_scheme* scheme = nullptr;       // one decode step (gathers the logits under TP)
    ab_scheme* loop_scheme = nullptr;  // one decode step + device sample feedback
    GemmScratch cls_tc;                // classifier's tensor-core GEMM scratch
    FusedStep* fused = nullptr;        // persistent single-launch step (batch 1, bf16)
    float* h_logits = nullptr;         // pinned [batch, vocab]
    int32_t* h_argmax = nullptr;
    uint32_t* h_flags = nullptr;       // pinned copy of the runtime's device flag word
    ab_decode_step* h_steps = nullptr;
    std::vector<float> vt_logits;  // host logits handed out through the vtable
    // Batched prefill: up to pf_rows prompt positions of one cache stream run as the rows
    // of one pass (set up on the first prefill). Passes are recorded per (stream, rows,
    // whether the classifier runs) and the most recently used few are kept.
    struct PrefillScheme {
        uint32_t stream, rows;
        bool head;
        ab_scheme* s;
        uint64_t used;
    };
    uint32_t pf_rows = 0;
    uint32_t pf_rows_wanted = 0;  // 0: the default
    ab_attention_block* pf_attn = nullptr;
    ab_swiglu_block* pf_ffn = nullptr;
    ab_tensor pf_x = {}, pf_step = {}, pf_logits = {}, pf_argmax = {};
    ab_tensor pf_logits_all = {}, pf_pairs = {}, pf_pairs_all = {};
    std::vector<PrefillScheme> pf_schemes;
    uint64_t pf_clock = 0;
    uint32_t pf_launches = 0;              // kernels and collectives of the last prefill
    ab_decode_step* h_pf_steps = nullptr;  // pinned [seq]
    float* h_pf_logits = nullptr;          // pinned [vocab]
};

namespace {

void free_t(ab_tensor& t) {
    if (t.data) cudaFree(t.data);
    t.data = nullptr;
}

ab_tensor alloc_t(ab_runtime* rt, int32_t dt, std::initializer_list<uint32_t> dims) {
    ab_tensor t = {};
    std::vector<uint32_t> d(dims);
    if (ab_tensor_zeros(rt, dt, (int32_t)d.size(), d.data(), &t) != AB_OK)
        fail(AB_ERR_CUDA, std::string("model allocation: ") + ab_last_error());
    return t;
}

void check(int status) {
    if (status != AB_OK) fail(status, ab_last_error());
}

void free_prefill(ab_llama* m) {
    for (auto& e : m->pf_schemes) ab_scheme_destroy(e.s);
    m->pf_schemes.clear();
    if (m->pf_attn) ab_attention_block_destroy(m->pf_attn);
    if (m->pf_ffn) ab_swiglu_block_destroy(m->pf_ffn);
    m->pf_attn = nullptr;
    m->pf_ffn = nullptr;
    for (ab_tensor* t : {&m->pf_x, &m->pf_step, &m->pf_logits, &m->pf_argmax, &m->pf_logits_all,
                         &m->pf_pairs, &m->pf_pairs_all})
        free_t(*t);
    if (m->h_pf_steps) cudaFreeHost(m->h_pf_steps);
    if (m->h_pf_logits) cudaFreeHost(m->h_pf_logits);
    m->h_pf_steps = nullptr;
    m->h_pf_logits = nullptr;
    m->pf_rows = 0;
}

void destroy_model(ab_llama* m) {
    if (!m) return;
    Runtime* rt = m->rt;
    if (rt) {
        rt->activate();
        cudaStreamSynchronize(rt->stream);
    }
    free_prefill(m);
    if (m->scheme) ab_scheme_destroy(m->scheme);
    if (m->loop_scheme) ab_scheme_destroy(m->loop_scheme);
    fused_step_destroy(m->fused);
    free_tc_scratch(&m->cls_tc);
    if (m->attn) ab_attention_block_destroy(m->attn);
    if (m->ffn) ab_swiglu_block_destroy(m->ffn);
    if (m->cache) ab_kvcache_destroy(m->cache);
    for (auto* v : {&m->rms_att, &m->wq, &m->wk, &m->wv, &m->wo, &m->rms_ffn, &m->w1, &m->w2,
                    &m->w3})
        for (auto& t : *v) free_t(t);
    for (ab_tensor* t : {&m->embed, &m->wcls, &m->rms_final, &m->x, &m->logits, &m->step,
                         &m->argmax, &m->history, &m->logits_all, &m->pairs, &m->pairs_all,
                         &m->amx_part, &m->amx_tickets})
        free_t(*t);
    if (m->h_logits) cudaFreeHost(m->h_logits);
    if (m->h_argmax) cudaFreeHost(m->h_argmax);
    if (m->h_flags) cudaFreeHost(m->h_flags);
    if (m->h_steps) cudaFreeHost(m->h_steps);
    delete m;
}

// One cache stream's view [seq, kv_heads, head] of a layer's cache.
ab_tensor stream_view(ab_tensor t, uint32_t stream) {
    if (t.rank == 4) {
        const uint64_t per = (uint64_t)t.dims[1] * t.dims[2] * t.dims[3];
        t.data = (char*)t.data + stream * per * dtype_size(t.dtype);
        t.rank = 3;
        t.dims[0] = t.dims[1];
        t.dims[1] = t.dims[2];
        t.dims[2] = t.dims[3];
        t.dims[3] = 0;
    }
    return t;
}

// The embedding and every layer over the rows of x with the DecodeSteps of `step`. Each row
// appends to and attends over its own cache stream, or, with stream >= 0, every row is a
// position of that one stream (a prompt's consecutive positions).
void record_layers(ab_llama* m, ab_scheme* s, ab_tensor x, ab_tensor step,
                   ab_attention_block* attn, ab_swiglu_block* ffn, int64_t stream) {
    const auto& c = m->c;
    if (m->comm && comm_has_peers(m->comm)) {
        // a new epoch per replay names this step's peer flags; sites count from zero
        comm_begin_recording(m->comm);
        record_tp_epoch(s, m->comm);
    }
    check(ab_embedding_record(s, m->embed, step, x));
    for (uint32_t l = 0; l < c.layers; l++) {
        ab_tensor key, value;
        check(ab_kvcache_layer(m->cache, l, &key, &value));
        if (stream >= 0) {
            key = stream_view(key, (uint32_t)stream);
            value = stream_view(value, (uint32_t)stream);
        }
        ab_attention_weights aw = {m->rms_att[l], m->wq[l], m->wk[l], m->wv[l], m->wo[l]};
        check(ab_attention_block_record(attn, s, x, &aw, key, value, step));
        ab_swiglu_weights fw = {m->rms_ffn[l], m->w1[l], m->w3[l], m->w2[l]};
        check(ab_swiglu_block_record(ffn, s, x, &fw));
    }
}

// Where the classifier and the greedy pick of `rows` residual rows leave their results:
// logits [rows, vocab_l] and argmax [rows]; under tensor parallelism the ranks' (value, id)
// candidates go through pairs / pairs_all and, when gathered, the logits into logits_all
// [world, rows, vocab_l].
struct HeadOut {
    const float* x;
    uint32_t rows;
    float* logits;
    int32_t* argmax;
    ArgPair* pairs;
    ArgPair* pairs_all;
    void* logits_all;
    const GemmScratch* tc;
    ArgPair* split_part;      // [rows, kArgmaxSplit] slice candidates (one GPU)
    uint32_t* split_tickets;  // [rows], zero between launches
};

// Final RmsNorm fused into the classifier's prologue (this rank's vocabulary rows), then the
// device argmax (merged over the ranks under tensor parallelism).
void record_head(ab_llama* m, ab_scheme* s, const HeadOut& h, bool gather_logits) {
    const auto& c = m->c;
    GemvParams g = {};
    g.seg[0] = m->wcls.data;
    g.seg_rows[0] = m->vocab_l;
    g.n_rows = m->vocab_l;
    g.units = (m->vocab_l + 1) / 2;
    g.K = c.dim;
    g.x = h.x;
    g.x_dtype = AB_F32;
    g.x_stride = c.dim;
    g.norm_w = m->rms_final.data;
    g.norm_dtype = m->rms_final.dtype;
    g.eps = c.norm_eps;
    g.out = h.logits;
    g.out_dtype = AB_F32;
    g.out_stride = m->vocab_l;
    if (h.tc) attach_tc_scratch(&g, *h.tc);
    record_gemv(s, "final_norm_classifier", g, c.dtype, h.rows, kProNorm, kEpiStore);
    const float* lg = h.logits;
    int32_t* am = h.argmax;
    const uint32_t batch = h.rows;
    if (m->world == 1) {
        const uint32_t vocab = c.vocab;
        ArgPair* part = h.split_part;
        uint32_t* tk = h.split_tickets;
        s->add("argmax", [=](cudaStream_t st) {
            return launch(st, dim3(kArgmaxSplit, batch), dim3(256), 0, true, argmax_split_kernel,
                          lg, vocab, part, tk, am);
        });
    } else {
        ArgPair* pr = h.pairs;
        ArgPair* pa = h.pairs_all;
        const uint32_t vl = m->vocab_l, off = (uint32_t)m->rank * m->vocab_l;
        const uint32_t world = (uint32_t)m->world;
        s->add("argmax", [=](cudaStream_t st) {
            return launch(st, dim3(batch), dim3(1024), 0, true, argmax_pair_kernel, lg, vl, off, pr);
        });
        record_allgather_bytes(s, "argmax_allgather", m->comm, pr, pa, (size_t)batch * 8);
        s->add("argmax_merge", [=](cudaStream_t st) {
            return launch(st, dim3((batch + 127) / 128), dim3(128), 0, true, argmax_merge_kernel,
                          (const ArgPair*)pa, world, batch, am);
        });
        if (gather_logits)
            record_allgather_bytes(s, "logits_allgather", m->comm, lg, h.logits_all,
                                   (size_t)batch * m->vocab_l * 4);
    }
}

// Records the full decode step into `s`: with the device sample feedback (the device
// loop) or, under tensor parallelism, with the logits gathered from every rank.
void record_step(ab_llama* m, ab_scheme* s, bool feedback, bool gather_logits) {
    s->nodes.clear();
    s->dirty = true;
    if (m->fused) {
        record_fused_step(s, m->fused, feedback);
        if (m->world > 1 && gather_logits)
            record_allgather_bytes(s, "logits_allgather", m->comm, m->logits.data,
                                   m->logits_all.data, (size_t)m->c.batch * m->vocab_l * 4);
        return;
    }
    const auto& c = m->c;
    ab_tensor x = m->x;
    if (c.batch == 1) {
        x.rank = 1;
        x.dims[0] = c.dim;
    }
    record_layers(m, s, x, m->step, m->attn, m->ffn, -1);
    const uint32_t batch = c.batch;
    int32_t* am = (int32_t*)m->argmax.data;
    record_head(m, s,
                {(const float*)m->x.data, batch, (float*)m->logits.data, am,
                 (ArgPair*)m->pairs.data, (ArgPair*)m->pairs_all.data, m->logits_all.data,
                 &m->cls_tc, (ArgPair*)m->amx_part.data, (uint32_t*)m->amx_tickets.data},
                gather_logits);
    if (feedback) {
        Step* stp = (Step*)m->step.data;
        int32_t* hist = (int32_t*)m->history.data;
        const uint32_t seq = c.seq;
        uint32_t* flags = m->rt->flags;
        s->add("sample_feedback", [=](cudaStream_t st) {
            return launch(st, dim3((batch + 127) / 128), dim3(128), 0, true, feedback_kernel, am,
                          stp, hist, batch, seq, flags);
        });
    }
}

// Records one prefill pass of `rows` positions of cache stream `stream`; with `head` the
// last row's logits and greedy id follow (the logits gathered over the ranks).
void record_prefill(ab_llama* m, ab_scheme* s, uint32_t stream, uint32_t rows, bool head) {
    s->nodes.clear();
    s->dirty = true;
    const auto& c = m->c;
    ab_tensor x = m->pf_x;
    if (rows == 1) {
        x.rank = 1;
        x.dims[0] = c.dim;
    } else {
        x.dims[0] = rows;
    }
    record_layers(m, s, x, m->pf_step, m->pf_attn, m->pf_ffn, stream);
    if (head)
        record_head(m, s,
                    {(const float*)m->pf_x.data + (uint64_t)(rows - 1) * c.dim, 1,
                     (float*)m->pf_logits.data, (int32_t*)m->pf_argmax.data,
                     (ArgPair*)m->pf_pairs.data, (ArgPair*)m->pf_pairs_all.data,
                     m->pf_logits_all.data, nullptr, (ArgPair*)m->amx_part.data,
                     (uint32_t*)m->amx_tickets.data},
                    true);
}

// Rows per prefill pass: 256 (the tensor-core GEMM's widest batch) unless the model or
// AMMON_B200_PREFILL_ROWS asks for fewer; never more than seq_len.
uint32_t prefill_rows(const ab_llama* m) {
    long r = 256;
    if (m->pf_rows_wanted) {
        r = m->pf_rows_wanted;
    } else if (const char* e = std::getenv("AMMON_B200_PREFILL_ROWS")) {
        r = std::atol(e);
    }
    r = std::max(1L, std::min(r, 256L));
    return (uint32_t)std::min<long>(r, m->c.seq);
}

void setup_prefill(ab_llama* m) {
    const uint32_t rows = prefill_rows(m);
    if (m->pf_rows == rows) return;
    free_prefill(m);
    const auto& c = m->c;
    ab_runtime* rt = static_cast<ab_runtime*>(m->rt);
    try {
        m->pf_attn = attention_block_new(rt, c.dim, m->heads_l, c.head_dim, c.seq, rows,
                                         c.rope_theta, m->comm);
        m->pf_ffn = swiglu_block_new(rt, c.dim, m->hidden_l, rows, m->comm);
        m->pf_x = alloc_t(rt, AB_F32, {rows, c.dim});
        m->pf_logits = alloc_t(rt, AB_F32, {1, m->vocab_l});
        m->pf_argmax = alloc_t(rt, AB_U32, {1});
        if (m->world > 1) {
            m->pf_logits_all = alloc_t(rt, AB_F32, {(uint32_t)m->world, 1, m->vocab_l});
            m->pf_pairs = alloc_t(rt, AB_U32, {1, 2});
            m->pf_pairs_all = alloc_t(rt, AB_U32, {(uint32_t)m->world, 1, 2});
        }
        check(ab_step_parcel(rt, rows, &m->pf_step));
        cuda_check(cudaMallocHost(&m->h_pf_steps, (size_t)c.seq * sizeof(ab_decode_step)),
                   "pinned prefill steps");
        cuda_check(cudaMallocHost(&m->h_pf_logits, (size_t)c.vocab * 4), "pinned logits");
    } catch (...) {
        free_prefill(m);
        throw;
    }
    m->pf_rows = rows;
}

// The recorded pass for (stream, rows, head), recording it on first use; the least
// recently used pass is dropped beyond kPrefillSchemes.
constexpr size_t kPrefillSchemes = 8;
ab_scheme* prefill_scheme(ab_llama* m, uint32_t stream, uint32_t rows, bool head) {
    m->pf_clock++;
    for (auto& e : m->pf_schemes)
        if (e.stream == stream && e.rows == rows && e.head == head) {
            e.used = m->pf_clock;
            return e.s;
        }
    if (m->pf_schemes.size() >= kPrefillSchemes) {
        auto lru = std::min_element(
            m->pf_schemes.begin(), m->pf_schemes.end(),
            [](const ab_llama::PrefillScheme& a, const ab_llama::PrefillScheme& b) {
                return a.used < b.used;
            });
        ab_scheme_destroy(lru->s);
        m->pf_schemes.erase(lru);
    }
    ab_scheme* s = nullptr;
    check(ab_scheme_create(static_cast<ab_runtime*>(m->rt), &s));
    try {
        record_prefill(m, s, stream, rows, head);
    } catch (...) {
        ab_scheme_destroy(s);
        throw;
    }
    m->pf_schemes.push_back({stream, rows, head, s, m->pf_clock});
    return s;
}

int vt_step(void* self, uint32_t token, uint32_t pos, const float** logits) {
    auto* m = (ab_llama*)self;
    ab_decode_step s = {token, pos};
    m->vt_logits.resize(m->c.vocab);
    int r = ab_llama_step(m, &s, 1, m->vt_logits.data(), nullptr);
    *logits = m->vt_logits.data();
    return r;
}
uint32_t vt_vocab(void* self) { return ((ab_llama*)self)->c.vocab; }
uint32_t vt_seq(void* self) { return ((ab_llama*)self)->c.seq; }

ab_llama* create_model(ab_runtime* rt, const ab_llama_config* cfg, ab_comm* comm) {
    if (!rt || !cfg) fail(AB_ERR_ARGUMENT, "null argument");
    const ab_llama_config c = *cfg;
    if (!c.dim || !c.layers || !c.heads || !c.kv_heads || !c.head_dim || !c.hidden || !c.vocab ||
        !c.seq || !c.batch)
        fail(AB_ERR_ARGUMENT, "model dims must be non-zero");
    if (c.heads * c.head_dim != c.dim) fail(AB_ERR_VALIDATION, "heads * head_dim must equal dim");
    if (c.dtype != AB_F32 && c.dtype != AB_BF16) fail(AB_ERR_ARGUMENT, "dtype f32 or bf16");
    const int32_t world = comm ? comm_world(comm) : 1;
    const int32_t rank = comm ? comm_rank(comm) : 0;
    if (c.heads % world || c.kv_heads % world || c.hidden % world || c.vocab % world)
        fail(AB_ERR_VALIDATION, "tensor parallelism over " + std::to_string(world) +
                                    " ranks needs heads, kv_heads, hidden and vocab divisible by it");
    auto* m = new ab_llama();
    m->rt = rt;
    m->c = c;
    m->comm = comm;
    m->rank = rank;
    m->world = world;
    m->heads_l = c.heads / world;
    m->kv_l = c.kv_heads / world;
    m->hidden_l = c.hidden / world;
    m->vocab_l = c.vocab / world;
    try {
        const int32_t dt = c.dtype;
        const uint32_t qd = m->heads_l * c.head_dim, kvd = m->kv_l * c.head_dim;
        m->embed = alloc_t(rt, dt, {c.vocab, c.dim});
        m->wcls = alloc_t(rt, dt, {m->vocab_l, c.dim});
        m->rms_final = alloc_t(rt, dt, {c.dim});
        for (uint32_t l = 0; l < c.layers; l++) {
            m->rms_att.push_back(alloc_t(rt, dt, {c.dim}));
            m->wq.push_back(alloc_t(rt, dt, {qd, c.dim}));
            m->wk.push_back(alloc_t(rt, dt, {kvd, c.dim}));
            m->wv.push_back(alloc_t(rt, dt, {kvd, c.dim}));
            m->wo.push_back(alloc_t(rt, dt, {c.dim, qd}));
            m->rms_ffn.push_back(alloc_t(rt, dt, {c.dim}));
            m->w1.push_back(alloc_t(rt, dt, {m->hidden_l, c.dim}));
            m->w2.push_back(alloc_t(rt, dt, {c.dim, m->hidden_l}));
            m->w3.push_back(alloc_t(rt, dt, {m->hidden_l, c.dim}));
        }
        check(ab_kvcache_create(rt, c.layers, c.seq, m->kv_l, c.head_dim, dt, c.batch, &m->cache));
        // NVLink peer slots for the per-block row all-reduce. That path carries at most
        // kTpPeerMaxRows rows (wider steps and prefill passes take NCCL), so the slots depend
        // on the width alone and every model of this width on the communicator shares them
        // (collective; falls back to NCCL on every rank when a peer cannot be opened)
        if (comm && world > 1)
            comm_peers_setup(comm, (size_t)kTpPeerMaxRows * c.dim);
        m->attn = attention_block_new(rt, c.dim, m->heads_l, c.head_dim, c.seq, c.batch,
                                      c.rope_theta, comm);
        m->ffn = swiglu_block_new(rt, c.dim, m->hidden_l, c.batch, comm);
        alloc_tc_scratch(rt, &m->cls_tc, c.batch, c.dim, (m->vocab_l + 127) / 128);
        m->x = alloc_t(rt, AB_F32, {c.batch, c.dim});
        m->logits = alloc_t(rt, AB_F32, {c.batch, m->vocab_l});
        m->argmax = alloc_t(rt, AB_U32, {c.batch});
        m->amx_part = alloc_t(rt, AB_U32, {c.batch, kArgmaxSplit, 2});
        m->amx_tickets = alloc_t(rt, AB_U32, {c.batch});
        m->history = alloc_t(rt, AB_U32, {c.seq, c.batch});
        if (world > 1) {
            m->logits_all = alloc_t(rt, AB_F32, {(uint32_t)world, c.batch, m->vocab_l});
            m->pairs = alloc_t(rt, AB_U32, {c.batch, 2});
            m->pairs_all = alloc_t(rt, AB_U32, {(uint32_t)world, c.batch, 2});
        }
        check(ab_step_parcel(rt, c.batch, &m->step));
        cuda_check(cudaMallocHost(&m->h_logits, (size_t)c.batch * c.vocab * 4), "pinned logits");
        cuda_check(cudaMallocHost(&m->h_argmax, (size_t)c.batch * 4), "pinned argmax");
        cuda_check(cudaMallocHost(&m->h_flags, 4), "pinned flag word");
        cuda_check(cudaMallocHost(&m->h_steps, (size_t)c.batch * sizeof(ab_decode_step)),
                   "pinned steps");
        check(ab_scheme_create(rt, &m->scheme));
        check(ab_scheme_create(rt, &m->loop_scheme));
        if (fused_step_enabled()) {
            // this rank's shard; every rank reaches the same decision (same config and
            // environment), so the collective exchange-block set-up is entered by all or none
            FusedStepModel fm;
            fm.world = (uint32_t)world;
            fm.rank = (uint32_t)rank;
            fm.batch = c.batch;
            fm.layers = c.layers;
            fm.dim = c.dim;
            fm.heads = m->heads_l;
            fm.kv_heads = m->kv_l;
            fm.head_dim = c.head_dim;
            fm.hidden = m->hidden_l;
            fm.vocab = m->vocab_l;
            fm.seq = c.seq;
            fm.dtype = c.dtype;
            fm.rope_theta = c.rope_theta;
            fm.norm_eps = c.norm_eps;
            bool go = fused_step_unsupported(fm, rt->sm_count).empty();
            if (go && world > 1) {
                unsigned char* local = nullptr;
                go = comm_fused_block(comm, fused_step_xblock_bytes(world, c.dim), &local,
                                      fm.xblock);
            }
            if (go) {
                fm.embed = m->embed.data;
                fm.wcls = m->wcls.data;
                fm.rms_final = m->rms_final.data;
                for (uint32_t l = 0; l < c.layers; l++) {
                    fm.rms_att.push_back(m->rms_att[l].data);
                    fm.wq.push_back(m->wq[l].data);
                    fm.wk.push_back(m->wk[l].data);
                    fm.wv.push_back(m->wv[l].data);
                    fm.wo.push_back(m->wo[l].data);
                    fm.rms_ffn.push_back(m->rms_ffn[l].data);
                    fm.w1.push_back(m->w1[l].data);
                    fm.w2.push_back(m->w2[l].data);
                    fm.w3.push_back(m->w3[l].data);
                    ab_tensor key, value;
                    check(ab_kvcache_layer(m->cache, l, &key, &value));
                    fm.kcache.push_back(key.data);
                    fm.vcache.push_back(value.data);
                }
                fm.x = (float*)m->x.data;
                fm.logits = (float*)m->logits.data;
                fm.argmax = (int32_t*)m->argmax.data;
                fm.step = m->step.data;
                fm.history = (int32_t*)m->history.data;
                m->fused = fused_step_create(rt, fm);
            }
        }
    } catch (...) {
        destroy_model(m);
        throw;
    }
    return m;
}

}  // namespace

extern "C" {

int32_t ab_sample_argmax(const float* logits, uint32_t n) {
    if (!logits || n == 0) return 0;
    uint32_t max_i = 0;
    float max_p = logits[0];
    for (uint32_t i = 1; i < n; i++)
        if (logits[i] > max_p) {
            max_i = i;
            max_p = logits[i];
        }
    return (int32_t)max_i;
}

int ab_generate_tokens(const ab_autoregressive_model* m, const int32_t* prompt, uint32_t prompt_len,
                       uint32_t max_new_tokens, int32_t has_stop, int32_t stop_on,
                       int32_t* out_tokens, uint32_t cap, uint32_t* out_len,
                       double* tokens_per_second) {
    return guard([&] {
        if (!m || !m->step || !m->vocab_size || !m->max_seq_len)
            fail(AB_ERR_ARGUMENT, "null model");
        if (!prompt || prompt_len == 0) fail(AB_ERR_ARGUMENT, "expected at least one prompt token");
        const uint32_t vocab = m->vocab_size(m->self);
        max_new_tokens = std::min(max_new_tokens, m->max_seq_len(m->self));
        uint32_t token = (uint32_t)prompt[0];
        uint32_t pos = 0, n = 0;
        bool started = false;
        std::chrono::steady_clock::time_point start;
        const uint32_t limit = max_new_tokens > 0 ? max_new_tokens - 1 : 0;
        while (pos < limit) {
            const float* logits = nullptr;
            const int r = m->step(m->self, token, pos, &logits);
            if (r != AB_OK) fail(r, std::string("model step: ") + ab_last_error());
            int32_t next;
            if ((uint64_t)pos < (uint64_t)prompt_len - 1)
                next = prompt[pos + 1];
            else
                next = ab_sample_argmax(logits, vocab);
            pos += 1;
            if (has_stop && stop_on == next) break;
            if (out_tokens && n < cap) out_tokens[n] = next;
            n++;
            token = (uint32_t)next;
            if (!started) {
                started = true;
                start = std::chrono::steady_clock::now();
            }
        }
        double elapsed = 0.0;
        if (started)
            elapsed = std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count();
        const double gen = pos > 0 ? (double)(pos - 1) : 0.0;
        if (out_len) *out_len = n;
        if (tokens_per_second) *tokens_per_second = elapsed > 0.0 ? gen / elapsed : 0.0;
    });
}

int ab_llama_create(ab_runtime* rt, const ab_llama_config* cfg, ab_llama** out) {
    return guard([&] {
        if (!out) fail(AB_ERR_ARGUMENT, "null argument");
        *out = create_model(rt, cfg, nullptr);
    });
}

int ab_llama_create_tp(ab_runtime* rt, const ab_llama_config* cfg, ab_comm* comm,
                       ab_llama** out) {
    return guard([&] {
        if (!out || !comm) fail(AB_ERR_ARGUMENT, "null argument");
        *out = create_model(rt, cfg, comm);
    });
}

int ab_llama_init_synthetic(ab_llama* m, uint64_t seed, float std) {
    return guard([&] {
        if (!m) fail(AB_ERR_ARGUMENT, "null model");
        Runtime* rt = m->rt;
        const auto& c = m->c;
        const uint64_t r = (uint64_t)m->rank;
        const uint64_t qd = (uint64_t)c.heads * c.head_dim, kvd = (uint64_t)c.kv_heads * c.head_dim;
        const uint64_t qd_l = (uint64_t)m->heads_l * c.head_dim;
        const uint64_t kvd_l = (uint64_t)m->kv_l * c.head_dim;
        // Every shard draws the global tensor's values at its own indices, so any rank
        // count decodes the same model. Stream ids are shared with the CPU oracle.
        auto rows = [&](ab_tensor& t, uint64_t stream, uint64_t row0, float mean, float sd) {
            fill_normal_region(rt, t, seed, stream, mean, sd, t.dims[t.rank - 1], row0, 0);
        };
        auto cols = [&](ab_tensor& t, uint64_t stream, uint64_t gcols, uint64_t col0) {
            fill_normal_region(rt, t, seed, stream, 0.0f, std, gcols, 0, col0);
        };
        rows(m->embed, 1, 0, 0.0f, std);
        rows(m->rms_final, 2, 0, 1.0f, 0.01f);
        rows(m->wcls, 3, r * m->vocab_l, 0.0f, std);
        for (uint32_t l = 0; l < c.layers; l++) {
            const uint64_t b = 16 + 16ull * l;
            rows(m->rms_att[l], b + 0, 0, 1.0f, 0.01f);
            rows(m->wq[l], b + 1, r * qd_l, 0.0f, std);
            rows(m->wk[l], b + 2, r * kvd_l, 0.0f, std);
            rows(m->wv[l], b + 3, r * kvd_l, 0.0f, std);
            cols(m->wo[l], b + 4, qd, r * qd_l);
            rows(m->rms_ffn[l], b + 5, 0, 1.0f, 0.01f);
            rows(m->w1[l], b + 6, r * m->hidden_l, 0.0f, std);
            cols(m->w2[l], b + 7, c.hidden, r * m->hidden_l);
            rows(m->w3[l], b + 8, r * m->hidden_l, 0.0f, std);
        }
        (void)kvd;
        rt->activate();
        cuda_check(cudaStreamSynchronize(rt->stream), "init synchronize");
    });
}

int ab_llama_weight(ab_llama* m, int32_t which, uint32_t layer, ab_tensor* out) {
    return guard([&] {
        if (!m || !out) fail(AB_ERR_ARGUMENT, "null argument");
        if (which >= 3 && layer >= m->c.layers) fail(AB_ERR_ARGUMENT, "layer out of range");
        switch (which) {
            case 0: *out = m->embed; break;
            case 1: *out = m->wcls; break;
            case 2: *out = m->rms_final; break;
            case 3: *out = m->rms_att[layer]; break;
            case 4: *out = m->wq[layer]; break;
            case 5: *out = m->wk[layer]; break;
            case 6: *out = m->wv[layer]; break;
            case 7: *out = m->wo[layer]; break;
            case 8: *out = m->rms_ffn[layer]; break;
            case 9: *out = m->w1[layer]; break;
            case 10: *out = m->w2[layer]; break;
            case 11: *out = m->w3[layer]; break;
            default: fail(AB_ERR_ARGUMENT, "unknown weight id");
        }
    });
}

int ab_llama_cache(ab_llama* m, ab_kvcache** out) {
    return guard([&] {
        if (!m || !out) fail(AB_ERR_ARGUMENT, "null argument");
        *out = m->cache;
    });
}

static void check_steps(const ab_llama* m, const ab_decode_step* steps, uint32_t n,
                        uint32_t extra) {
    if (n != m->c.batch)
        fail(AB_ERR_ARGUMENT, "step needs " + std::to_string(m->c.batch) + " DecodeSteps, got " +
                                  std::to_string(n));
    for (uint32_t b = 0; b < n; b++) {
        if (steps[b].token >= m->c.vocab)
            fail(AB_ERR_ARGUMENT, "token " + std::to_string(steps[b].token) +
                                      " out of range for vocab " + std::to_string(m->c.vocab));
        if ((uint64_t)steps[b].position + extra >= m->c.seq + (extra ? 1 : 0))
            fail(AB_ERR_ARGUMENT, "position " + std::to_string(steps[b].position) +
                                      (extra ? " + " + std::to_string(extra) + " steps passes"
                                             : " beyond") +
                                      " max_seq_len " + std::to_string(m->c.seq));
    }
}

int ab_llama_step(ab_llama* m, const ab_decode_step* steps, uint32_t n, float* logits_host,
                  int32_t* argmax_host) {
    return guard([&] {
        if (!m || !steps) fail(AB_ERR_ARGUMENT, "null argument");
        check_steps(m, steps, n, 0);
        Runtime* rt = m->rt;
        rt->activate();
        if (m->scheme->nodes.empty()) record_step(m, m->scheme, false, m->world > 1);
        std::memcpy(m->h_steps, steps, sizeof(ab_decode_step) * n);
        cuda_check(cudaMemcpyAsync(m->step.data, m->h_steps, sizeof(ab_decode_step) * n,
                                   cudaMemcpyHostToDevice, rt->stream),
                   "deposit steps");
        check(ab_scheme_submit(m->scheme));
        const size_t lbytes = (size_t)n * m->c.vocab * 4;
        const void* lsrc = m->world > 1 ? m->logits_all.data : m->logits.data;
        // a caller buffer page-locked through ab_host_register over the whole copy takes the
        // logits straight from the device (under tensor parallelism too at batch 1, where the
        // gathered [rank][vocab slice] rows are already [vocab]); any other goes through the
        // pinned staging buffer
        const bool direct = logits_host && (m->world == 1 || n == 1) &&
                            host_range_registered(logits_host, lbytes);
        if (logits_host)
            cuda_check(cudaMemcpyAsync(direct ? (void*)logits_host : (void*)m->h_logits, lsrc,
                                       lbytes, cudaMemcpyDeviceToHost, rt->stream),
                       "logits readback");
        if (argmax_host)
            cuda_check(cudaMemcpyAsync(m->h_argmax, m->argmax.data, (size_t)n * 4,
                                       cudaMemcpyDeviceToHost, rt->stream),
                       "argmax readback");
        // the flag word rides along: one synchronisation for the whole step
        cuda_check(cudaMemcpyAsync(m->h_flags, rt->flags, 4, cudaMemcpyDeviceToHost, rt->stream),
                   "flag word readback");
        cuda_check(cudaStreamSynchronize(rt->stream), "step synchronize");
        if (*m->h_flags) rt->check_flags();
        if (logits_host && !direct) {
            if (m->world == 1) {
                std::memcpy(logits_host, m->h_logits, lbytes);
            } else {
                // gathered as [rank][batch][vocab slice] -> [batch][vocab]
                const size_t vl = m->vocab_l;
                for (uint32_t b = 0; b < n; b++)
                    for (int32_t r = 0; r < m->world; r++)
                        std::memcpy(logits_host + (size_t)b * m->c.vocab + r * vl,
                                    m->h_logits + ((size_t)r * n + b) * vl, vl * 4);
            }
        }
        if (argmax_host) std::memcpy(argmax_host, m->h_argmax, (size_t)n * 4);
    });
}

int ab_llama_decode_device(ab_llama* m, const ab_decode_step* start, uint32_t n, uint32_t steps,
                           int32_t* tokens_out) {
    return guard([&] {
        if (!m || !start) fail(AB_ERR_ARGUMENT, "null argument");
        const auto& c = m->c;
        check_steps(m, start, n, steps);
        Runtime* rt = m->rt;
        rt->activate();
        if (m->loop_scheme->nodes.empty()) record_step(m, m->loop_scheme, true, false);
        std::memcpy(m->h_steps, start, sizeof(ab_decode_step) * n);
        cuda_check(cudaMemcpyAsync(m->step.data, m->h_steps, sizeof(ab_decode_step) * n,
                                   cudaMemcpyHostToDevice, rt->stream),
                   "deposit steps");
        for (uint32_t i = 0; i < steps; i++) check(ab_scheme_submit(m->loop_scheme));
        if (tokens_out) {
            std::vector<int32_t> hist((size_t)c.seq * c.batch);
            cuda_check(cudaMemcpyAsync(hist.data(), m->history.data, hist.size() * 4,
                                       cudaMemcpyDeviceToHost, rt->stream),
                       "history readback");
            cuda_check(cudaStreamSynchronize(rt->stream), "decode synchronize");
            for (uint32_t i = 0; i < steps; i++)
                for (uint32_t b = 0; b < n; b++) {
                    const uint64_t p = (uint64_t)start[b].position + 1 + i;
                    tokens_out[(size_t)i * n + b] = p < c.seq ? hist[p * c.batch + b] : -1;
                }
        }
        cuda_check(cudaStreamSynchronize(rt->stream), "decode synchronize");
        rt->check_flags();
    });
}

int ab_llama_prefill_scheme(ab_llama* m, uint32_t stream, uint32_t rows, int32_t head,
                            ab_scheme** out) {
    return guard([&] {
        if (!m || !out) fail(AB_ERR_ARGUMENT, "null argument");
        if (stream >= m->c.batch) fail(AB_ERR_ARGUMENT, "stream out of range");
        m->rt->activate();
        setup_prefill(m);
        if (rows == 0 || rows > m->pf_rows)
            fail(AB_ERR_ARGUMENT, "rows must be 1.." + std::to_string(m->pf_rows));
        *out = prefill_scheme(m, stream, rows, head != 0);
    });
}

int ab_llama_prefill_launches(const ab_llama* m, uint32_t* out) {
    return guard([&] {
        if (!m || !out) fail(AB_ERR_ARGUMENT, "null argument");
        *out = m->pf_launches;
    });
}

int ab_llama_prefill_rows(ab_llama* m, uint32_t rows) {
    return guard([&] {
        if (!m) fail(AB_ERR_ARGUMENT, "null model");
        if (rows > 256) fail(AB_ERR_ARGUMENT, "prefill passes take at most 256 rows");
        m->pf_rows_wanted = rows;
    });
}

}  // extern "C"

namespace {

// Runs positions [pos0, pos0 + n) of cache stream `stream` through prefill passes; the last
// pass ends with the classifier and the greedy pick of its last row when `head`.
void run_prefill(ab_llama* m, uint32_t stream, const int32_t* tokens, uint32_t n, uint32_t pos0,
                 bool head) {
    Runtime* rt = m->rt;
    rt->activate();
    setup_prefill(m);
    const uint32_t R = m->pf_rows;
    // pinned steps for the whole prompt: each pass's copy reads its own slice
    cuda_check(cudaStreamSynchronize(rt->stream), "prefill synchronize");
    for (uint32_t i = 0; i < n; i++) m->h_pf_steps[i] = {(uint32_t)tokens[i], pos0 + i};
    m->pf_launches = 0;
    for (uint32_t done = 0; done < n;) {
        const uint32_t rows = std::min(R, n - done);
        const bool last = done + rows == n;
        ab_scheme* s = prefill_scheme(m, stream, rows, head && last);
        cuda_check(cudaMemcpyAsync(m->pf_step.data, m->h_pf_steps + done,
                                   sizeof(ab_decode_step) * rows, cudaMemcpyHostToDevice,
                                   rt->stream),
                   "deposit prefill steps");
        check(ab_scheme_submit(s));
        m->pf_launches += (uint32_t)s->nodes.size();
        done += rows;
    }
}

void check_prompt(const ab_llama* m, uint32_t stream, const int32_t* tokens, uint32_t n,
                  uint32_t pos0) {
    const auto& c = m->c;
    if (stream >= c.batch)
        fail(AB_ERR_ARGUMENT, "stream " + std::to_string(stream) + " out of range for batch " +
                                  std::to_string(c.batch));
    if (n == 0) fail(AB_ERR_ARGUMENT, "expected at least one prompt token");
    if ((uint64_t)pos0 + n > c.seq)
        fail(AB_ERR_ARGUMENT, "positions " + std::to_string(pos0) + " + " + std::to_string(n) +
                                  " tokens pass max_seq_len " + std::to_string(c.seq));
    for (uint32_t i = 0; i < n; i++)
        if (tokens[i] < 0 || (uint32_t)tokens[i] >= c.vocab)
            fail(AB_ERR_ARGUMENT, "token " + std::to_string(tokens[i]) +
                                      " out of range for vocab " + std::to_string(c.vocab));
}

// Reads back the prefill's last-row logits ([vocab], gathered over the ranks) and greedy id.
void read_prefill_head(ab_llama* m, float* logits_host, int32_t* argmax_host) {
    Runtime* rt = m->rt;
    const size_t vl = m->vocab_l;
    if (logits_host) {
        const void* src = m->world > 1 ? m->pf_logits_all.data : m->pf_logits.data;
        // gathered as [rank][1][vocab slice]: already the vocabulary order
        cuda_check(cudaMemcpyAsync(m->h_pf_logits, src, (size_t)m->world * vl * 4,
                                   cudaMemcpyDeviceToHost, rt->stream),
                   "prefill logits readback");
    }
    int32_t am = 0;
    if (argmax_host)
        cuda_check(cudaMemcpyAsync(&am, m->pf_argmax.data, 4, cudaMemcpyDeviceToHost, rt->stream),
                   "prefill argmax readback");
    cuda_check(cudaStreamSynchronize(rt->stream), "prefill synchronize");
    rt->check_flags();
    if (logits_host) std::memcpy(logits_host, m->h_pf_logits, (size_t)m->c.vocab * 4);
    if (argmax_host) *argmax_host = am;
}

}  // namespace

extern "C" {

int ab_llama_prefill(ab_llama* m, uint32_t stream, const int32_t* tokens, uint32_t n,
                     uint32_t pos0, float* logits_host, int32_t* argmax_host) {
    return guard([&] {
        if (!m || !tokens) fail(AB_ERR_ARGUMENT, "null argument");
        check_prompt(m, stream, tokens, n, pos0);
        run_prefill(m, stream, tokens, n, pos0, true);
        read_prefill_head(m, logits_host, argmax_host);
    });
}

int ab_llama_generate_tokens(ab_llama* m, const int32_t* prompt, uint32_t prompt_len,
                             uint32_t max_new_tokens, int32_t has_stop, int32_t stop_on,
                             int32_t* out_tokens, uint32_t cap, uint32_t* out_len,
                             double* tokens_per_second) {
    return guard([&] {
        if (!m) fail(AB_ERR_ARGUMENT, "null model");
        if (m->c.batch != 1) fail(AB_ERR_ARGUMENT, "generate_tokens needs a batch-1 model");
        if (!prompt || prompt_len == 0) fail(AB_ERR_ARGUMENT, "expected at least one prompt token");
        const auto& c = m->c;
        // generate_tokens (src/generate.rs:43-91) steps through positions 0 .. limit - 1:
        // prompt tokens are forced ids until the prompt runs out, then greedy picks; a next
        // id equal to the stop id ends it before it is emitted.
        const uint32_t cap_steps = std::min(max_new_tokens, c.seq);
        const uint32_t limit = cap_steps > 0 ? cap_steps - 1 : 0;
        const uint32_t S = std::min(prompt_len, limit);  // prompt positions stepped through
        uint32_t k_stop = 0;  // first forced id equal to the stop id (0: none)
        for (uint32_t k = 1; has_stop && k <= S && k < prompt_len; k++)
            if (prompt[k] == stop_on) {
                k_stop = k;
                break;
            }
        const uint32_t P = k_stop ? k_stop : S;
        const bool sample = !k_stop && S == prompt_len;  // the last prompt step picks the next id
        uint32_t n = 0;
        auto emit = [&](int32_t t) {
            if (out_tokens && n < cap) out_tokens[n] = t;
            n++;
        };
        double elapsed = 0.0;
        uint32_t decoded = 0;
        if (P > 0) {
            check_prompt(m, 0, prompt, P, 0);
            run_prefill(m, 0, prompt, P, 0, sample);
            const uint32_t last_forced = k_stop ? k_stop - 1 : std::min(P, prompt_len - 1);
            for (uint32_t k = 1; k <= last_forced; k++) emit(prompt[k]);
            if (sample) {
                int32_t next = 0;
                read_prefill_head(m, nullptr, &next);
                const auto start = std::chrono::steady_clock::now();
                for (uint32_t pos = P;; pos++) {
                    if (has_stop && next == stop_on) break;
                    emit(next);
                    if (pos >= limit) break;
                    ab_decode_step st = {(uint32_t)next, pos};
                    check(ab_llama_step(m, &st, 1, nullptr, &next));
                    decoded++;
                }
                elapsed = std::chrono::duration<double>(std::chrono::steady_clock::now() - start)
                              .count();
            }
            m->rt->activate();
            cuda_check(cudaStreamSynchronize(m->rt->stream), "generate synchronize");
            m->rt->check_flags();
        }
        if (out_len) *out_len = n;
        if (tokens_per_second) *tokens_per_second = elapsed > 0.0 ? decoded / elapsed : 0.0;
    });
}

int ab_llama_step_trace(ab_llama* m, uint64_t* out, uint32_t cap, uint32_t* barriers,
                        uint32_t* grid) {
    return guard([&] {
        if (!m || !barriers || !grid) fail(AB_ERR_ARGUMENT, "null argument");
        std::vector<uint64_t> t;
        m->rt->activate();
        cuda_check(cudaStreamSynchronize(m->rt->stream), "trace synchronize");
        if (!fused_step_trace(m->fused, &t, barriers, grid)) {
            *barriers = 0;
            *grid = 0;
            return;
        }
        if (out) std::memcpy(out, t.data(), std::min<size_t>(cap, t.size()) * 8);
    });
}

int ab_llama_scheme(ab_llama* m, ab_scheme** out) {
    return guard([&] {
        if (!m || !out) fail(AB_ERR_ARGUMENT, "null argument");
        if (m->scheme->nodes.empty()) record_step(m, m->scheme, false, m->world > 1);
        *out = m->scheme;
    });
}

int ab_llama_logits(ab_llama* m, ab_tensor* out) {
    return guard([&] {
        if (!m || !out) fail(AB_ERR_ARGUMENT, "null argument");
        *out = m->world > 1 ? m->logits_all : m->logits;
    });
}

int ab_llama_reset(ab_llama* m) {
    return guard([&] {
        if (!m) fail(AB_ERR_ARGUMENT, "null model");
        check(ab_kvcache_zero(m->cache));
        m->rt->activate();
        cuda_check(cudaStreamSynchronize(m->rt->stream), "reset synchronize");
    });
}

int ab_llama_as_model(ab_llama* m, ab_autoregressive_model* out) {
    return guard([&] {
        if (!m || !out) fail(AB_ERR_ARGUMENT, "null argument");
        if (m->c.batch != 1) fail(AB_ERR_ARGUMENT, "AutoregressiveModel view needs batch 1");
        out->self = m;
        out->vocab_size = vt_vocab;
        out->max_seq_len = vt_seq;
        out->step = vt_step;
    });
}

int ab_llama_destroy(ab_llama* m) {
    return guard([&] { destroy_model(m); });
}

}  // extern "C"
