// Host decode loop (src/generate.rs, src/tokenizer.rs:179-189) and the Llama-shaped
// model the harness decodes with. The reference leaves model assembly to architecture
// crates (README.md:5,21); this one composes the modules in the llama2.c order:
// Embedding, layers x [CausalAttentionBlock, SwiGluBlock], final RmsNorm, classifier.
//
// One decode step is one CUDA graph recorded once: the DecodeStep parcel is refreshed
// by a deposit before each replay, so nothing is re-recorded per token.
#include <chrono>
#include <cstring>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "ops.h"

using namespace ab;

namespace ab {

// Device argmax of each row of logits [batch, vocab]: first index of the maximum, the
// tie rule of sample_argmax (src/tokenizer.rs:179-189). NaNs never win.
__global__ void __launch_bounds__(1024)
    argmax_kernel(const float* __restrict__ logits, uint32_t vocab, int32_t* __restrict__ out) {
    pdl_wait();
    __shared__ float bv[32];
    __shared__ uint32_t bi[32];
    const float* row = logits + (uint64_t)blockIdx.x * vocab;
    float best = -INFINITY;
    uint32_t idx = 0xffffffffu;
    for (uint32_t i = threadIdx.x; i < vocab; i += blockDim.x) {
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
        if (lane == 0) out[blockIdx.x] = idx == 0xffffffffu ? 0 : (int32_t)idx;
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
    ab_tensor embed = {}, wcls = {}, rms_final = {};
    std::vector<ab_tensor> rms_att, wq, wk, wv, wo, rms_ffn, w1, w2, w3;
    ab_kvcache* cache = nullptr;
    ab_attention_block* attn = nullptr;
    ab_swiglu_block* ffn = nullptr;
    ab_tensor x = {}, logits = {}, step = {}, argmax = {}, history = {};
    ab_scheme* scheme = nullptr;       // one decode step
    ab_scheme* loop_scheme = nullptr;  // one decode step + device sample feedback
    GemmScratch cls_tc;                // classifier's tensor-core GEMM scratch
    float* h_logits = nullptr;  // pinned [batch, vocab]
    int32_t* h_argmax = nullptr;
    ab_decode_step* h_steps = nullptr;
    std::vector<float> vt_logits;  // host logits handed out through the vtable
};

namespace {

void free_t(Runtime* rt, ab_tensor& t) {
    if (t.data) cudaFree(t.data);
    (void)rt;
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

void destroy_model(ab_llama* m) {
    if (!m) return;
    Runtime* rt = m->rt;
    if (rt) {
        rt->activate();
        cudaStreamSynchronize(rt->stream);
    }
    if (m->scheme) ab_scheme_destroy(m->scheme);
    if (m->loop_scheme) ab_scheme_destroy(m->loop_scheme);
    free_tc_scratch(&m->cls_tc);
    if (m->attn) ab_attention_block_destroy(m->attn);
    if (m->ffn) ab_swiglu_block_destroy(m->ffn);
    if (m->cache) ab_kvcache_destroy(m->cache);
    for (auto* v : {&m->rms_att, &m->wq, &m->wk, &m->wv, &m->wo, &m->rms_ffn, &m->w1, &m->w2,
                    &m->w3})
        for (auto& t : *v) free_t(rt, t);
    for (ab_tensor* t : {&m->embed, &m->wcls, &m->rms_final, &m->x, &m->logits, &m->step,
                         &m->argmax, &m->history})
        free_t(rt, *t);
    if (m->h_logits) cudaFreeHost(m->h_logits);
    if (m->h_argmax) cudaFreeHost(m->h_argmax);
    if (m->h_steps) cudaFreeHost(m->h_steps);
    delete m;
}

// Records the full decode step into `s` (with the device sample feedback when asked).
void record_step(ab_llama* m, ab_scheme* s, bool feedback) {
    s->nodes.clear();
    s->dirty = true;
    const auto& c = m->c;
    ab_tensor x = m->x;
    if (c.batch == 1) {
        x.rank = 1;
        x.dims[0] = c.dim;
    }
    check(ab_embedding_record(s, m->embed, m->step, x));
    for (uint32_t l = 0; l < c.layers; l++) {
        ab_tensor key, value;
        check(ab_kvcache_layer(m->cache, l, &key, &value));
        ab_attention_weights aw = {m->rms_att[l], m->wq[l], m->wk[l], m->wv[l], m->wo[l]};
        check(ab_attention_block_record(m->attn, s, x, &aw, key, value, m->step));
        ab_swiglu_weights fw = {m->rms_ffn[l], m->w1[l], m->w3[l], m->w2[l]};
        check(ab_swiglu_block_record(m->ffn, s, x, &fw));
    }
    // final RmsNorm fused into the classifier GEMV's prologue
    GemvParams g = {};
    g.seg[0] = m->wcls.data;
    g.seg_rows[0] = c.vocab;
    g.n_rows = c.vocab;
    g.units = (c.vocab + 1) / 2;
    g.K = c.dim;
    g.x = m->x.data;
    g.x_dtype = AB_F32;
    g.x_stride = c.dim;
    g.norm_w = m->rms_final.data;
    g.norm_dtype = m->rms_final.dtype;
    g.eps = c.norm_eps;
    g.out = m->logits.data;
    g.out_dtype = AB_F32;
    g.out_stride = c.vocab;
    attach_tc_scratch(&g, m->cls_tc);
    record_gemv(s, "final_norm_classifier", g, c.dtype, c.batch, kProNorm, kEpiStore);
    const float* lg = (const float*)m->logits.data;
    int32_t* am = (int32_t*)m->argmax.data;
    const uint32_t vocab = c.vocab, batch = c.batch;
    s->add("argmax", [=](cudaStream_t st) {
        return launch(st, dim3(batch), dim3(1024), 0, true, argmax_kernel, lg, vocab, am);
    });
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
        if (!rt || !cfg || !out) fail(AB_ERR_ARGUMENT, "null argument");
        const ab_llama_config c = *cfg;
        if (!c.dim || !c.layers || !c.heads || !c.kv_heads || !c.head_dim || !c.hidden || !c.vocab ||
            !c.seq || !c.batch)
            fail(AB_ERR_ARGUMENT, "model dims must be non-zero");
        if (c.heads * c.head_dim != c.dim)
            fail(AB_ERR_VALIDATION, "heads * head_dim must equal dim");
        if (c.dtype != AB_F32 && c.dtype != AB_BF16) fail(AB_ERR_ARGUMENT, "dtype f32 or bf16");
        auto* m = new ab_llama();
        m->rt = rt;
        m->c = c;
        try {
            const int32_t dt = c.dtype;
            const uint32_t qd = c.heads * c.head_dim, kvd = c.kv_heads * c.head_dim;
            m->embed = alloc_t(rt, dt, {c.vocab, c.dim});
            m->wcls = alloc_t(rt, dt, {c.vocab, c.dim});
            m->rms_final = alloc_t(rt, dt, {c.dim});
            for (uint32_t l = 0; l < c.layers; l++) {
                m->rms_att.push_back(alloc_t(rt, dt, {c.dim}));
                m->wq.push_back(alloc_t(rt, dt, {qd, c.dim}));
                m->wk.push_back(alloc_t(rt, dt, {kvd, c.dim}));
                m->wv.push_back(alloc_t(rt, dt, {kvd, c.dim}));
                m->wo.push_back(alloc_t(rt, dt, {c.dim, qd}));
                m->rms_ffn.push_back(alloc_t(rt, dt, {c.dim}));
                m->w1.push_back(alloc_t(rt, dt, {c.hidden, c.dim}));
                m->w2.push_back(alloc_t(rt, dt, {c.dim, c.hidden}));
                m->w3.push_back(alloc_t(rt, dt, {c.hidden, c.dim}));
            }
            check(ab_kvcache_create(rt, c.layers, c.seq, c.kv_heads, c.head_dim, dt, c.batch,
                                    &m->cache));
            check(ab_attention_block_create(rt, c.dim, c.heads, c.seq, c.batch, c.rope_theta,
                                            &m->attn));
            check(ab_swiglu_block_create(rt, c.dim, c.hidden, c.batch, &m->ffn));
            alloc_tc_scratch(rt, &m->cls_tc, c.batch, c.dim, (c.vocab + 127) / 128);
            m->x = alloc_t(rt, AB_F32, {c.batch, c.dim});
            m->logits = alloc_t(rt, AB_F32, {c.batch, c.vocab});
            m->argmax = alloc_t(rt, AB_U32, {c.batch});
            m->history = alloc_t(rt, AB_U32, {c.seq, c.batch});
            check(ab_step_parcel(rt, c.batch, &m->step));
            cuda_check(cudaMallocHost(&m->h_logits, (size_t)c.batch * c.vocab * 4), "pinned logits");
            cuda_check(cudaMallocHost(&m->h_argmax, (size_t)c.batch * 4), "pinned argmax");
            cuda_check(cudaMallocHost(&m->h_steps, (size_t)c.batch * sizeof(ab_decode_step)),
                       "pinned steps");
            check(ab_scheme_create(rt, &m->scheme));
            check(ab_scheme_create(rt, &m->loop_scheme));
        } catch (...) {
            destroy_model(m);
            throw;
        }
        *out = m;
    });
}

int ab_llama_init_synthetic(ab_llama* m, uint64_t seed, float std) {
    return guard([&] {
        if (!m) fail(AB_ERR_ARGUMENT, "null model");
        ab_runtime* rt = static_cast<ab_runtime*>(m->rt);
        auto fill = [&](ab_tensor& t, uint64_t stream, float mean, float sd) {
            check(ab_tensor_fill_normal(rt, t, seed, stream, mean, sd));
        };
        // stream ids shared with the CPU oracle's generator
        fill(m->embed, 1, 0.0f, std);
        fill(m->rms_final, 2, 1.0f, 0.01f);
        fill(m->wcls, 3, 0.0f, std);
        for (uint32_t l = 0; l < m->c.layers; l++) {
            const uint64_t b = 16 + 16ull * l;
            fill(m->rms_att[l], b + 0, 1.0f, 0.01f);
            fill(m->wq[l], b + 1, 0.0f, std);
            fill(m->wk[l], b + 2, 0.0f, std);
            fill(m->wv[l], b + 3, 0.0f, std);
            fill(m->wo[l], b + 4, 0.0f, std);
            fill(m->rms_ffn[l], b + 5, 1.0f, 0.01f);
            fill(m->w1[l], b + 6, 0.0f, std);
            fill(m->w2[l], b + 7, 0.0f, std);
            fill(m->w3[l], b + 8, 0.0f, std);
        }
        m->rt->activate();
        cuda_check(cudaStreamSynchronize(m->rt->stream), "init synchronize");
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

int ab_llama_step(ab_llama* m, const ab_decode_step* steps, uint32_t n, float* logits_host,
                  int32_t* argmax_host) {
    return guard([&] {
        if (!m || !steps) fail(AB_ERR_ARGUMENT, "null argument");
        if (n != m->c.batch)
            fail(AB_ERR_ARGUMENT, "step needs " + std::to_string(m->c.batch) + " DecodeSteps, got " +
                                      std::to_string(n));
        for (uint32_t b = 0; b < n; b++) {
            if (steps[b].token >= m->c.vocab)
                fail(AB_ERR_ARGUMENT, "token " + std::to_string(steps[b].token) +
                                          " out of range for vocab " + std::to_string(m->c.vocab));
            if (steps[b].position >= m->c.seq)
                fail(AB_ERR_ARGUMENT, "position " + std::to_string(steps[b].position) +
                                          " beyond max_seq_len " + std::to_string(m->c.seq));
        }
        Runtime* rt = m->rt;
        rt->activate();
        if (m->scheme->nodes.empty()) record_step(m, m->scheme, false);
        std::memcpy(m->h_steps, steps, sizeof(ab_decode_step) * n);
        cuda_check(cudaMemcpyAsync(m->step.data, m->h_steps, sizeof(ab_decode_step) * n,
                                   cudaMemcpyHostToDevice, rt->stream),
                   "deposit steps");
        check(ab_scheme_submit(m->scheme));
        const size_t lbytes = (size_t)n * m->c.vocab * 4;
        if (logits_host)
            cuda_check(cudaMemcpyAsync(m->h_logits, m->logits.data, lbytes, cudaMemcpyDeviceToHost,
                                       rt->stream),
                       "logits readback");
        if (argmax_host)
            cuda_check(cudaMemcpyAsync(m->h_argmax, m->argmax.data, (size_t)n * 4,
                                       cudaMemcpyDeviceToHost, rt->stream),
                       "argmax readback");
        cuda_check(cudaStreamSynchronize(rt->stream), "step synchronize");
        rt->check_flags();
        if (logits_host) std::memcpy(logits_host, m->h_logits, lbytes);
        if (argmax_host) std::memcpy(argmax_host, m->h_argmax, (size_t)n * 4);
    });
}

int ab_llama_decode_device(ab_llama* m, const ab_decode_step* start, uint32_t n, uint32_t steps,
                           int32_t* tokens_out) {
    return guard([&] {
        if (!m || !start) fail(AB_ERR_ARGUMENT, "null argument");
        const auto& c = m->c;
        if (n != c.batch)
            fail(AB_ERR_ARGUMENT, "decode needs " + std::to_string(c.batch) + " start steps");
        for (uint32_t b = 0; b < n; b++) {
            if (start[b].token >= c.vocab) fail(AB_ERR_ARGUMENT, "start token out of range");
            if ((uint64_t)start[b].position + steps > c.seq)
                fail(AB_ERR_ARGUMENT, "decode of " + std::to_string(steps) + " steps from position " +
                                          std::to_string(start[b].position) + " passes max_seq_len " +
                                          std::to_string(c.seq));
        }
        Runtime* rt = m->rt;
        rt->activate();
        if (m->loop_scheme->nodes.empty()) record_step(m, m->loop_scheme, true);
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

int ab_llama_scheme(ab_llama* m, ab_scheme** out) {
    return guard([&] {
        if (!m || !out) fail(AB_ERR_ARGUMENT, "null argument");
        if (m->scheme->nodes.empty()) record_step(m, m->scheme, false);
        *out = m->scheme;
    });
}

int ab_llama_logits(ab_llama* m, ab_tensor* out) {
    return guard([&] {
        if (!m || !out) fail(AB_ERR_ARGUMENT, "null argument");
        *out = m->logits;
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
