// Modules of src/modules.rs on the fused sm_100a kernels.
//
// CausalAttentionBlock::record (op order src/blocks.rs:178-259) becomes three launches:
//   1. RMSNorm prologue + [wq; wk; wv] GEMV + RoPE + K/V cache append   (gemv.cu)
//   2. flash-decoding attention with in-kernel split combine             (attention.cu)
//   3. wo GEMV + residual add into x                                     (gemv.cu)
// SwiGluBlock::record (src/blocks.rs:262-278) becomes two:
//   1. RMSNorm prologue + interleaved (w1, w3) GEMV + SwiGLU            (gemv.cu)
//   2. w2 GEMV + residual add into x                                     (gemv.cu)
#include <algorithm>

#include "common.cuh"
#include "internal.h"
#include "ops.h"

using namespace ab;

struct ab_kvcache {
    Runtime* rt;
    uint32_t layers, seq, kv_heads, head, batch;
    int32_t dtype;
    ab_tensor key, value;  // [layers, batch, seq, kv_heads, head] stored flat
};

struct ab_attention_block {
    Runtime* rt;
    uint32_t hidden, heads, head, seq, max_batch;
    float theta;
    uint32_t nsplit_max;
    uint64_t part_floats = 0;  // floats of `part`
    float* q = nullptr;         // [max_batch, heads * head] rotated queries
    void* attn_out = nullptr;   // [max_batch, heads * head] (f32 or bf16)
    float* part = nullptr;      // split partials
    uint32_t* counters = nullptr;
    GemmScratch tc;  // tensor-core GEMM scratch (max_batch > kGemvMaxBatch)
    ab_comm* tp = nullptr;   // tensor parallelism: wo output is all-reduced into x
    float* tp_y = nullptr;   // [max_batch, hidden] partial projection
};

struct ab_swiglu_block {
    Runtime* rt;
    uint32_t hidden, inter, max_batch;
    void* hb = nullptr;  // [max_batch, inter] (f32 or bf16)
    GemmScratch tc;
    ab_comm* tp = nullptr;
    float* tp_y = nullptr;
};

namespace {

// x [hidden] -> batch 1, [B, hidden] -> batch B.
uint32_t x_batch(const ab_tensor& x, uint32_t hidden, uint32_t max_batch) {
    expect_data("x", x);
    expect_dtype("x", x, AB_F32);
    expect_rank_in("x", x, 1, 2);
    expect_dim("x", x, x.rank - 1, "hidden", hidden);
    const uint32_t b = x.rank == 2 ? x.dims[0] : 1;
    if (b > max_batch)
        invalid("parameter `x`: batch " + std::to_string(b) + " exceeds the block's max_batch " +
                std::to_string(max_batch));
    return b;
}

void expect_linear(const char* param, const ab_tensor& w, uint32_t rows, uint32_t cols,
                   int32_t dtype) {
    expect_data(param, w);
    expect_rank(param, w, 2);
    expect_dtype(param, w, dtype);
    expect_dim(param, w, 1, "in", cols);
    if (rows) expect_dim(param, w, 0, "out", rows);
}

void* device_alloc(Runtime* rt, size_t bytes) {
    void* p = nullptr;
    rt->activate();
    cuda_check(cudaMalloc(&p, std::max<size_t>(bytes, 16)), "cudaMalloc");
    cuda_check(cudaMemset(p, 0, std::max<size_t>(bytes, 16)), "cudaMemset");
    return p;
}

}  // namespace

namespace ab {

ab_attention_block* attention_block_new(ab_runtime* rt, uint32_t hidden, uint32_t heads,
                                        uint32_t head, uint32_t seq_len, uint32_t max_batch,
                                        float rope_theta, ab_comm* tp) {
    if (!heads || !head) fail(AB_ERR_ARGUMENT, "query_heads and head size must be > 0");
    if (!seq_len || !max_batch) fail(AB_ERR_ARGUMENT, "seq_len and max_batch must be > 0");
    auto* b = new ab_attention_block();
    b->rt = rt;
    b->hidden = hidden;
    b->heads = heads;
    b->head = head;
    b->seq = seq_len;
    b->max_batch = max_batch;
    b->theta = rope_theta;
    b->tp = tp;
    // worst case over every kv head count the weights may bring (at most one per head)
    b->nsplit_max = attention_max_splits(max_batch * heads, seq_len, rt->sm_count, 256);
    uint64_t floats = 0, counters = 0;
    attention_scratch_size(max_batch, heads, head, b->nsplit_max, &floats, &counters);
    const uint64_t qd = (uint64_t)heads * head;
    try {
        b->q = (float*)device_alloc(rt, max_batch * qd * 4);
        b->attn_out = device_alloc(rt, max_batch * qd * 4);
        b->part = (float*)device_alloc(rt, floats * 4);
        b->part_floats = floats;
        b->counters = (uint32_t*)device_alloc(rt, counters * 4);
        if (tp) b->tp_y = (float*)device_alloc(rt, (size_t)max_batch * hidden * 4);
        alloc_tc_scratch(rt, &b->tc, max_batch, (uint32_t)std::max<uint64_t>(qd, hidden),
                         (uint32_t)((3 * std::max<uint64_t>(qd, hidden) + 127) / 128));
    } catch (...) {
        cudaFree(b->q);
        cudaFree(b->attn_out);
        cudaFree(b->part);
        cudaFree(b->counters);
        if (b->tp_y) cudaFree(b->tp_y);
        free_tc_scratch(&b->tc);
        delete b;
        throw;
    }
    return b;
}

ab_swiglu_block* swiglu_block_new(ab_runtime* rt, uint32_t hidden, uint32_t intermediate,
                                  uint32_t max_batch, ab_comm* tp) {
    if (!hidden || !intermediate || !max_batch)
        fail(AB_ERR_ARGUMENT, "hidden, intermediate and max_batch must be > 0");
    auto* b = new ab_swiglu_block();
    b->rt = rt;
    b->hidden = hidden;
    b->inter = intermediate;
    b->max_batch = max_batch;
    b->tp = tp;
    try {
        b->hb = device_alloc(rt, (size_t)max_batch * intermediate * 4);
        if (tp) b->tp_y = (float*)device_alloc(rt, (size_t)max_batch * hidden * 4);
        alloc_tc_scratch(rt, &b->tc, max_batch, std::max(hidden, intermediate),
                         std::max((intermediate + 63) / 64, (hidden + 127) / 128));
    } catch (...) {
        if (b->hb) cudaFree(b->hb);
        if (b->tp_y) cudaFree(b->tp_y);
        free_tc_scratch(&b->tc);
        delete b;
        throw;
    }
    return b;
}

}  // namespace ab

extern "C" {

int ab_embedding_record(ab_scheme* s, ab_tensor table, ab_tensor step, ab_tensor x) {
    return guard([&] {
        if (!s) fail(AB_ERR_ARGUMENT, "null scheme");
        record_embed(s, table, step, x);
    });
}

int ab_rmsnorm_record(ab_scheme* s, ab_tensor x, ab_tensor weight, ab_tensor out) {
    return guard([&] {
        if (!s) fail(AB_ERR_ARGUMENT, "null scheme");
        record_rmsnorm_ref(s, x, weight, out, 1e-5f);
    });
}

int ab_rmsnorm_record_inplace(ab_scheme* s, ab_tensor x, ab_tensor weight) {
    return guard([&] {
        if (!s) fail(AB_ERR_ARGUMENT, "null scheme");
        record_rmsnorm_ref(s, x, weight, x, 1e-5f);
    });
}

// ---- KvCache ---------------------------------------------------------------------------
int ab_kvcache_create(ab_runtime* rt, uint32_t layers, uint32_t seq_len, uint32_t kv_heads,
                      uint32_t head_size, int32_t dtype, uint32_t batch, ab_kvcache** out) {
    return guard([&] {
        if (!rt || !out) fail(AB_ERR_ARGUMENT, "null argument");
        if (!layers || !seq_len || !kv_heads || !head_size || !batch)
            fail(AB_ERR_ARGUMENT, "KvCache dims must be non-zero");
        if (dtype != AB_F32 && dtype != AB_BF16) fail(AB_ERR_ARGUMENT, "KvCache dtype f32 or bf16");
        auto* c = new ab_kvcache();
        c->rt = rt;
        c->layers = layers;
        c->seq = seq_len;
        c->kv_heads = kv_heads;
        c->head = head_size;
        c->batch = batch;
        c->dtype = dtype;
        const uint64_t n = (uint64_t)layers * batch * seq_len * kv_heads * head_size;
        const uint32_t flat[1] = {0};
        (void)flat;
        try {
            for (ab_tensor* t : {&c->key, &c->value}) {
                t->dtype = dtype;
                t->rank = 1;
                t->dims[0] = 0;
                t->data = device_alloc(rt, n * dtype_size(dtype));
            }
        } catch (...) {
            if (c->key.data) cudaFree(c->key.data);
            if (c->value.data) cudaFree(c->value.data);
            delete c;
            throw;
        }
        *out = c;
    });
}

int ab_kvcache_layer(const ab_kvcache* c, uint32_t layer, ab_tensor* key, ab_tensor* value) {
    return guard([&] {
        if (!c || !key || !value) fail(AB_ERR_ARGUMENT, "null argument");
        if (layer >= c->layers)
            invalid("KvCache::layer: layer " + std::to_string(layer) + " out of range (" +
                    std::to_string(c->layers) + " layers)");
        const uint64_t per = (uint64_t)c->batch * c->seq * c->kv_heads * c->head;
        const size_t esz = dtype_size(c->dtype);
        for (int which = 0; which < 2; which++) {
            ab_tensor t = {};
            t.dtype = c->dtype;
            t.data = (char*)(which ? c->value.data : c->key.data) + layer * per * esz;
            if (c->batch == 1) {
                t.rank = 3;
                t.dims[0] = c->seq;
                t.dims[1] = c->kv_heads;
                t.dims[2] = c->head;
            } else {
                t.rank = 4;
                t.dims[0] = c->batch;
                t.dims[1] = c->seq;
                t.dims[2] = c->kv_heads;
                t.dims[3] = c->head;
            }
            *(which ? value : key) = t;
        }
    });
}

int ab_kvcache_zero(ab_kvcache* c) {
    return guard([&] {
        if (!c) fail(AB_ERR_ARGUMENT, "null cache");
        const uint64_t n = (uint64_t)c->layers * c->batch * c->seq * c->kv_heads * c->head;
        c->rt->activate();
        cuda_check(cudaMemsetAsync(c->key.data, 0, n * dtype_size(c->dtype), c->rt->stream),
                   "zero cache");
        cuda_check(cudaMemsetAsync(c->value.data, 0, n * dtype_size(c->dtype), c->rt->stream),
                   "zero cache");
    });
}

int ab_kvcache_destroy(ab_kvcache* c) {
    return guard([&] {
        if (!c) return;
        c->rt->activate();
        cudaStreamSynchronize(c->rt->stream);
        cudaFree(c->key.data);
        cudaFree(c->value.data);
        delete c;
    });
}

// ---- CausalAttentionBlock ------------------------------------------------------------------
int ab_attention_block_create(ab_runtime* rt, uint32_t hidden, uint32_t query_heads,
                              uint32_t seq_len, uint32_t max_batch, float rope_theta,
                              ab_attention_block** out) {
    return guard([&] {
        if (!rt || !out) fail(AB_ERR_ARGUMENT, "null argument");
        if (query_heads == 0 || hidden % query_heads != 0)
            fail(AB_ERR_VALIDATION, "hidden " + std::to_string(hidden) +
                                        " is not divisible by query_heads " +
                                        std::to_string(query_heads));
        *out = attention_block_new(rt, hidden, query_heads, hidden / query_heads, seq_len,
                                   max_batch, rope_theta, nullptr);
    });
}

int ab_attention_block_record(ab_attention_block* blk, ab_scheme* s, ab_tensor x,
                              const ab_attention_weights* w, ab_tensor key, ab_tensor value,
                              ab_tensor step) {
    return guard([&] {
        if (!blk || !s || !w) fail(AB_ERR_ARGUMENT, "null argument");
        const uint32_t hidden = blk->hidden, head = blk->head, heads = blk->heads;
        const uint32_t qd = heads * head;
        const uint32_t batch = x_batch(x, hidden, blk->max_batch);
        expect_data("norm", w->norm);
        expect_rank("norm", w->norm, 1);
        expect_float("norm", w->norm);
        expect_dim("norm", w->norm, 0, "hidden", hidden);
        const int32_t wdt = w->query.dtype;
        if (wdt != AB_F32 && wdt != AB_BF16) expect_float("query", w->query);
        expect_linear("query", w->query, qd, hidden, wdt);
        expect_linear("key", w->key, 0, hidden, wdt);
        expect_linear("value", w->value, 0, hidden, wdt);
        expect_linear("output", w->output, hidden, qd, wdt);
        const uint32_t kvd = w->key.dims[0];
        if (w->value.dims[0] != kvd) invalid("attention: wk and wv row counts differ");
        if (kvd > qd || kvd % 2 != 0)
            invalid("attention: kv width must be even and no wider than q");
        if (head > 128) invalid("attention: head size " + std::to_string(head) + " exceeds 128");
        if (kvd % head) invalid("attention: kv width must be a whole number of heads");
        const uint32_t kv_heads = kvd / head;
        // cache views: [B, seq, kv, head] (a cache per batch row) or [seq, kv, head] (one
        // cache every row reads and appends to: at batch 1, or the consecutive positions of
        // one sequence -- a prompt -- whose rows must then carry distinct positions)
        expect_data("key", key);
        expect_data("value", value);
        expect_float("key", key);
        expect_dtype("value", value, key.dtype);
        const int cr = key.rank == 3 ? 3 : 4;
        expect_rank("key", key, cr);
        expect_rank("value", value, cr);
        const int o = cr - 3;
        if (cr == 4) {
            if (key.dims[0] < batch) expect_dim("key", key, 0, "batch", batch);
        }
        expect_dim("key", key, o + 0, "seq", blk->seq);
        expect_dim("key", key, o + 1, "kv_heads", kv_heads);
        expect_dim("key", key, o + 2, "head", head);
        for (int a = 0; a < cr; a++)
            if (value.dims[a] != key.dims[a])
                invalid("parameter `value`: dims must match key " + shape_str(key));
        expect_step(step, batch);
        const void* segs[3] = {w->query.data, w->key.data, w->value.data};
        if (!gemv_fusable(wdt, hidden, segs, 3) || !gemv_fusable(wdt, qd, &w->output.data, 1))
            invalid("attention: hidden and q widths must be multiples of 8 (bf16) or 4 (f32) "
                    "elements with 16-byte aligned weights");
        if (!attention_fusable(heads, kv_heads, head, key.dtype))
            invalid("attention: fused path needs query_heads / kv_heads in {1, 2, 4, 8} and "
                    "head * element size a multiple of 16 bytes");

        const uint64_t cache_stride = cr == 3 ? 0 : (uint64_t)blk->seq * kvd;
        const Step* st = (const Step*)step.data;
        uint32_t* flags = s->rt ? s->rt->flags : nullptr;
        const int32_t act = wdt;  // activation dtype feeding the projections

        // 1. norm + QKV + RoPE + cache append
        GemvParams g = {};
        g.seg[0] = w->query.data;
        g.seg[1] = w->key.data;
        g.seg[2] = w->value.data;
        g.seg_rows[0] = qd;
        g.seg_rows[1] = kvd;
        g.seg_rows[2] = kvd;
        g.n_rows = qd + 2 * kvd;
        g.units = g.n_rows / 2;
        g.K = hidden;
        g.x = x.data;
        g.x_dtype = AB_F32;
        g.x_stride = hidden;
        g.norm_w = w->norm.data;
        g.norm_dtype = w->norm.dtype;
        g.eps = 1e-5f;
        g.q = blk->q;
        g.qd = qd;
        g.kvd = kvd;
        g.head = head;
        g.seq = blk->seq;
        g.theta = blk->theta;
        g.kcache = key.data;
        g.vcache = value.data;
        g.kv_dtype = key.dtype;
        g.cache_stride = cache_stride;
        g.step = st;
        g.flags = flags;
        attach_tc_scratch(&g, blk->tc);
        // validation is complete: nothing below throws a validation error after the
        // first node is added
        const uint32_t nsplit = attention_choose_splits(
            batch, kv_heads, blk->seq, s->rt ? s->rt->sm_count : 148, blk->nsplit_max);
        AttnParams a = {};
        a.q = blk->q;
        a.kcache = key.data;
        a.vcache = value.data;
        a.kv_dtype = key.dtype;
        a.cache_stride = cache_stride;
        a.out = blk->attn_out;
        a.out_dtype = act;
        a.heads = heads;
        a.kv_heads = kv_heads;
        a.head = head;
        a.seq = blk->seq;
        a.batch = batch;
        a.nsplit = nsplit;
        // a split covers several 64-position tiles: a split pays a partial write and a
        // share of the fold, which shorter ones do not earn back
        a.min_chunk = attention_min_chunk();
        uint64_t floats = 0, counters = 0;
        attention_scratch_size(batch, heads, head, nsplit, &floats, &counters);
        a.part_o = blk->part;
        a.part_ml = blk->part + (uint64_t)batch * heads * nsplit * head;
        a.part_cap = blk->part_floats;
        a.counters = blk->counters;
        a.step = st;
        a.flags = flags;

        GemvParams o2 = {};
        o2.seg[0] = w->output.data;
        o2.seg_rows[0] = hidden;
        o2.n_rows = hidden;
        o2.units = (hidden + 1) / 2;
        o2.K = qd;
        o2.x = blk->attn_out;
        o2.x_dtype = act;
        o2.x_stride = qd;
        o2.out = x.data;
        o2.out_dtype = AB_F32;
        o2.out_stride = hidden;
        attach_tc_scratch(&o2, blk->tc);

        const size_t before = s->nodes.size();
        try {
            record_gemv(s, "attn_qkv_rope", g, wdt, batch, kProNorm, kEpiQkv);
            record_attention(s, "attn_decode", a);
            if (blk->tp) {
                // partial projection of this rank's heads; rank 0 adds the residual, and
                // the all-reduce sums every rank's part straight into x: over NVLink peer
                // slots at GEMV batches, else through NCCL
                o2.out = blk->tp_y;
                o2.addend = comm_rank(blk->tp) == 0 ? (const float*)x.data : nullptr;
                if (comm_has_peers(blk->tp) && batch <= kTpPeerMaxRows) {
                    const TpPush tgt = comm_push_target(blk->tp);
                    o2.out = tgt.out;
                    record_gemv(s, "attn_wo_partial", o2, wdt, batch, kProNone, kEpiStore);
                    record_tp_reduce(s, "attn_allreduce", blk->tp, tgt, (float*)x.data,
                                     batch * hidden);
                } else {
                    record_gemv(s, "attn_wo_partial", o2, wdt, batch, kProNone, kEpiStore);
                    record_allreduce_f32(s, "attn_allreduce", blk->tp, blk->tp_y,
                                         (float*)x.data, (size_t)batch * hidden);
                }
            } else {
                record_gemv(s, "attn_wo_residual", o2, wdt, batch, kProNone, kEpiResidual);
            }
        } catch (...) {
            s->nodes.resize(before);
            throw;
        }
    });
}

int ab_attention_block_destroy(ab_attention_block* b) {
    return guard([&] {
        if (!b) return;
        b->rt->activate();
        cudaStreamSynchronize(b->rt->stream);
        cudaFree(b->q);
        cudaFree(b->attn_out);
        cudaFree(b->part);
        cudaFree(b->counters);
        if (b->tp_y) cudaFree(b->tp_y);
        free_tc_scratch(&b->tc);
        delete b;
    });
}

// ---- SwiGluBlock ----------------------------------------------------------------------------
int ab_swiglu_block_create(ab_runtime* rt, uint32_t hidden, uint32_t intermediate,
                           uint32_t max_batch, ab_swiglu_block** out) {
    return guard([&] {
        if (!rt || !out) fail(AB_ERR_ARGUMENT, "null argument");
        *out = swiglu_block_new(rt, hidden, intermediate, max_batch, nullptr);
    });
}

int ab_swiglu_block_record(ab_swiglu_block* blk, ab_scheme* s, ab_tensor x,
                           const ab_swiglu_weights* w) {
    return guard([&] {
        if (!blk || !s || !w) fail(AB_ERR_ARGUMENT, "null argument");
        const uint32_t hidden = blk->hidden, inter = blk->inter;
        const uint32_t batch = x_batch(x, hidden, blk->max_batch);
        expect_data("norm", w->norm);
        expect_rank("norm", w->norm, 1);
        expect_float("norm", w->norm);
        expect_dim("norm", w->norm, 0, "hidden", hidden);
        const int32_t wdt = w->gate.dtype;
        if (wdt != AB_F32 && wdt != AB_BF16) expect_float("gate", w->gate);
        expect_linear("gate", w->gate, inter, hidden, wdt);
        expect_linear("up", w->up, inter, hidden, wdt);
        expect_linear("down", w->down, hidden, inter, wdt);
        const void* segs[2] = {w->gate.data, w->up.data};
        if (!gemv_fusable(wdt, hidden, segs, 2) || !gemv_fusable(wdt, inter, &w->down.data, 1))
            invalid("swiglu: hidden and intermediate widths must be multiples of 8 (bf16) or 4 "
                    "(f32) elements with 16-byte aligned weights");

        GemvParams g = {};
        g.seg[0] = w->gate.data;
        g.seg[1] = w->up.data;
        g.seg_rows[0] = inter;
        g.seg_rows[1] = inter;
        g.n_rows = 2 * inter;
        g.units = inter;
        g.K = hidden;
        g.x = x.data;
        g.x_dtype = AB_F32;
        g.x_stride = hidden;
        g.norm_w = w->norm.data;
        g.norm_dtype = w->norm.dtype;
        g.eps = 1e-5f;
        g.out = blk->hb;
        g.out_dtype = wdt;
        g.out_stride = inter;
        attach_tc_scratch(&g, blk->tc);

        GemvParams d = {};
        d.seg[0] = w->down.data;
        d.seg_rows[0] = hidden;
        d.n_rows = hidden;
        d.units = (hidden + 1) / 2;
        d.K = inter;
        d.x = blk->hb;
        d.x_dtype = wdt;
        d.x_stride = inter;
        d.out = x.data;
        d.out_dtype = AB_F32;
        d.out_stride = hidden;
        attach_tc_scratch(&d, blk->tc);

        const size_t before = s->nodes.size();
        try {
            record_gemv(s, "ffn_gate_up_swiglu", g, wdt, batch, kProNorm, kEpiSwiglu);
            if (blk->tp) {
                d.out = blk->tp_y;
                d.addend = comm_rank(blk->tp) == 0 ? (const float*)x.data : nullptr;
                if (comm_has_peers(blk->tp) && batch <= kTpPeerMaxRows) {
                    const TpPush tgt = comm_push_target(blk->tp);
                    d.out = tgt.out;
                    record_gemv(s, "ffn_down_partial", d, wdt, batch, kProNone, kEpiStore);
                    record_tp_reduce(s, "ffn_allreduce", blk->tp, tgt, (float*)x.data,
                                     batch * hidden);
                } else {
                    record_gemv(s, "ffn_down_partial", d, wdt, batch, kProNone, kEpiStore);
                    record_allreduce_f32(s, "ffn_allreduce", blk->tp, blk->tp_y,
                                         (float*)x.data, (size_t)batch * hidden);
                }
            } else {
                record_gemv(s, "ffn_down_residual", d, wdt, batch, kProNone, kEpiResidual);
            }
        } catch (...) {
            s->nodes.resize(before);
            throw;
        }
    });
}

int ab_swiglu_block_destroy(ab_swiglu_block* b) {
    return guard([&] {
        if (!b) return;
        b->rt->activate();
        cudaStreamSynchronize(b->rt->stream);
        cudaFree(b->hb);
        if (b->tp_y) cudaFree(b->tp_y);
        free_tc_scratch(&b->tc);
        delete b;
    });
}

}  // extern "C"
