/*
 * CPU oracle for the Ammon per-token decode layer path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker: the parity tests, the
 * smoke check and the CPU-baseline leg of bench.py load it. Nothing in the
 * product library (ammon_b200/) links, loads or calls it.
 *
 * Every function restates one Ammon kernel or host routine in plain C, in the
 * same arithmetic order where the reference fixes one. Citations are to files
 * of the Ammon crate (src/, tests/). The reference itself cannot be compiled
 * in this environment (its Goldy dependency is an un-vendored path crate and
 * there is no Rust toolchain), so the oracle is pinned against the known-answer
 * values and the fp64 attention oracle that the reference's own test file
 * holds (tests/kernels.rs), not against reference binaries.
 *
 * Places where the reference leaves the order open (Goldy's workgroup_sum /
 * workgroup_max / workgroup_softmax_in_place intrinsics and its cuBLAS-backed
 * matmul) are marked "order unpinned"; the oracle picks one order and tests
 * compare against it within a tolerance.
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off -shared, pthreads).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <pthread.h>
#include <string.h>

#define OR_WORKGROUP 256          /* src/kernels.rs:5 */
#define OR_ATTENTION_SPLIT 8      /* src/kernels.rs:229 */
#define OR_ATTENTION_MAX_HEAD 128 /* src/kernels.rs:231 */

/* ------------------------------------------------------------------------ */
/* Row-parallel helper (pthreads). Work is split into contiguous index       */
/* ranges, so every row keeps its serial summation order.                    */
/* ------------------------------------------------------------------------ */
static int g_threads = 1;

typedef void (*range_fn)(void* ctx, int64_t lo, int64_t hi);
typedef struct {
    range_fn fn;
    void* ctx;
    int64_t lo, hi;
} range_job;

static void* range_main(void* p) {
    range_job* j = (range_job*)p;
    j->fn(j->ctx, j->lo, j->hi);
    return NULL;
}

static void parallel_range(int64_t n, int64_t min_per_thread, range_fn fn, void* ctx) {
    int t = g_threads;
    if (t > 64) t = 64;
    if (t <= 1 || n < 2 * min_per_thread) {
        fn(ctx, 0, n);
        return;
    }
    if ((int64_t)t > n / min_per_thread) t = (int)(n / min_per_thread);
    pthread_t th[64];
    range_job jobs[64] = {{0}};
    int64_t chunk = (n + t - 1) / t;
    int started = 0;
    for (int i = 0; i < t; i++) {
        jobs[i].fn = fn;
        jobs[i].ctx = ctx;
        jobs[i].lo = (int64_t)i * chunk;
        jobs[i].hi = jobs[i].lo + chunk < n ? jobs[i].lo + chunk : n;
        if (jobs[i].lo >= jobs[i].hi) break;
        if (i == 0) continue;
        if (pthread_create(&th[i], NULL, range_main, &jobs[i]) != 0) {
            range_main(&jobs[i]);
            jobs[i].fn = NULL;
        }
        started = i + 1;
    }
    range_main(&jobs[0]);
    for (int i = 1; i < started; i++)
        if (jobs[i].fn) pthread_join(th[i], NULL);
}

/* ------------------------------------------------------------------------ */
/* bf16 helpers (round to nearest even, NaN kept quiet)                      */
/* ------------------------------------------------------------------------ */
static inline float bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline uint16_t f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return (uint16_t)(u >> 16);
}

static inline float round_bf16(float f) { return bf16_to_f32(f32_to_bf16(f)); }

void or_f32_to_bf16(const float* in, uint16_t* out, uint64_t n) {
    for (uint64_t i = 0; i < n; i++) out[i] = f32_to_bf16(in[i]);
}

void or_bf16_to_f32(const uint16_t* in, float* out, uint64_t n) {
    for (uint64_t i = 0; i < n; i++) out[i] = bf16_to_f32(in[i]);
}

/* ------------------------------------------------------------------------ */
/* Seeded synthetic data shared with the GPU initialiser.                    */
/*                                                                          */
/* splitmix64 finaliser (Steele, Lea, Flood 2014) as a stateless hash, and  */
/* an Irwin-Hall sum of twelve 16-bit uniforms as the normal deviate: the   */
/* sum has mean 0 and variance 1 exactly, and every step is integer         */
/* arithmetic followed by one exact scaling and one fused multiply-add, so  */
/* the CPU and the GPU produce bit-identical values.                         */
/* ------------------------------------------------------------------------ */
static inline uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint64_t or_stream_key(uint64_t seed, uint64_t stream) {
    return mix64(seed * 0xD1B54A32D192ED03ull ^ mix64(stream));
}

float or_normal_at(uint64_t key, uint64_t i, float mean, float std) {
    uint32_t s = 0;
    for (int j = 0; j < 3; j++) {
        uint64_t h = mix64(key + 3ull * i + (uint64_t)j);
        s += (uint32_t)(h & 0xffff) + (uint32_t)((h >> 16) & 0xffff) +
             (uint32_t)((h >> 32) & 0xffff) + (uint32_t)(h >> 48);
    }
    float z = (float)((int32_t)(2u * s) - 786420) * (1.0f / 131072.0f);
    return fmaf(std, z, mean);
}

typedef struct {
    void* out;
    uint64_t key;
    float mean, std;
} fill_ctx;

static void fill_f32_range(void* p, int64_t lo, int64_t hi) {
    fill_ctx* c = (fill_ctx*)p;
    for (int64_t i = lo; i < hi; i++)
        ((float*)c->out)[i] = or_normal_at(c->key, (uint64_t)i, c->mean, c->std);
}

static void fill_bf16_range(void* p, int64_t lo, int64_t hi) {
    fill_ctx* c = (fill_ctx*)p;
    for (int64_t i = lo; i < hi; i++)
        ((uint16_t*)c->out)[i] = f32_to_bf16(or_normal_at(c->key, (uint64_t)i, c->mean, c->std));
}

void or_fill_normal_f32(float* out, uint64_t n, uint64_t seed, uint64_t stream, float mean,
                        float std) {
    fill_ctx c = {out, or_stream_key(seed, stream), mean, std};
    parallel_range((int64_t)n, 1 << 16, fill_f32_range, &c);
}

void or_fill_normal_bf16(uint16_t* out, uint64_t n, uint64_t seed, uint64_t stream, float mean,
                         float std) {
    fill_ctx c = {out, or_stream_key(seed, stream), mean, std};
    parallel_range((int64_t)n, 1 << 16, fill_bf16_range, &c);
}

/* Uniform token ids in [lo, hi): one hash per id. */
void or_uniform_tokens(int32_t* out, uint32_t n, uint64_t seed, uint64_t stream, uint32_t lo,
                       uint32_t hi) {
    uint64_t key = or_stream_key(seed, stream);
    for (uint32_t i = 0; i < n; i++) out[i] = (int32_t)(lo + mix64(key + i) % (uint64_t)(hi - lo));
}

/* xorshift32 generator of the reference's tests: tests/kernels.rs:380-390. */
void or_pseudo_random(float* out, uint32_t len, uint32_t seed) {
    uint32_t state = seed * 2654435761u + 1u;
    for (uint32_t i = 0; i < len; i++) {
        state ^= state << 13;
        state ^= state >> 17;
        state ^= state << 5;
        out[i] = (float)(state % 2001u) / 1000.0f - 1.0f;
    }
}

/* ------------------------------------------------------------------------ */
/* Kernels of src/kernels.rs                                                 */
/* ------------------------------------------------------------------------ */

/* embed: src/kernels.rs:35-47. x[i] = embed[token * dim + i]. */
void or_embed(const float* table, uint32_t dim, uint32_t token, float* x) {
    for (uint32_t i = 0; i < dim; i++) x[i] = table[(uint64_t)token * dim + i];
}

/* gemv: src/kernels.rs:49-73. Serial in-order fp32 sum per output row, written at
 * xout[pos * d + i]. */
void or_gemv(const float* x, uint32_t n, const float* w, uint32_t d, float* xout, uint32_t pos) {
    for (uint32_t i = 0; i < d; i++) {
        float sum = 0.0f;
        const float* row = w + (uint64_t)i * n;
        for (uint32_t j = 0; j < n; j++) sum = sum + row[j] * x[j];
        xout[(uint64_t)pos * d + i] = sum;
    }
}

/* Linear / TensorKernels::matmul_into (src/kernels.rs:518-528; call sites
 * src/blocks.rs:220-225,254-255,268-274,305-315). The reference delegates to Goldy's
 * cuBLAS-backed matmul, whose summation order is unpinned; the oracle uses the serial
 * order of the reference's own gemv kernel (src/kernels.rs:67-70). Rows are
 * independent, so the pthread split over rows keeps each row's order. */
typedef struct {
    const void* w;
    uint32_t d_in;
    const float* x;
    float* out;
} matmul_ctx;

static void matmul_f32_range(void* p, int64_t lo, int64_t hi) {
    matmul_ctx* c = (matmul_ctx*)p;
    for (int64_t i = lo; i < hi; i++) {
        float sum = 0.0f;
        const float* row = (const float*)c->w + (uint64_t)i * c->d_in;
        for (uint32_t j = 0; j < c->d_in; j++) sum = sum + row[j] * c->x[j];
        c->out[i] = sum;
    }
}

static void matmul_bf16_range(void* p, int64_t lo, int64_t hi) {
    matmul_ctx* c = (matmul_ctx*)p;
    for (int64_t i = lo; i < hi; i++) {
        float sum = 0.0f;
        const uint16_t* row = (const uint16_t*)c->w + (uint64_t)i * c->d_in;
        for (uint32_t j = 0; j < c->d_in; j++) sum = sum + bf16_to_f32(row[j]) * c->x[j];
        c->out[i] = sum;
    }
}

void or_matmul_f32(const float* w, uint32_t d_out, uint32_t d_in, const float* x, float* out) {
    matmul_ctx c = {w, d_in, x, out};
    parallel_range((int64_t)d_out, 64, matmul_f32_range, &c);
}

/* Same serial order with bf16 weights and activations, fp32 accumulation. */
void or_matmul_bf16(const uint16_t* w, uint32_t d_out, uint32_t d_in, const float* x,
                    float* out) {
    matmul_ctx c = {w, d_in, x, out};
    parallel_range((int64_t)d_out, 64, matmul_bf16_range, &c);
}

/* workgroup_sum of 256 lane values. Goldy's tree order is unpinned; the oracle
 * folds halves (lane l += lane l + s for s = 128, 64, ..., 1). */
static float workgroup_sum256(float* lanes) {
    for (int s = OR_WORKGROUP / 2; s > 0; s >>= 1)
        for (int l = 0; l < s; l++) lanes[l] = lanes[l] + lanes[l + s];
    return lanes[0];
}

/* rmsnorm: src/kernels.rs:75-101. 256 strided partial sums of squares, workgroup_sum,
 * divide by size, add 1e-5, reciprocal square root, then o = w * (ss * x). */
static float rms_scale(const float* x, uint32_t size, float eps) {
    float lanes[OR_WORKGROUP];
    for (uint32_t l = 0; l < OR_WORKGROUP; l++) {
        float ss = 0.0f;
        for (uint32_t j = l; j < size; j += OR_WORKGROUP) {
            float v = x[j];
            ss = ss + v * v;
        }
        lanes[l] = ss;
    }
    float ss = workgroup_sum256(lanes);
    ss = ss / (float)size;
    ss = ss + eps;
    return 1.0f / sqrtf(ss);
}

void or_rmsnorm(const float* x, const float* weight, float* o, uint32_t size) {
    float ss = rms_scale(x, size, 1e-5f);
    for (uint32_t j = 0; j < size; j++) o[j] = weight[j] * (ss * x[j]);
}

/* rmsnorm_inplace: src/kernels.rs:103-128. */
void or_rmsnorm_inplace(float* x, const float* weight, uint32_t size) {
    float ss = rms_scale(x, size, 1e-5f);
    for (uint32_t j = 0; j < size; j++) x[j] = weight[j] * (ss * x[j]);
}

/* RoPE frequency and rotation of one pair: src/kernels.rs:195-199. */
static inline void rope_cs(uint32_t i, uint32_t head_size, uint32_t pos, float theta, float* c,
                           float* s) {
    int32_t head_dim = (int32_t)(i % head_size);
    float freq = 1.0f / powf(theta, (float)head_dim / (float)head_size);
    float val = (float)pos * freq;
    *c = cosf(val);
    *s = sinf(val);
}

/* rope: src/kernels.rs:130-172. Rotates q pairs, and k pairs below kv_dim in place at
 * row `pos` of k. */
void or_rope(float* q, uint32_t q_len, uint32_t head_size, float* k, uint32_t kv_dim,
             uint32_t pos, float theta) {
    uint64_t k_base = (uint64_t)pos * kv_dim;
    for (uint32_t i = 0; i < q_len; i += 2) {
        float fcr, fci;
        rope_cs(i, head_size, pos, theta, &fcr, &fci);
        float v0 = q[i], v1 = q[i + 1];
        q[i] = v0 * fcr - v1 * fci;
        q[i + 1] = v0 * fci + v1 * fcr;
        if (i < kv_dim) {
            v0 = k[k_base + i];
            v1 = k[k_base + i + 1];
            k[k_base + i] = v0 * fcr - v1 * fci;
            k[k_base + i + 1] = v0 * fci + v1 * fcr;
        }
    }
}

/* rope_store: src/kernels.rs:174-210. Rotates q in place and writes RoPE(k_proj) into
 * k[pos * kv_dim ..]. */
void or_rope_store(float* q, uint32_t q_len, uint32_t head_size, const float* k_proj,
                   uint32_t kv_dim, float* k, uint32_t pos, float theta) {
    uint64_t k_base = (uint64_t)pos * kv_dim;
    for (uint32_t i = 0; i < q_len; i += 2) {
        float fcr, fci;
        rope_cs(i, head_size, pos, theta, &fcr, &fci);
        float q0 = q[i], q1 = q[i + 1];
        q[i] = q0 * fcr - q1 * fci;
        q[i + 1] = q0 * fci + q1 * fcr;
        if (i < kv_dim) {
            float k0 = k_proj[i], k1 = k_proj[i + 1];
            k[k_base + i] = k0 * fcr - k1 * fci;
            k[k_base + i + 1] = k0 * fci + k1 * fcr;
        }
    }
}

/* cache_store: src/kernels.rs:212-226. dst[pos * row + i] = src[i]. */
void or_cache_store(const float* src, uint32_t n, float* dst, uint32_t row, uint32_t pos) {
    for (uint32_t i = 0; i < n; i++) dst[(uint64_t)pos * row + i] = src[i];
}

/* K/V element readers so the attention restatements serve fp32 and bf16 caches. */
typedef struct {
    const void* p;
    int bf16;
} kv_ref;

static inline float kv_at(kv_ref r, uint64_t i) {
    return r.bf16 ? bf16_to_f32(((const uint16_t*)r.p)[i]) : ((const float*)r.p)[i];
}

/* attention_partial: src/kernels.rs:228-345, for query head h and split s, in the
 * reference's lane order: 16 lanes per position with lane l summing dims l, l+16, ...,
 * the 16 lane sums added in order, `ways = 128 / head` groups summing positions
 * way, way+ways, ... and folded in way order. */
static void attention_partial_one(const float* q, uint32_t q_heads, uint32_t head, kv_ref key,
                                  kv_ref value, uint32_t kv_heads, float* partial,
                                  uint32_t splits, uint32_t h, uint32_t split, uint32_t pos) {
    uint32_t t0 = split * OR_ATTENTION_SPLIT;
    if (t0 > pos) return;
    uint32_t n = pos + 1 - t0;
    if (n > 8) n = 8;
    uint32_t kv_mul = q_heads / kv_heads;
    uint32_t kv_dim = kv_heads * head;
    uint32_t head_base = (h / kv_mul) * head;
    const float* qs = q + (uint64_t)h * head;
    float scores[8] = {0}, probs[8] = {0};
    for (uint32_t p = 0; p < n; p++) {
        uint64_t k_base = (uint64_t)(t0 + p) * kv_dim + head_base;
        float lanes[16];
        for (uint32_t l = 0; l < 16; l++) {
            float dot = 0.0f;
            for (uint32_t i = l; i < head; i += 16) dot = dot + qs[i] * kv_at(key, k_base + i);
            lanes[l] = dot;
        }
        float sum = 0.0f;
        for (uint32_t l = 0; l < 16; l++) sum = sum + lanes[l];
        scores[p] = sum / sqrtf((float)head);
    }
    float m = scores[0];
    for (uint32_t j = 1; j < n; j++)
        if (scores[j] > m) m = scores[j];
    for (uint32_t j = 0; j < n; j++) probs[j] = expf(scores[j] - m);
    uint32_t ways = 128 / head;
    uint64_t out = ((uint64_t)h * splits + split) * (head + 2);
    for (uint32_t i = 0; i < head; i++) {
        float total = 0.0f;
        for (uint32_t w = 0; w < ways; w++) {
            float acc = 0.0f;
            for (uint32_t j = w; j < n; j += ways)
                acc = acc + probs[j] * kv_at(value, (uint64_t)(t0 + j) * kv_dim + head_base + i);
            total = (w == 0) ? acc : total + acc;
        }
        partial[out + i] = total;
    }
    float l = 0.0f;
    for (uint32_t j = 0; j < n; j++) l = l + probs[j];
    partial[out + head] = m;
    partial[out + head + 1] = l;
}

static void attention_partial_all(const float* q, uint32_t q_heads, uint32_t head, kv_ref key,
                                  kv_ref value, uint32_t kv_heads, float* partial,
                                  uint32_t splits, uint32_t pos) {
    for (uint32_t h = 0; h < q_heads; h++)
        for (uint32_t s = 0; s < splits; s++)
            attention_partial_one(q, q_heads, head, key, value, kv_heads, partial, splits, h, s,
                                  pos);
}

void or_attention_partial(const float* q, uint32_t q_heads, uint32_t head, const float* key,
                          const float* value, uint32_t kv_heads, float* partial, uint32_t splits,
                          uint32_t pos) {
    kv_ref k = {key, 0}, v = {value, 0};
    attention_partial_all(q, q_heads, head, k, v, kv_heads, partial, splits, pos);
}

/* attention_combine: src/kernels.rs:347-410. live = pos / 8 + 1. The max runs over the
 * live splits (order irrelevant); ways = 256 / head groups accumulate splits way,
 * way+ways, ... and the group totals are folded in way order. */
void or_attention_combine(const float* partial, uint32_t q_heads, uint32_t splits,
                          uint32_t head, float* xb, uint32_t pos) {
    uint32_t slot = head + 2;
    uint32_t live = pos / OR_ATTENTION_SPLIT + 1;
    uint32_t ways = 256 / head;
    for (uint32_t h = 0; h < q_heads; h++) {
        uint64_t base = (uint64_t)h * splits * slot;
        float m = partial[base + head];
        for (uint32_t s = 0; s < live; s++) {
            float v = partial[base + (uint64_t)s * slot + head];
            if (v > m) m = v;
        }
        float sums[256] = {0};
        for (uint32_t w = 0; w < ways; w++) {
            float l = 0.0f;
            for (uint32_t j = w; j < live; j += ways) {
                uint64_t o = base + (uint64_t)j * slot;
                float wt = expf(partial[o + head] - m);
                l = l + partial[o + head + 1] * wt;
            }
            sums[w] = l;
        }
        float norm = sums[0];
        for (uint32_t w = 1; w < ways; w++) norm = norm + sums[w];
        for (uint32_t i = 0; i < head; i++) {
            float total = 0.0f;
            for (uint32_t w = 0; w < ways; w++) {
                float acc = 0.0f;
                for (uint32_t j = w; j < live; j += ways) {
                    uint64_t o = base + (uint64_t)j * slot;
                    float wt = expf(partial[o + head] - m);
                    acc = acc + partial[o + i] * wt;
                }
                total = (w == 0) ? acc : total + acc;
            }
            xb[(uint64_t)h * head + i] = total / norm;
        }
    }
}

/* attention (serial): src/kernels.rs:412-460. workgroup_softmax_in_place is a Goldy
 * intrinsic (order unpinned): max, exp(x - max), serial sum, divide. */
void or_attention(const float* q, uint32_t q_heads, uint32_t head, float* att, uint32_t seq,
                  float* xb, const float* key, const float* value, uint32_t kv_heads,
                  uint32_t pos) {
    uint32_t kv_mul = q_heads / kv_heads;
    uint32_t kv_dim = kv_heads * head;
    for (uint32_t h = 0; h < q_heads; h++) {
        uint32_t kv_head = h / kv_mul;
        float* a = att + (uint64_t)h * seq;
        for (uint32_t t = 0; t <= pos; t++) {
            float score = 0.0f;
            uint64_t k_base = (uint64_t)t * kv_dim + kv_head * head;
            for (uint32_t i = 0; i < head; i++)
                score = score + q[(uint64_t)h * head + i] * key[k_base + i];
            a[t] = score / sqrtf((float)head);
        }
        float mx = a[0];
        for (uint32_t t = 1; t <= pos; t++)
            if (a[t] > mx) mx = a[t];
        float sum = 0.0f;
        for (uint32_t t = 0; t <= pos; t++) {
            a[t] = expf(a[t] - mx);
            sum = sum + a[t];
        }
        for (uint32_t t = 0; t <= pos; t++) a[t] = a[t] / sum;
        for (uint32_t i = 0; i < head; i++) {
            float acc = 0.0f;
            for (uint32_t t = 0; t <= pos; t++)
                acc = acc + a[t] * value[(uint64_t)t * kv_dim + kv_head * head + i];
            xb[(uint64_t)h * head + i] = acc;
        }
    }
}

/* swiglu: src/kernels.rs:462-476. hb[i] = hb[i] * (1 / (1 + exp(-hb[i]))) * hb2[i]. */
void or_swiglu(float* hb, const float* hb2, uint32_t n) {
    for (uint32_t i = 0; i < n; i++) {
        float val = hb[i];
        val = val * (1.0f / (1.0f + expf(-val)));
        val = val * hb2[i];
        hb[i] = val;
    }
}

/* TensorKernels::add_into: src/kernels.rs:506-516. */
void or_add(const float* a, const float* b, float* out, uint32_t n) {
    for (uint32_t i = 0; i < n; i++) out[i] = a[i] + b[i];
}

/* fp64 attention oracle of the reference's tests: tests/kernels.rs:400-427. */
void or_cpu_attention_f64(uint32_t q_heads, uint32_t kv_heads, uint32_t head, const float* q,
                          const float* key, const float* value, uint32_t pos, double* out) {
    uint32_t kv_dim = kv_heads * head;
    uint32_t kv_mul = q_heads / kv_heads;
    double* scores = (double*)malloc(sizeof(double) * (pos + 1));
    for (uint32_t h = 0; h < q_heads; h++) {
        uint32_t kv_base = (h / kv_mul) * head;
        double mx = -INFINITY;
        for (uint32_t t = 0; t <= pos; t++) {
            double dot = 0.0;
            for (uint32_t i = 0; i < head; i++)
                dot += (double)q[(uint64_t)h * head + i] *
                       (double)key[(uint64_t)t * kv_dim + kv_base + i];
            scores[t] = dot / sqrt((double)head);
            if (scores[t] > mx) mx = scores[t];
        }
        double total = 0.0;
        for (uint32_t t = 0; t <= pos; t++) {
            scores[t] = exp(scores[t] - mx);
            total += scores[t];
        }
        for (uint32_t i = 0; i < head; i++) {
            double acc = 0.0;
            for (uint32_t t = 0; t <= pos; t++)
                acc += scores[t] * (double)value[(uint64_t)t * kv_dim + kv_base + i];
            out[(uint64_t)h * head + i] = acc / total;
        }
    }
    free(scores);
}

/* sample_argmax: src/tokenizer.rs:179-189. First index of the maximum. */
int32_t or_sample_argmax(const float* logits, uint32_t n) {
    uint32_t max_i = 0;
    float max_p = logits[0];
    for (uint32_t i = 1; i < n; i++)
        if (logits[i] > max_p) {
            max_i = i;
            max_p = logits[i];
        }
    return (int32_t)max_i;
}

/* ------------------------------------------------------------------------ */
/* Llama-shaped decode model composed from the modules, in the op order of  */
/* record_attention (src/blocks.rs:178-259) and record_ffn (:262-278). The   */
/* architecture crate that would assemble it is not part of the reference;   */
/* the composition (embedding, L x [attention, ffn], final RMSNorm,          */
/* classifier) follows the module API of src/modules.rs.                     */
/*                                                                          */
/* bf16 mode (no reference counterpart: the reference is fp32 only) stores   */
/* weights, embeddings and K/V in bf16 and rounds to bf16 every activation   */
/* that feeds a Linear (the normalised x, the attention output and the       */
/* SwiGLU product). Accumulation and the residual stream stay fp32.          */
/* ------------------------------------------------------------------------ */
typedef struct {
    uint32_t dim, layers, heads, kv_heads, head_dim, hidden, vocab, seq;
    float theta, eps;
    int32_t bf16;
} or_config;

typedef struct {
    or_config c;
    /* fp32 mode: float arrays; bf16 mode: uint16 arrays (norm gains always fp32
     * holding bf16-representable values). */
    void* embed;
    void* wcls;
    float* rms_final;
    float** rms_att;
    float** rms_ffn;
    void **wq, **wk, **wv, **wo, **w1, **w2, **w3;
} or_model;

typedef struct {
    float *x, *xb, *xb2, *q, *k, *v, *hb, *hb2, *partial, *logits;
    void *key_cache, *value_cache; /* [layers, seq, kv_heads, head_dim] */
    uint32_t splits;
} or_state;

static void* alloc_w(const or_config* c, uint64_t n) {
    return calloc(n, c->bf16 ? 2 : 4);
}

static void fill_w(const or_config* c, void* p, uint64_t n, uint64_t seed, uint64_t stream,
                   float mean, float std) {
    if (c->bf16)
        or_fill_normal_bf16((uint16_t*)p, n, seed, stream, mean, std);
    else
        or_fill_normal_f32((float*)p, n, seed, stream, mean, std);
}

static void fill_gain(const or_config* c, float* p, uint64_t n, uint64_t seed, uint64_t stream) {
    or_fill_normal_f32(p, n, seed, stream, 1.0f, 0.01f);
    if (c->bf16)
        for (uint64_t i = 0; i < n; i++) p[i] = round_bf16(p[i]);
}

/* Stream ids of the synthetic weights; the GPU initialiser uses the same ids. */
enum {
    OR_STREAM_EMBED = 1,
    OR_STREAM_RMS_FINAL = 2,
    OR_STREAM_WCLS = 3,
    OR_STREAM_LAYER_BASE = 16,
    OR_STREAM_LAYER_STRIDE = 16,
};

or_model* or_model_create(const or_config* c, uint64_t seed, float std) {
    or_model* m = (or_model*)calloc(1, sizeof(or_model));
    m->c = *c;
    uint32_t d = c->dim, L = c->layers, qd = c->heads * c->head_dim,
             kvd = c->kv_heads * c->head_dim, f = c->hidden;
    m->embed = alloc_w(c, (uint64_t)c->vocab * d);
    fill_w(c, m->embed, (uint64_t)c->vocab * d, seed, OR_STREAM_EMBED, 0.0f, std);
    m->wcls = alloc_w(c, (uint64_t)c->vocab * d);
    fill_w(c, m->wcls, (uint64_t)c->vocab * d, seed, OR_STREAM_WCLS, 0.0f, std);
    m->rms_final = (float*)malloc(4ull * d);
    fill_gain(c, m->rms_final, d, seed, OR_STREAM_RMS_FINAL);
    m->rms_att = (float**)calloc(L, sizeof(void*));
    m->rms_ffn = (float**)calloc(L, sizeof(void*));
    void*** all[7] = {&m->wq, &m->wk, &m->wv, &m->wo, &m->w1, &m->w2, &m->w3};
    for (int t = 0; t < 7; t++) *all[t] = (void**)calloc(L, sizeof(void*));
    for (uint32_t l = 0; l < L; l++) {
        uint64_t b = OR_STREAM_LAYER_BASE + (uint64_t)l * OR_STREAM_LAYER_STRIDE;
        m->rms_att[l] = (float*)malloc(4ull * d);
        fill_gain(c, m->rms_att[l], d, seed, b + 0);
        m->wq[l] = alloc_w(c, (uint64_t)qd * d);
        fill_w(c, m->wq[l], (uint64_t)qd * d, seed, b + 1, 0.0f, std);
        m->wk[l] = alloc_w(c, (uint64_t)kvd * d);
        fill_w(c, m->wk[l], (uint64_t)kvd * d, seed, b + 2, 0.0f, std);
        m->wv[l] = alloc_w(c, (uint64_t)kvd * d);
        fill_w(c, m->wv[l], (uint64_t)kvd * d, seed, b + 3, 0.0f, std);
        m->wo[l] = alloc_w(c, (uint64_t)d * qd);
        fill_w(c, m->wo[l], (uint64_t)d * qd, seed, b + 4, 0.0f, std);
        m->rms_ffn[l] = (float*)malloc(4ull * d);
        fill_gain(c, m->rms_ffn[l], d, seed, b + 5);
        m->w1[l] = alloc_w(c, (uint64_t)f * d);
        fill_w(c, m->w1[l], (uint64_t)f * d, seed, b + 6, 0.0f, std);
        m->w2[l] = alloc_w(c, (uint64_t)d * f);
        fill_w(c, m->w2[l], (uint64_t)d * f, seed, b + 7, 0.0f, std);
        m->w3[l] = alloc_w(c, (uint64_t)f * d);
        fill_w(c, m->w3[l], (uint64_t)f * d, seed, b + 8, 0.0f, std);
    }
    return m;
}

void or_model_destroy(or_model* m) {
    if (!m) return;
    for (uint32_t l = 0; l < m->c.layers; l++) {
        free(m->rms_att[l]);
        free(m->rms_ffn[l]);
        free(m->wq[l]);
        free(m->wk[l]);
        free(m->wv[l]);
        free(m->wo[l]);
        free(m->w1[l]);
        free(m->w2[l]);
        free(m->w3[l]);
    }
    free(m->rms_att);
    free(m->rms_ffn);
    free(m->wq);
    free(m->wk);
    free(m->wv);
    free(m->wo);
    free(m->w1);
    free(m->w2);
    free(m->w3);
    free(m->embed);
    free(m->wcls);
    free(m->rms_final);
    free(m);
}

const or_config* or_model_config(const or_model* m) { return &m->c; }

/* Raw pointers to the synthetic weights, for tests that feed the same values to the
 * GPU path. which: 0 embed, 1 wcls, 2 rms_final, 3 rms_att, 4 wq, 5 wk, 6 wv, 7 wo,
 * 8 rms_ffn, 9 w1, 10 w2, 11 w3. */
const void* or_model_weight(const or_model* m, int which, uint32_t layer) {
    switch (which) {
        case 0: return m->embed;
        case 1: return m->wcls;
        case 2: return m->rms_final;
        case 3: return m->rms_att[layer];
        case 4: return m->wq[layer];
        case 5: return m->wk[layer];
        case 6: return m->wv[layer];
        case 7: return m->wo[layer];
        case 8: return m->rms_ffn[layer];
        case 9: return m->w1[layer];
        case 10: return m->w2[layer];
        case 11: return m->w3[layer];
        default: return NULL;
    }
}

or_state* or_state_create(const or_model* m) {
    const or_config* c = &m->c;
    or_state* s = (or_state*)calloc(1, sizeof(or_state));
    uint32_t d = c->dim, qd = c->heads * c->head_dim, kvd = c->kv_heads * c->head_dim;
    uint32_t wide = d > qd ? d : qd;
    s->splits = (c->seq + OR_ATTENTION_SPLIT - 1) / OR_ATTENTION_SPLIT;
    if (s->splits == 0) s->splits = 1;
    s->x = (float*)calloc(d, 4);
    s->xb = (float*)calloc(wide, 4);
    s->xb2 = (float*)calloc(wide, 4);
    s->q = (float*)calloc(qd, 4);
    s->k = (float*)calloc(kvd, 4);
    s->v = (float*)calloc(kvd, 4);
    s->hb = (float*)calloc(c->hidden, 4);
    s->hb2 = (float*)calloc(c->hidden, 4);
    s->partial = (float*)calloc((uint64_t)c->heads * s->splits * (c->head_dim + 2), 4);
    s->logits = (float*)calloc(c->vocab, 4);
    uint64_t cache = (uint64_t)c->layers * c->seq * kvd;
    s->key_cache = calloc(cache, c->bf16 ? 2 : 4);
    s->value_cache = calloc(cache, c->bf16 ? 2 : 4);
    return s;
}

void or_state_destroy(or_state* s) {
    if (!s) return;
    free(s->x);
    free(s->xb);
    free(s->xb2);
    free(s->q);
    free(s->k);
    free(s->v);
    free(s->hb);
    free(s->hb2);
    free(s->partial);
    free(s->logits);
    free(s->key_cache);
    free(s->value_cache);
    free(s);
}

static void linear(const or_config* c, const void* w, uint32_t d_out, uint32_t d_in,
                   const float* x, float* out) {
    if (c->bf16)
        or_matmul_bf16((const uint16_t*)w, d_out, d_in, x, out);
    else
        or_matmul_f32((const float*)w, d_out, d_in, x, out);
}

static void round_vec(const or_config* c, float* v, uint32_t n) {
    if (!c->bf16) return;
    for (uint32_t i = 0; i < n; i++) v[i] = round_bf16(v[i]);
}

static void norm_into(const or_config* c, const float* x, const float* w, float* o) {
    float ss = rms_scale(x, c->dim, c->eps);
    for (uint32_t j = 0; j < c->dim; j++) o[j] = w[j] * (ss * x[j]);
    round_vec(c, o, c->dim);
}

/* One attention block (src/blocks.rs:218-258) for layer l at position pos. */
void or_attention_block(const or_model* m, or_state* s, uint32_t l, uint32_t pos) {
    const or_config* c = &m->c;
    uint32_t d = c->dim, hd = c->head_dim, qd = c->heads * hd, kvd = c->kv_heads * hd;
    uint64_t layer_off = (uint64_t)l * c->seq * kvd;
    norm_into(c, s->x, m->rms_att[l], s->xb);
    linear(c, m->wq[l], qd, d, s->xb, s->q);
    linear(c, m->wk[l], kvd, d, s->xb, s->k);
    linear(c, m->wv[l], kvd, d, s->xb, s->v);
    /* rope_store (src/kernels.rs:174-210) and cache_store (:212-226). */
    uint64_t k_base = (uint64_t)pos * kvd;
    for (uint32_t i = 0; i < qd; i += 2) {
        float fcr, fci;
        rope_cs(i, hd, pos, c->theta, &fcr, &fci);
        float q0 = s->q[i], q1 = s->q[i + 1];
        s->q[i] = q0 * fcr - q1 * fci;
        s->q[i + 1] = q0 * fci + q1 * fcr;
        if (i < kvd) {
            float k0 = s->k[i], k1 = s->k[i + 1];
            float r0 = k0 * fcr - k1 * fci, r1 = k0 * fci + k1 * fcr;
            if (c->bf16) {
                uint16_t* kc = (uint16_t*)s->key_cache + layer_off;
                kc[k_base + i] = f32_to_bf16(r0);
                kc[k_base + i + 1] = f32_to_bf16(r1);
            } else {
                float* kc = (float*)s->key_cache + layer_off;
                kc[k_base + i] = r0;
                kc[k_base + i + 1] = r1;
            }
        }
    }
    for (uint32_t i = 0; i < kvd; i++) {
        if (c->bf16)
            ((uint16_t*)s->value_cache + layer_off)[k_base + i] = f32_to_bf16(s->v[i]);
        else
            ((float*)s->value_cache + layer_off)[k_base + i] = s->v[i];
    }
    /* attention_partial + attention_combine (src/blocks.rs:240-253). */
    kv_ref key = {c->bf16 ? (const void*)((uint16_t*)s->key_cache + layer_off)
                          : (const void*)((float*)s->key_cache + layer_off),
                  c->bf16};
    kv_ref value = {c->bf16 ? (const void*)((uint16_t*)s->value_cache + layer_off)
                            : (const void*)((float*)s->value_cache + layer_off),
                    c->bf16};
    attention_partial_all(s->q, c->heads, hd, key, value, c->kv_heads, s->partial, s->splits,
                          pos);
    or_attention_combine(s->partial, c->heads, s->splits, hd, s->xb, pos);
    round_vec(c, s->xb, qd);
    linear(c, m->wo[l], d, qd, s->xb, s->xb2);
    for (uint32_t i = 0; i < d; i++) s->x[i] = s->x[i] + s->xb2[i];
}

/* One SwiGLU block (src/blocks.rs:262-278). */
void or_ffn_block(const or_model* m, or_state* s, uint32_t l) {
    const or_config* c = &m->c;
    uint32_t d = c->dim, f = c->hidden;
    norm_into(c, s->x, m->rms_ffn[l], s->xb);
    linear(c, m->w1[l], f, d, s->xb, s->hb);
    linear(c, m->w3[l], f, d, s->xb, s->hb2);
    or_swiglu(s->hb, s->hb2, f);
    round_vec(c, s->hb, f);
    linear(c, m->w2[l], d, f, s->hb, s->xb);
    for (uint32_t i = 0; i < d; i++) s->x[i] = s->x[i] + s->xb[i];
}

/* Token embedding row into x (src/kernels.rs:35-47). */
void or_embed_token(const or_model* m, or_state* s, uint32_t token) {
    const or_config* c = &m->c;
    if (c->bf16) {
        const uint16_t* row = (const uint16_t*)m->embed + (uint64_t)token * c->dim;
        for (uint32_t i = 0; i < c->dim; i++) s->x[i] = bf16_to_f32(row[i]);
    } else {
        or_embed((const float*)m->embed, c->dim, token, s->x);
    }
}

/* Final RMSNorm and classifier into s->logits. */
void or_classify(const or_model* m, or_state* s) {
    const or_config* c = &m->c;
    norm_into(c, s->x, m->rms_final, s->xb);
    linear(c, m->wcls, c->vocab, c->dim, s->xb, s->logits);
}

/* AutoregressiveModel::step (src/model.rs:10) for this composition. Returns logits. */
const float* or_model_step(const or_model* m, or_state* s, uint32_t token, uint32_t pos) {
    or_embed_token(m, s, token);
    for (uint32_t l = 0; l < m->c.layers; l++) {
        or_attention_block(m, s, l, pos);
        or_ffn_block(m, s, l);
    }
    or_classify(m, s);
    return s->logits;
}

const float* or_state_tensor(const or_state* s, int which) {
    switch (which) {
        case 0: return s->x;
        case 1: return s->xb;
        case 2: return s->q;
        case 3: return s->logits;
        case 4: return s->hb;
        default: return NULL;
    }
}

const void* or_state_cache(const or_state* s, int value) {
    return value ? s->value_cache : s->key_cache;
}

/* generate_tokens: src/generate.rs:43-91. Forced prompt tokens are emitted too; the
 * loop runs while pos < max_new_tokens - 1 with max_new_tokens clamped to the model's
 * max_seq_len. Returns the number of tokens written to out (at most cap); *margins
 * receives, per greedy step, the gap between the best and second-best logit (or -1
 * for forced steps), so callers can flag near-ties. */
int32_t or_generate_tokens(const or_model* m, or_state* s, const int32_t* prompt,
                           uint32_t prompt_len, uint32_t max_new_tokens, int32_t has_stop,
                           int32_t stop_on, int32_t* out, float* margins, uint32_t cap) {
    if (prompt_len == 0) return -1;
    if (max_new_tokens > m->c.seq) max_new_tokens = m->c.seq;
    uint32_t token = (uint32_t)prompt[0];
    uint32_t pos = 0;
    uint32_t n = 0;
    uint32_t limit = max_new_tokens > 0 ? max_new_tokens - 1 : 0;
    while (pos < limit) {
        const float* logits = or_model_step(m, s, token, pos);
        int32_t next;
        float margin = -1.0f;
        if ((uint64_t)pos < (uint64_t)prompt_len - 1) {
            next = prompt[pos + 1];
        } else {
            next = or_sample_argmax(logits, m->c.vocab);
            float second = -INFINITY;
            for (uint32_t i = 0; i < m->c.vocab; i++)
                if ((int32_t)i != next && logits[i] > second) second = logits[i];
            margin = logits[next] - second;
        }
        pos += 1;
        if (has_stop && stop_on == next) break;
        if (n < cap) {
            out[n] = next;
            if (margins) margins[n] = margin;
        }
        n++;
        token = (uint32_t)next;
    }
    return (int32_t)n;
}

/* Threads used by the row-parallel loops (1 = serial). */
void or_set_threads(int32_t n) { g_threads = n > 0 ? (n > 64 ? 64 : n) : 1; }

int32_t or_get_threads(void) { return g_threads; }
