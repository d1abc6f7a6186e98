// The public kernels of the reference (src/kernels.rs), as standalone sm_100a kernels
// with the reference's parameter contracts. The fused decode path (gemv.cu,
// attention.cu, blocks.cu) does not use the serial ones; they stay available to callers
// and tests exactly as the reference exposes them.
//
// Serial-order kernels (gemv, rmsnorm) use explicitly rounded multiply and add so their
// results are bit-identical to the reference's in-order fp32 arithmetic.
#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace ab {

// ---- embed: src/kernels.rs:35-47 ----------------------------------------------------
// Grid (chunks, batch). 16-byte source vectors when the row is vector-aligned.
template <typename TT, typename XT>
__global__ void embed_kernel(const TT* __restrict__ table, uint32_t vocab, uint32_t dim,
                             const Step* __restrict__ step, XT* __restrict__ x, uint32_t* flags,
                             int vec) {
    pdl_wait();
    pdl_trigger();
    const uint32_t b = blockIdx.y;
    const uint32_t token = step[b].token;
    XT* dst = x + (uint64_t)b * dim;
    const uint32_t tid = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t stride = gridDim.x * blockDim.x;
    if (token >= vocab) {
        if (tid == 0) atomicOr(flags, kFlagTokenRange);
        for (uint32_t i = tid; i < dim; i += stride) dst[i] = from_f32<XT>(0.0f);
        return;
    }
    const TT* src = table + (uint64_t)token * dim;
    constexpr int V = 16 / sizeof(TT);
    if (vec) {
        // 16-byte row vectors in, 16-byte vectors out (two for a bf16 -> f32 gather); four
        // loads per thread in flight before the stores
        const uint32_t nv = dim / V;
        for (uint32_t v0 = tid; v0 < nv; v0 += 4 * stride) {
            uint4 raw[4];
#pragma unroll
            for (int u = 0; u < 4; u++)
                if (v0 + u * stride < nv)
                    raw[u] = *reinterpret_cast<const uint4*>(src + (uint64_t)(v0 + u * stride) * V);
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const uint32_t v = v0 + u * stride;
                if (v >= nv) break;
                if constexpr (sizeof(TT) == sizeof(XT)) {
                    *reinterpret_cast<uint4*>(dst + (uint64_t)v * V) = raw[u];
                } else {
                    const TT* e = reinterpret_cast<const TT*>(&raw[u]);
                    float4* d4 = reinterpret_cast<float4*>(dst + (uint64_t)v * V);
                    d4[0] = make_float4(to_f32(e[0]), to_f32(e[1]), to_f32(e[2]), to_f32(e[3]));
                    d4[1] = make_float4(to_f32(e[4]), to_f32(e[5]), to_f32(e[6]), to_f32(e[7]));
                }
            }
        }
    } else {
        for (uint32_t i = tid; i < dim; i += stride) dst[i] = from_f32<XT>(to_f32(src[i]));
    }
}

// ---- gemv (serial): src/kernels.rs:49-73 --------------------------------------------------
__global__ void gemv_serial_kernel(const float* __restrict__ x, uint32_t n,
                                   const float* __restrict__ w, uint32_t d, float* __restrict__ xout,
                                   uint32_t out_cols, uint32_t seq, const Step* __restrict__ step,
                                   uint32_t* flags) {
    pdl_wait();
    uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= d) return;
    uint32_t pos = step[0].position;
    if (pos >= seq) {
        if (i == 0) atomicOr(flags, kFlagPositionRange);
        return;
    }
    const float* row = w + (uint64_t)i * n;
    float sum = 0.0f;
    for (uint32_t j = 0; j < n; j++) sum = __fadd_rn(sum, __fmul_rn(row[j], x[j]));
    xout[(uint64_t)pos * out_cols + i] = sum;
}

// ---- rmsnorm: src/kernels.rs:75-128 ----------------------------------------------------
// One 256-thread block per row: strided partials per lane (thread t sums elements t,
// t + 256, ... in order), a halving tree in shared memory, then o = w * (ss * x) with
// ss = 1 / sqrt(mean + eps). STAGED rows are first copied into shared memory with 16-byte
// loads (which also makes the in-place form safe), and outputs go out 8 at a time; the
// arithmetic and its order are the same in both forms.
template <typename T>
__device__ __forceinline__ void load8(const T* p, float* v) {
    if constexpr (sizeof(T) == 2) {
        const uint4 r = *reinterpret_cast<const uint4*>(p);
        v[0] = bf16lo(r.x); v[1] = bf16hi(r.x); v[2] = bf16lo(r.y); v[3] = bf16hi(r.y);
        v[4] = bf16lo(r.z); v[5] = bf16hi(r.z); v[6] = bf16lo(r.w); v[7] = bf16hi(r.w);
    } else {
        const float4 a = reinterpret_cast<const float4*>(p)[0];
        const float4 b = reinterpret_cast<const float4*>(p)[1];
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
}
template <typename T>
__device__ __forceinline__ void store8(T* p, const float* v) {
    if constexpr (sizeof(T) == 2) {
        uint4 r;
        __nv_bfloat162 h;
        h = __floats2bfloat162_rn(v[0], v[1]); r.x = *reinterpret_cast<uint32_t*>(&h);
        h = __floats2bfloat162_rn(v[2], v[3]); r.y = *reinterpret_cast<uint32_t*>(&h);
        h = __floats2bfloat162_rn(v[4], v[5]); r.z = *reinterpret_cast<uint32_t*>(&h);
        h = __floats2bfloat162_rn(v[6], v[7]); r.w = *reinterpret_cast<uint32_t*>(&h);
        *reinterpret_cast<uint4*>(p) = r;
    } else {
        reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
        reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
}

template <typename XT, typename WT, typename OT, bool STAGED>
__global__ void __launch_bounds__(256)
    rmsnorm_ref_kernel(const XT* x, const WT* __restrict__ w, OT* o, uint32_t size, float eps) {
    pdl_wait();
    __shared__ float lanes[256];
    extern __shared__ float xs[];  // STAGED: the row as f32
    const uint32_t t = threadIdx.x;
    const XT* xr = x + (uint64_t)blockIdx.x * size;
    OT* orow = o + (uint64_t)blockIdx.x * size;
    if (STAGED) {
        // four 8-element vectors per thread in flight, then into shared memory
        const uint32_t n = size / 8;
        for (uint32_t v0 = t; v0 < n; v0 += 1024) {
            float r[4][8];
#pragma unroll
            for (int u = 0; u < 4; u++)
                if (v0 + u * 256 < n) load8(xr + (uint64_t)(v0 + u * 256) * 8, r[u]);
#pragma unroll
            for (int u = 0; u < 4; u++) {
                if (v0 + u * 256 < n) {
                    float4* d = reinterpret_cast<float4*>(xs + (v0 + u * 256) * 8);
                    d[0] = make_float4(r[u][0], r[u][1], r[u][2], r[u][3]);
                    d[1] = make_float4(r[u][4], r[u][5], r[u][6], r[u][7]);
                }
            }
        }
        __syncthreads();
    }
    float ss = 0.0f;
    for (uint32_t j = t; j < size; j += 256) {
        const float v = STAGED ? xs[j] : to_f32(xr[j]);
        ss = __fadd_rn(ss, __fmul_rn(v, v));
    }
    lanes[t] = ss;
    __syncthreads();
    for (uint32_t s = 128; s > 0; s >>= 1) {
        if (t < s) lanes[t] = __fadd_rn(lanes[t], lanes[t + s]);
        __syncthreads();
    }
    float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(lanes[0], (float)size), eps)));
    if (STAGED) {
#pragma unroll 4
        for (uint32_t v = t; v < size / 8; v += 256) {
            float wv[8], ov[8];
            load8(w + (uint64_t)v * 8, wv);
            const float4 xa = reinterpret_cast<const float4*>(xs + v * 8)[0];
            const float4 xb = reinterpret_cast<const float4*>(xs + v * 8)[1];
            const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
            for (int k = 0; k < 8; k++) ov[k] = __fmul_rn(wv[k], __fmul_rn(scale, xv[k]));
            store8(orow + (uint64_t)v * 8, ov);
        }
    } else {
        for (uint32_t j = t; j < size; j += 256)
            orow[j] = from_f32<OT>(__fmul_rn(to_f32(w[j]), __fmul_rn(scale, to_f32(xr[j]))));
    }
    pdl_trigger();
}

// ---- rope / rope_store: src/kernels.rs:130-210 ----------------------------------------------
__device__ __forceinline__ void rotate(float a, float b, float c, float s, float* r0, float* r1) {
    *r0 = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
    *r1 = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
}

// One block per q row b (one token): row b rotates at step[b].position, and so does row
// step[b].position of k (the row's own cache at k + b * k_stride, or one shared cache with
// k_stride 0). A thread keeps one pair index j across heads when head / 2 divides 256, so
// cos/sin are evaluated once per (row, j) instead of once per element pair.
__global__ void __launch_bounds__(256)
    rope_rows_kernel(float* q, uint32_t q_len, uint32_t head, float* k, uint32_t kv_dim,
                     uint64_t k_stride, uint32_t seq, const Step* __restrict__ step, float theta,
                     uint32_t* flags) {
    pdl_wait();
    const uint32_t b = blockIdx.x;
    const uint32_t pos = step[b].position;
    if (pos >= seq) {
        if (threadIdx.x == 0) atomicOr(flags, kFlagPositionRange);
        return;
    }
    float* qr = q + (uint64_t)b * q_len;
    float* kr = k + (uint64_t)b * k_stride + (uint64_t)pos * kv_dim;
    if (q_len % 4 == 0 && kv_dim % 4 == 0 && ((uintptr_t)qr | (uintptr_t)kr) % 16 == 0) {
        // two pairs per thread through 16-byte accesses
        uint32_t last0 = 0xFFFFFFFFu, last1 = 0xFFFFFFFFu;
        float c0 = 1.0f, s0 = 0.0f, c1 = 1.0f, s1 = 0.0f;
        for (uint32_t i = threadIdx.x * 4; i < q_len; i += 1024) {
            const uint32_t j0 = i % head, j1 = (i + 2) % head;
            if (j0 != last0) {
                rope_cos_sin(j0, head, pos, theta, &c0, &s0);
                last0 = j0;
            }
            if (j1 != last1) {
                rope_cos_sin(j1, head, pos, theta, &c1, &s1);
                last1 = j1;
            }
            float4 v = *reinterpret_cast<float4*>(qr + i);
            rotate(v.x, v.y, c0, s0, &v.x, &v.y);
            rotate(v.z, v.w, c1, s1, &v.z, &v.w);
            *reinterpret_cast<float4*>(qr + i) = v;
            if (i < kv_dim) {
                float4 u = *reinterpret_cast<float4*>(kr + i);
                rotate(u.x, u.y, c0, s0, &u.x, &u.y);
                rotate(u.z, u.w, c1, s1, &u.z, &u.w);
                *reinterpret_cast<float4*>(kr + i) = u;
            }
        }
        pdl_trigger();
        return;
    }
    uint32_t last = 0xFFFFFFFFu;
    float c = 1.0f, s = 0.0f;
    for (uint32_t i = threadIdx.x * 2; i < q_len; i += 512) {
        const uint32_t j = i % head;
        if (j != last) {
            rope_cos_sin(j, head, pos, theta, &c, &s);
            last = j;
        }
        float2 v = *reinterpret_cast<float2*>(qr + i);
        rotate(v.x, v.y, c, s, &v.x, &v.y);
        *reinterpret_cast<float2*>(qr + i) = v;
        if (i < kv_dim) {
            float2 u = *reinterpret_cast<float2*>(kr + i);
            rotate(u.x, u.y, c, s, &u.x, &u.y);
            *reinterpret_cast<float2*>(kr + i) = u;
        }
    }
    pdl_trigger();
}

__global__ void rope_store_ref_kernel(float* q, uint32_t q_len, uint32_t head,
                                      const float* __restrict__ k_proj, uint32_t kv_dim, float* k,
                                      uint32_t seq, const Step* __restrict__ step, float theta,
                                      uint32_t* flags) {
    pdl_wait();
    uint32_t i = (blockIdx.x * blockDim.x + threadIdx.x) * 2;
    if (i >= q_len) return;
    uint32_t pos = step[0].position;
    if (pos >= seq) {
        if (i == 0) atomicOr(flags, kFlagPositionRange);
        return;
    }
    float c, s;
    rope_cos_sin(i, head, pos, theta, &c, &s);
    rotate(q[i], q[i + 1], c, s, &q[i], &q[i + 1]);
    if (i < kv_dim) {
        float* kr = k + (uint64_t)pos * kv_dim;
        rotate(k_proj[i], k_proj[i + 1], c, s, &kr[i], &kr[i + 1]);
    }
}

// ---- cache_store: src/kernels.rs:212-226 ------------------------------------------------
template <typename ST, typename DT>
__global__ void cache_store_kernel(const ST* __restrict__ src, uint32_t n, DT* dst, uint32_t row,
                                   uint32_t seq, const Step* __restrict__ step, uint32_t* flags) {
    pdl_wait();
    uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint32_t pos = step[0].position;
    if (pos >= seq) {
        if (i == 0) atomicOr(flags, kFlagPositionRange);
        return;
    }
    dst[(uint64_t)pos * row + i] = from_f32<DT>(to_f32(src[i]));
}

// ---- attention_partial / attention_combine: src/kernels.rs:228-410 ------------------------
// Partial layout [q_heads, splits, head + 2] and 8-position splits as the reference. One
// 128-thread block per (head, split); each warp scores two positions with a shuffle
// reduction.
template <typename KT>
__global__ void __launch_bounds__(128)
    attention_partial_ref_kernel(const float* __restrict__ q, uint32_t q_heads, uint32_t head,
                                 const KT* __restrict__ key, const KT* __restrict__ value,
                                 uint32_t kv_heads, uint32_t seq, float* partial, uint32_t splits,
                                 const Step* __restrict__ step, uint32_t* flags) {
    pdl_wait();
    __shared__ float qs[128];
    __shared__ float sc[8];
    const uint32_t h = blockIdx.x / splits, split = blockIdx.x % splits;
    const uint32_t pos = step[0].position;
    if (pos >= seq) {
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(flags, kFlagPositionRange);
        return;
    }
    const uint32_t t0 = split * 8;
    if (t0 > pos) return;
    const uint32_t n = min(pos + 1 - t0, 8u);
    const uint32_t kv_mul = q_heads / kv_heads, kv_dim = kv_heads * head;
    const uint32_t base = (h / kv_mul) * head;
    const uint32_t tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    for (uint32_t i = tid; i < head; i += 128) qs[i] = q[(uint64_t)h * head + i];
    __syncthreads();
    const float rs = sqrtf((float)head);
    for (uint32_t p = warp; p < n; p += 4) {
        const KT* kr = key + (uint64_t)(t0 + p) * kv_dim + base;
        float d = 0.0f;
        for (uint32_t i = lane; i < head; i += 32) d += qs[i] * to_f32(kr[i]);
        d = warp_sum(d);
        if (lane == 0) sc[p] = d / rs;
    }
    __syncthreads();
    float m = sc[0];
    for (uint32_t j = 1; j < n; j++) m = fmaxf(m, sc[j]);
    float* out = partial + ((uint64_t)h * splits + split) * (head + 2);
    for (uint32_t i = tid; i < head; i += 128) {
        float acc = 0.0f;
        for (uint32_t j = 0; j < n; j++)
            acc += expf(sc[j] - m) * to_f32(value[(uint64_t)(t0 + j) * kv_dim + base + i]);
        out[i] = acc;
    }
    if (tid == 0) {
        float l = 0.0f;
        for (uint32_t j = 0; j < n; j++) l += expf(sc[j] - m);
        out[head] = m;
        out[head + 1] = l;
    }
    pdl_trigger();
}

// One 256-thread block per head; reads only the live splits (pos / 8 + 1).
template <typename OT>
__global__ void __launch_bounds__(256)
    attention_combine_ref_kernel(const float* __restrict__ partial, uint32_t splits, uint32_t head,
                                 OT* xb, uint32_t seq, const Step* __restrict__ step) {
    pdl_wait();
    extern __shared__ float wts[];  // [splits]
    __shared__ float red[8];
    __shared__ float gmax, gnorm;
    const uint32_t h = blockIdx.x, tid = threadIdx.x;
    const uint32_t pos = min(step[0].position, seq - 1);
    const uint32_t live = pos / 8 + 1;
    const uint32_t slot = head + 2;
    const float* base = partial + (uint64_t)h * splits * slot;
    float m = -INFINITY;
    for (uint32_t s = tid; s < live; s += 256) m = fmaxf(m, base[(uint64_t)s * slot + head]);
    m = warp_max(m);
    if (tid % 32 == 0) red[tid / 32] = m;
    __syncthreads();
    if (tid == 0) {
        float g = red[0];
        for (int w = 1; w < 8; w++) g = fmaxf(g, red[w]);
        gmax = g;
    }
    __syncthreads();
    float l = 0.0f;
    for (uint32_t s = tid; s < live; s += 256) {
        float w = expf(base[(uint64_t)s * slot + head] - gmax);
        wts[s] = w;
        l += w * base[(uint64_t)s * slot + head + 1];
    }
    l = warp_sum(l);
    __syncthreads();
    if (tid % 32 == 0) red[tid / 32] = l;
    __syncthreads();
    if (tid == 0) {
        float g = 0.0f;
        for (int w = 0; w < 8; w++) g += red[w];
        gnorm = g;
    }
    __syncthreads();
    for (uint32_t i = tid; i < head; i += 256) {
        float acc = 0.0f;
        for (uint32_t s = 0; s < live; s++) acc += wts[s] * base[(uint64_t)s * slot + i];
        xb[(uint64_t)h * head + i] = from_f32<OT>(acc / gnorm);
    }
    pdl_trigger();
}

// ---- attention (serial scores): src/kernels.rs:412-460 --------------------------------------
__global__ void __launch_bounds__(256)
    attention_serial_ref_kernel(const float* __restrict__ q, uint32_t q_heads, uint32_t head,
                                float* att, uint32_t seq, float* xb, const float* __restrict__ key,
                                const float* __restrict__ value, uint32_t kv_heads,
                                const Step* __restrict__ step, uint32_t* flags) {
    pdl_wait();
    __shared__ float red[8];
    __shared__ float bval;
    const uint32_t h = blockIdx.x, tid = threadIdx.x;
    const uint32_t pos = step[0].position;
    if (pos >= seq) {
        if (h == 0 && tid == 0) atomicOr(flags, kFlagPositionRange);
        return;
    }
    const uint32_t kv_mul = q_heads / kv_heads, kv_dim = kv_heads * head;
    const uint32_t kvh = h / kv_mul;
    float* a = att + (uint64_t)h * seq;
    const float* qh = q + (uint64_t)h * head;
    const float rs = sqrtf((float)head);
    float mx = -INFINITY;
    for (uint32_t t = tid; t <= pos; t += 256) {
        const float* kr = key + (uint64_t)t * kv_dim + kvh * head;
        float sc = 0.0f;
        for (uint32_t i = 0; i < head; i++) sc += qh[i] * kr[i];
        sc = sc / rs;
        a[t] = sc;
        mx = fmaxf(mx, sc);
    }
    mx = warp_max(mx);
    if (tid % 32 == 0) red[tid / 32] = mx;
    __syncthreads();
    if (tid == 0) {
        float g = red[0];
        for (int w = 1; w < 8; w++) g = fmaxf(g, red[w]);
        bval = g;
    }
    __syncthreads();
    mx = bval;
    float sum = 0.0f;
    for (uint32_t t = tid; t <= pos; t += 256) {
        float e = expf(a[t] - mx);
        a[t] = e;
        sum += e;
    }
    sum = warp_sum(sum);
    __syncthreads();
    if (tid % 32 == 0) red[tid / 32] = sum;
    __syncthreads();
    if (tid == 0) {
        float g = 0.0f;
        for (int w = 0; w < 8; w++) g += red[w];
        bval = g;
    }
    __syncthreads();
    const float inv = 1.0f / bval;
    for (uint32_t t = tid; t <= pos; t += 256) a[t] *= inv;
    __syncthreads();
    for (uint32_t i = tid; i < head; i += 256) {
        float acc = 0.0f;
        for (uint32_t t = 0; t <= pos; t++)
            acc += a[t] * value[(uint64_t)t * kv_dim + kvh * head + i];
        xb[(uint64_t)h * head + i] = acc;
    }
    pdl_trigger();
}

// ---- swiglu: src/kernels.rs:462-476; add: src/kernels.rs:506-516 -----------------------------
template <typename T>
__global__ void swiglu_kernel(T* hb, const T* __restrict__ hb2, uint64_t n) {
    pdl_wait();
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
         i += (uint64_t)gridDim.x * blockDim.x) {
        hb[i] = from_f32<T>(silu_mul(to_f32(hb[i]), to_f32(hb2[i])));
    }
    pdl_trigger();
}

template <typename T>
__global__ void add_kernel(const T* a, const T* b, T* out, uint64_t n) {
    pdl_wait();
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
         i += (uint64_t)gridDim.x * blockDim.x)
        out[i] = from_f32<T>(to_f32(a[i]) + to_f32(b[i]));
    pdl_trigger();
}

static unsigned blocks_for(uint64_t n, unsigned per, const Runtime* rt) {
    uint64_t b = (n + per - 1) / per;
    uint64_t cap = rt ? (uint64_t)rt->sm_count * 32 : 4096;
    return (unsigned)std::max<uint64_t>(1, std::min(b, cap));
}

static uint32_t* flags_of(ab_scheme* s) { return s->rt ? s->rt->flags : nullptr; }

// Shared by Embedding::record and the kernel entry point.
void record_embed(ab_scheme* s, ab_tensor table, ab_tensor step, ab_tensor x) {
    expect_data("table", table);
    expect_data("x", x);
    expect_rank("table", table, 2);
    expect_float("table", table);
    expect_float("x", x);
    expect_rank_in("x", x, 1, 2);
    const uint32_t vocab = table.dims[0], dim = table.dims[1];
    const uint32_t batch = x.rank == 2 ? x.dims[0] : 1;
    expect_dim("x", x, x.rank - 1, "dim", dim);
    expect_step(step, batch);
    if (table.dtype == AB_F32 && x.dtype == AB_BF16)
        invalid("parameter `x`: an f32 table gathers into an f32 x");
    const size_t esz = dtype_size(table.dtype);
    const int vec = (dim % (16 / esz) == 0) && ((uintptr_t)table.data % 16 == 0) &&
                    ((uintptr_t)x.data % 16 == 0);
    uint32_t* flags = flags_of(s);
    const Step* st = (const Step*)step.data;
    // each thread moves up to four 16-byte vectors of its row
    const unsigned chunks = std::max(1u, std::min(64u, (dim / (unsigned)(16 / esz) + 1023) / 1024));
    dim3 grid(chunks, batch);
    if (table.dtype == AB_F32) {
        const float* tb = (const float*)table.data;
        float* xo = (float*)x.data;
        s->add("embed", [=](cudaStream_t st_) {
            return launch(st_, grid, dim3(256), 0, true, embed_kernel<float, float>, tb, vocab, dim,
                          st, xo, flags, vec);
        });
    } else if (x.dtype == AB_F32) {
        const bf16* tb = (const bf16*)table.data;
        float* xo = (float*)x.data;
        s->add("embed", [=](cudaStream_t st_) {
            return launch(st_, grid, dim3(256), 0, true, embed_kernel<bf16, float>, tb, vocab, dim,
                          st, xo, flags, vec);
        });
    } else {
        const bf16* tb = (const bf16*)table.data;
        bf16* xo = (bf16*)x.data;
        s->add("embed", [=](cudaStream_t st_) {
            return launch(st_, grid, dim3(256), 0, true, embed_kernel<bf16, bf16>, tb, vocab, dim,
                          st, xo, flags, vec);
        });
    }
}

// Shared by RmsNorm::record[_inplace] and the kernel entry points. x [dim] or [rows, dim].
void record_rmsnorm_ref(ab_scheme* s, ab_tensor x, ab_tensor weight, ab_tensor o, float eps) {
    expect_data("x", x);
    expect_data("weight", weight);
    expect_data("o", o);
    expect_float("x", x);
    expect_float("weight", weight);
    expect_float("o", o);
    expect_rank_in("x", x, 1, 2);
    expect_rank("weight", weight, 1);
    const uint32_t dim = x.dims[x.rank - 1];
    const uint32_t rows = x.rank == 2 ? x.dims[0] : 1;
    expect_dim("weight", weight, 0, "dim", dim);
    if (numel(o) != numel(x))
        invalid("parameter `o`: dim `dim` must match x " + shape_str(x) + ", got " + shape_str(o));
    if (o.data == x.data && o.dtype != x.dtype)
        invalid("parameter `o`: an in-place norm keeps x's dtype");
    auto go = [&](auto xtag, auto wtag, auto otag) {
        using X = decltype(xtag);
        using W = decltype(wtag);
        using O = decltype(otag);
        const X* xp = (const X*)x.data;
        const W* wp = (const W*)weight.data;
        O* op = (O*)o.data;
        // rows of 8-element vectors on 16-byte boundaries are staged in shared memory
        const bool staged = dim % 8 == 0 && (size_t)dim * 4 <= 160 * 1024 &&
                            (uintptr_t)xp % 16 == 0 && (uintptr_t)wp % 16 == 0 &&
                            (uintptr_t)op % 16 == 0;
        if (staged) {
            auto kern = rmsnorm_ref_kernel<X, W, O, true>;
            const size_t smem = (size_t)dim * 4;
            s->add("rmsnorm", [=](cudaStream_t st) {
                if (smem > 48 * 1024) {
                    cudaError_t e = cudaFuncSetAttribute(
                        kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
                    if (e != cudaSuccess) return e;
                }
                return launch(st, dim3(rows), dim3(256), smem, true, kern, xp, wp, op, dim, eps);
            });
        } else {
            s->add("rmsnorm", [=](cudaStream_t st) {
                return launch(st, dim3(rows), dim3(256), 0, true,
                              rmsnorm_ref_kernel<X, W, O, false>, xp, wp, op, dim, eps);
            });
        }
    };
    auto by_w_o = [&](auto xtag) {
        if (weight.dtype == AB_F32 && o.dtype == AB_F32) go(xtag, float(), float());
        else if (weight.dtype == AB_F32) go(xtag, float(), bf16());
        else if (o.dtype == AB_F32) go(xtag, bf16(), float());
        else go(xtag, bf16(), bf16());
    };
    if (x.dtype == AB_F32) by_w_o(float());
    else by_w_o(bf16());
}

}  // namespace ab

using namespace ab;

extern "C" {

int ab_kernel_embed(ab_scheme* s, ab_tensor table, ab_tensor step, ab_tensor x) {
    return guard([&] {
        if (!s) fail(AB_ERR_ARGUMENT, "null scheme");
        record_embed(s, table, step, x);
    });
}

int ab_kernel_gemv(ab_scheme* s, ab_tensor x, ab_tensor w, ab_tensor xout, ab_tensor step) {
    return guard([&] {
        if (!s) fail(AB_ERR_ARGUMENT, "null scheme");
        expect_data("x", x);
        expect_data("w", w);
        expect_data("xout", xout);
        expect_rank("x", x, 1);
        expect_rank("w", w, 2);
        expect_rank("xout", xout, 2);
        expect_dtype("x", x, AB_F32);
        expect_dtype("w", w, AB_F32);
        expect_dtype("xout", xout, AB_F32);
        const uint32_t n = x.dims[0], d = w.dims[0];
        expect_dim("w", w, 1, "n", n);
        if (xout.dims[1] < d) expect_dim("xout", xout, 1, "d", d);
        expect_step(step, 1);
        const float *xp = (const float*)x.data, *wp = (const float*)w.data;
        float* op = (float*)xout.data;
        const uint32_t cols = xout.dims[1], seq = xout.dims[0];
        const Step* st = (const Step*)step.data;
        uint32_t* flags = flags_of(s);
        s->add("gemv", [=](cudaStream_t stream) {
            return launch(stream, dim3((d + 255) / 256), dim3(256), 0, true, gemv_serial_kernel, xp,
                          n, wp, d, op, cols, seq, st, flags);
        });
    });
}

int ab_kernel_rmsnorm(ab_scheme* s, ab_tensor x, ab_tensor weight, ab_tensor o) {
    return guard([&] {
        if (!s) fail(AB_ERR_ARGUMENT, "null scheme");
        record_rmsnorm_ref(s, x, weight, o, 1e-5f);
    });
}

int ab_kernel_rmsnorm_inplace(ab_scheme* s, ab_tensor x, ab_tensor weight) {
    return guard([&] {
        if (!s) fail(AB_ERR_ARGUMENT, "null scheme");
        record_rmsnorm_ref(s, x, weight, x, 1e-5f);
    });
}

static void check_rope_shapes(ab_tensor q, ab_tensor k, const char* kname) {
    expect_data("q", q);
    expect_data(kname, k);
    expect_rank("q", q, 2);
    expect_rank(kname, k, 3);
    expect_dtype("q", q, AB_F32);
    expect_dtype(kname, k, AB_F32);
    expect_dim(kname, k, 2, "head", q.dims[1]);
    if (q.dims[1] % 2) invalid("parameter `q`: dim `head` must be even");
}

int ab_kernel_rope(ab_scheme* s, ab_tensor q, ab_tensor k, ab_tensor step, float theta) {
    return guard([&] {
        if (!s) fail(AB_ERR_ARGUMENT, "null scheme");
        // q [heads, head] (one token) or [batch, heads, head] (one DecodeStep per row); k
        // [seq, kv_heads, head] shared by the rows or [>= batch, seq, kv_heads, head]
        expect_data("q", q);
        expect_data("k", k);
        expect_rank_in("q", q, 2, 3);
        expect_rank_in("k", k, 3, 4);
        expect_dtype("q", q, AB_F32);
        expect_dtype("k", k, AB_F32);
        const uint32_t batch = q.rank == 3 ? q.dims[0] : 1;
        const uint32_t head = q.dims[q.rank - 1];
        const int o = k.rank - 3;
        expect_dim("k", k, o + 2, "head", head);
        if (head % 2) invalid("parameter `q`: dim `head` must be even");
        if (k.rank == 4 && k.dims[0] < batch) expect_dim("k", k, 0, "batch", batch);
        expect_step(step, batch);
        const uint32_t q_len = (uint32_t)(numel(q) / batch);
        const uint32_t kv_dim = k.dims[o + 1] * k.dims[o + 2], seq = k.dims[o];
        const uint64_t k_stride = k.rank == 4 ? (uint64_t)seq * kv_dim : 0;
        float *qp = (float*)q.data, *kp = (float*)k.data;
        const Step* st = (const Step*)step.data;
        uint32_t* flags = flags_of(s);
        s->add("rope", [=](cudaStream_t stream) {
            return launch(stream, dim3(batch), dim3(256), 0, true, rope_rows_kernel, qp, q_len,
                          head, kp, kv_dim, k_stride, seq, st, theta, flags);
        });
    });
}

int ab_kernel_rope_store(ab_scheme* s, ab_tensor q, ab_tensor k_proj, ab_tensor k, ab_tensor step,
                         float theta) {
    return guard([&] {
        if (!s) fail(AB_ERR_ARGUMENT, "null scheme");
        check_rope_shapes(q, k, "k");
        expect_data("k_proj", k_proj);
        expect_rank("k_proj", k_proj, 1);
        expect_dtype("k_proj", k_proj, AB_F32);
        const uint32_t kv_dim = k_proj.dims[0];
        if (k.dims[1] * k.dims[2] != kv_dim)
            invalid("parameter `k`: dim `kv_dim` (kv_heads * head) must be " +
                    std::to_string(kv_dim) + ", got " + shape_str(k));
        if (kv_dim > numel(q) || kv_dim % 2)
            invalid("parameter `k_proj`: kv width must be even and no wider than q");
        expect_step(step, 1);
        const uint32_t q_len = (uint32_t)numel(q), head = q.dims[1], seq = k.dims[0];
        float *qp = (float*)q.data, *kp = (float*)k.data;
        const float* kpj = (const float*)k_proj.data;
        const Step* st = (const Step*)step.data;
        uint32_t* flags = flags_of(s);
        const unsigned grid = (q_len / 2 + 255) / 256;
        s->add("rope_store", [=](cudaStream_t stream) {
            return launch(stream, dim3(std::max(1u, grid)), dim3(256), 0, true,
                          rope_store_ref_kernel, qp, q_len, head, kpj, kv_dim, kp, seq, st, theta,
                          flags);
        });
    });
}

int ab_kernel_cache_store(ab_scheme* s, ab_tensor src, ab_tensor dst, ab_tensor step) {
    return guard([&] {
        if (!s) fail(AB_ERR_ARGUMENT, "null scheme");
        expect_data("src", src);
        expect_data("dst", dst);
        expect_rank("src", src, 1);
        expect_rank("dst", dst, 3);
        expect_float("src", src);
        expect_float("dst", dst);
        const uint32_t n = src.dims[0], row = dst.dims[1] * dst.dims[2], seq = dst.dims[0];
        if (n > row)
            invalid("parameter `src`: dim `kv_dim` " + std::to_string(n) + " exceeds cache row " +
                    std::to_string(row));
        expect_step(step, 1);
        const Step* st = (const Step*)step.data;
        uint32_t* flags = flags_of(s);
        const unsigned grid = std::max(1u, (n + 255) / 256);
        auto go = [&](auto stag, auto dtag) {
            using S = decltype(stag);
            using D = decltype(dtag);
            const S* sp = (const S*)src.data;
            D* dp = (D*)dst.data;
            s->add("cache_store", [=](cudaStream_t stream) {
                return launch(stream, dim3(grid), dim3(256), 0, true, cache_store_kernel<S, D>, sp,
                              n, dp, row, seq, st, flags);
            });
        };
        if (src.dtype == AB_F32 && dst.dtype == AB_F32) go(float(), float());
        else if (src.dtype == AB_F32) go(float(), bf16());
        else if (dst.dtype == AB_F32) go(bf16(), float());
        else go(bf16(), bf16());
    });
}

int ab_kernel_attention_partial(ab_scheme* s, ab_tensor q, ab_tensor key_cache,
                                ab_tensor value_cache, ab_tensor partial, ab_tensor step) {
    return guard([&] {
        if (!s) fail(AB_ERR_ARGUMENT, "null scheme");
        expect_data("q", q);
        expect_data("key_cache", key_cache);
        expect_data("value_cache", value_cache);
        expect_data("partial", partial);
        expect_rank("q", q, 2);
        expect_rank("key_cache", key_cache, 3);
        expect_rank("value_cache", value_cache, 3);
        expect_rank("partial", partial, 3);
        expect_dtype("q", q, AB_F32);
        expect_dtype("partial", partial, AB_F32);
        expect_float("key_cache", key_cache);
        expect_dtype("value_cache", value_cache, key_cache.dtype);
        const uint32_t q_heads = q.dims[0], head = q.dims[1];
        const uint32_t seq = key_cache.dims[0], kv_heads = key_cache.dims[1];
        expect_dim("key_cache", key_cache, 2, "head", head);
        for (int a = 0; a < 3; a++)
            expect_dim("value_cache", value_cache, a, a == 0 ? "seq" : a == 1 ? "kv_heads" : "head",
                       key_cache.dims[a]);
        if (head > 128) invalid("attention: head size " + std::to_string(head) + " exceeds 128");
        if (kv_heads == 0 || q_heads % kv_heads)
            invalid("parameter `key_cache`: kv_heads must divide q_heads");
        expect_dim("partial", partial, 0, "q_heads", q_heads);
        expect_dim("partial", partial, 2, "slot", head + 2);
        const uint32_t splits = partial.dims[1];
        if (splits < (seq + 7) / 8)
            invalid("parameter `partial`: dim `splits` must cover seq / 8 = " +
                    std::to_string((seq + 7) / 8));
        expect_step(step, 1);
        const float* qp = (const float*)q.data;
        float* pp = (float*)partial.data;
        const Step* st = (const Step*)step.data;
        uint32_t* flags = flags_of(s);
        auto go = [&](auto tag) {
            using T = decltype(tag);
            const T* kp = (const T*)key_cache.data;
            const T* vp = (const T*)value_cache.data;
            s->add("attn_partial", [=](cudaStream_t stream) {
                return launch(stream, dim3(q_heads * splits), dim3(128), 0, true,
                              attention_partial_ref_kernel<T>, qp, q_heads, head, kp, vp, kv_heads,
                              seq, pp, splits, st, flags);
            });
        };
        if (key_cache.dtype == AB_F32) go(float());
        else go(bf16());
    });
}

int ab_kernel_attention_combine(ab_scheme* s, ab_tensor partial, ab_tensor xb, ab_tensor step) {
    return guard([&] {
        if (!s) fail(AB_ERR_ARGUMENT, "null scheme");
        expect_data("partial", partial);
        expect_data("xb", xb);
        expect_rank("partial", partial, 3);
        expect_rank("xb", xb, 2);
        expect_dtype("partial", partial, AB_F32);
        expect_float("xb", xb);
        const uint32_t q_heads = partial.dims[0], splits = partial.dims[1];
        const uint32_t head = xb.dims[1];
        expect_dim("xb", xb, 0, "q_heads", q_heads);
        expect_dim("partial", partial, 2, "slot", head + 2);
        if (head > 256) invalid("attention: head size exceeds 256");
        expect_step(step, 1);
        const float* pp = (const float*)partial.data;
        const Step* st = (const Step*)step.data;
        const uint32_t seq = splits * 8;
        const size_t smem = (size_t)splits * 4;
        if (smem > 200 * 1024) invalid("parameter `partial`: too many splits");
        auto go = [&](auto tag) {
            using O = decltype(tag);
            O* op = (O*)xb.data;
            s->add("attn_combine", [=](cudaStream_t stream) {
                if (smem > 48 * 1024) {
                    cudaError_t e = cudaFuncSetAttribute(attention_combine_ref_kernel<O>,
                                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                         (int)smem);
                    if (e != cudaSuccess) return e;
                }
                return launch(stream, dim3(q_heads), dim3(256), smem, true,
                              attention_combine_ref_kernel<O>, pp, splits, head, op, seq, st);
            });
        };
        if (xb.dtype == AB_F32) go(float());
        else go(bf16());
    });
}

int ab_kernel_attention(ab_scheme* s, ab_tensor q, ab_tensor att, ab_tensor xb, ab_tensor key_cache,
                        ab_tensor value_cache, ab_tensor step) {
    return guard([&] {
        if (!s) fail(AB_ERR_ARGUMENT, "null scheme");
        expect_data("q", q);
        expect_data("att", att);
        expect_data("xb", xb);
        expect_data("key_cache", key_cache);
        expect_data("value_cache", value_cache);
        expect_rank("q", q, 2);
        expect_rank("att", att, 2);
        expect_rank("xb", xb, 2);
        expect_rank("key_cache", key_cache, 3);
        expect_rank("value_cache", value_cache, 3);
        for (auto* p : {&q, &att, &xb, &key_cache, &value_cache}) (void)p;
        expect_dtype("q", q, AB_F32);
        expect_dtype("att", att, AB_F32);
        expect_dtype("xb", xb, AB_F32);
        expect_dtype("key_cache", key_cache, AB_F32);
        expect_dtype("value_cache", value_cache, AB_F32);
        const uint32_t q_heads = q.dims[0], head = q.dims[1];
        const uint32_t seq = key_cache.dims[0], kv_heads = key_cache.dims[1];
        expect_dim("att", att, 0, "q_heads", q_heads);
        expect_dim("att", att, 1, "seq", seq);
        expect_dim("xb", xb, 0, "q_heads", q_heads);
        expect_dim("xb", xb, 1, "head", head);
        expect_dim("key_cache", key_cache, 2, "head", head);
        for (int a = 0; a < 3; a++)
            expect_dim("value_cache", value_cache, a, a == 0 ? "seq" : a == 1 ? "kv_heads" : "head",
                       key_cache.dims[a]);
        if (kv_heads == 0 || q_heads % kv_heads)
            invalid("parameter `key_cache`: kv_heads must divide q_heads");
        expect_step(step, 1);
        const float* qp = (const float*)q.data;
        float* ap = (float*)att.data;
        float* xp = (float*)xb.data;
        const float* kp = (const float*)key_cache.data;
        const float* vp = (const float*)value_cache.data;
        const Step* st = (const Step*)step.data;
        uint32_t* flags = flags_of(s);
        s->add("attn_serial", [=](cudaStream_t stream) {
            return launch(stream, dim3(q_heads), dim3(256), 0, true, attention_serial_ref_kernel, qp,
                          q_heads, head, ap, seq, xp, kp, vp, kv_heads, st, flags);
        });
    });
}

int ab_kernel_swiglu(ab_scheme* s, ab_tensor hb, ab_tensor hb2) {
    return guard([&] {
        if (!s) fail(AB_ERR_ARGUMENT, "null scheme");
        expect_data("hb", hb);
        expect_data("hb2", hb2);
        expect_float("hb", hb);
        expect_dtype("hb2", hb2, hb.dtype);
        if (numel(hb) != numel(hb2))
            invalid("parameter `hb2`: dim `hidden` must match hb " + shape_str(hb));
        const uint64_t n = numel(hb);
        const unsigned grid = blocks_for(n, 256, s->rt);
        auto go = [&](auto tag) {
            using T = decltype(tag);
            T* a = (T*)hb.data;
            const T* b = (const T*)hb2.data;
            s->add("swiglu", [=](cudaStream_t stream) {
                return launch(stream, dim3(grid), dim3(256), 0, true, swiglu_kernel<T>, a, b, n);
            });
        };
        if (hb.dtype == AB_F32) go(float());
        else go(bf16());
    });
}

int ab_tensor_add_into(ab_scheme* s, ab_tensor a, ab_tensor b, ab_tensor out) {
    return guard([&] {
        if (!s) fail(AB_ERR_ARGUMENT, "null scheme");
        expect_data("a", a);
        expect_data("b", b);
        expect_data("out", out);
        expect_float("a", a);
        expect_dtype("b", b, a.dtype);
        expect_dtype("out", out, a.dtype);
        if (numel(a) != numel(b) || numel(a) != numel(out))
            invalid("add: element counts differ: " + shape_str(a) + ", " + shape_str(b) + ", " +
                    shape_str(out));
        const uint64_t n = numel(a);
        const unsigned grid = blocks_for(n, 256, s->rt);
        auto go = [&](auto tag) {
            using T = decltype(tag);
            const T* ap = (const T*)a.data;
            const T* bp = (const T*)b.data;
            T* op = (T*)out.data;
            s->add("add", [=](cudaStream_t stream) {
                return launch(stream, dim3(grid), dim3(256), 0, true, add_kernel<T>, ap, bp, op, n);
            });
        };
        if (a.dtype == AB_F32) go(float());
        else go(bf16());
    });
}

}  // extern "C"
