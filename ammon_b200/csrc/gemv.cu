// Bandwidth-bound GEMV for the decode path (Linear at batch <= 4, and the fused block
// projections), replacing Goldy's cuBLAS-backed matmul_into (src/kernels.rs:518-528).
//
// Design (B200):
//  - Each CTA owns a contiguous, balanced range of output row pairs ("units"). Its work
//    is the linear sequence (unit, 512-byte chunk) and the 8 warps split that sequence
//    evenly, so no warp idles at the end whatever K and the row count are. Partial sums
//    land in per-(unit, warp) shared-memory slots and are folded in warp order, so the
//    result is deterministic.
//  - Weights stream through 16-byte non-coherent loads that do not allocate in L1, four
//    chunks of two rows in flight per lane.
//  - Programmatic dependent launch: before waiting on the previous kernel, each warp
//    prefetches the first chunks of its weight rows into L2, so weight streaming starts
//    while the previous kernel drains. Activations are read only after the wait.
//  - Activations are staged once per CTA in shared memory (with the RMSNorm prologue
//    applied: src/kernels.rs:75-101 order o = w * (ss * x)).
//  - Epilogues fuse what the reference runs as separate dispatches: RoPE + K/V cache
//    append (src/kernels.rs:174-226), SwiGLU (src/kernels.rs:462-476) and the residual
//    add (src/kernels.rs:506-516).
#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "internal.h"
#include "ops.h"

namespace ab {

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kGemvUnroll = 4;

template <typename WT>
struct VecTraits;
template <>
struct VecTraits<float> {
    static constexpr int V = 4;
};
template <>
struct VecTraits<bf16> {
    static constexpr int V = 8;
};

// dot of one 16-byte weight vector with one 16-byte activation vector
__device__ __forceinline__ float dot16(const uint4& w, const uint4& x, float acc, float) {
    acc = fmaf(__uint_as_float(w.x), __uint_as_float(x.x), acc);
    acc = fmaf(__uint_as_float(w.y), __uint_as_float(x.y), acc);
    acc = fmaf(__uint_as_float(w.z), __uint_as_float(x.z), acc);
    acc = fmaf(__uint_as_float(w.w), __uint_as_float(x.w), acc);
    return acc;
}
__device__ __forceinline__ float dot16(const uint4& w, const uint4& x, float acc, bf16) {
    acc = fmaf(bf16lo(w.x), bf16lo(x.x), acc);
    acc = fmaf(bf16hi(w.x), bf16hi(x.x), acc);
    acc = fmaf(bf16lo(w.y), bf16lo(x.y), acc);
    acc = fmaf(bf16hi(w.y), bf16hi(x.y), acc);
    acc = fmaf(bf16lo(w.z), bf16lo(x.z), acc);
    acc = fmaf(bf16hi(w.z), bf16hi(x.z), acc);
    acc = fmaf(bf16lo(w.w), bf16lo(x.w), acc);
    acc = fmaf(bf16hi(w.w), bf16hi(x.w), acc);
    return acc;
}

__device__ __forceinline__ float load_elem(const void* p, int32_t dt, uint64_t i) {
    return dt == AB_F32 ? ((const float*)p)[i] : __bfloat162float(((const bf16*)p)[i]);
}

__device__ __forceinline__ void store_elem(void* p, int32_t dt, uint64_t i, float v) {
    if (dt == AB_F32)
        ((float*)p)[i] = v;
    else
        ((bf16*)p)[i] = __float2bfloat16_rn(v);
}

// Row pointers of unit u (pair of virtual rows).
template <typename WT, int EPI>
__device__ __forceinline__ void unit_rows(const GemvParams& p, uint32_t u, const WT** r0,
                                          const WT** r1) {
    const uint64_t K = p.K;
    if (EPI == kEpiSwiglu) {
        *r0 = (const WT*)p.seg[0] + (uint64_t)u * K;
        *r1 = (const WT*)p.seg[1] + (uint64_t)u * K;
        return;
    }
    uint32_t v = 2 * u;
    int s = 0;
    if (v >= p.seg_rows[0]) {
        v -= p.seg_rows[0];
        s = 1;
        if (v >= p.seg_rows[1]) {
            v -= p.seg_rows[1];
            s = 2;
        }
    }
    const WT* base = (const WT*)p.seg[s];
    *r0 = base + (uint64_t)v * K;
    *r1 = (v + 1 < p.seg_rows[s]) ? *r0 + K : *r0;
}

template <typename WT, int NB, int PRO, int EPI>
__global__ void __launch_bounds__(kGemvThreads, 4) gemv_kernel(const GemvParams p) {
    using XS = WT;
    constexpr int V = VecTraits<WT>::V;
    constexpr int CH = 32 * V;  // elements per warp chunk (512 bytes)
    extern __shared__ __align__(16) unsigned char smem[];
    const uint32_t Kpad = p.nchunks * CH;
    XS* xs = reinterpret_cast<XS*>(smem);
    float* part = reinterpret_cast<float*>(smem + (size_t)NB * Kpad * sizeof(XS));
    __shared__ float red[kGemvWarps][NB];

    const uint32_t tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    const uint32_t u0 = (uint32_t)((uint64_t)blockIdx.x * p.units / gridDim.x);
    const uint32_t u1 = (uint32_t)((uint64_t)(blockIdx.x + 1) * p.units / gridDim.x);
    const uint32_t ucta = u1 - u0;
    const uint32_t nc = p.nchunks;
    const uint32_t T = ucta * nc;
    const uint32_t wa = (uint32_t)((uint64_t)warp * T / kGemvWarps);
    const uint32_t wb = (uint32_t)((uint64_t)(warp + 1) * T / kGemvWarps);

    // 1. Weights do not depend on the previous kernel: prefetch this warp's first chunks
    //    (both rows) into L2 while the predecessor finishes.
    if (wa < wb) {
        const uint32_t ul = wa / nc, c = wa - ul * nc;
        const WT *r0, *r1;
        unit_rows<WT, EPI>(p, u0 + ul, &r0, &r1);
        const uint32_t avail = min(nc - c, p.prefetch_chunks);
        const uint64_t e0 = (uint64_t)c * CH;
        const uint64_t bytes = min((uint64_t)avail * CH, (uint64_t)p.K - e0) * sizeof(WT);
        // lane 0 prefetches row 0's span, lane 1 row 1's
        if (lane < 2 && avail > 0 && bytes >= 16) {
            const WT* r = lane == 0 ? r0 : r1;
            prefetch_l2_bulk(r + e0, (uint32_t)(bytes & ~15ull));
        }
    }

    // 2. Activations depend on the previous kernel.
    pdl_wait();

    // 3. Stage activations [NB][Kpad] in shared memory, zero padded.
    float scale[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) scale[b] = 1.0f;
    if (PRO == kProNorm) {
        float ss[NB];
#pragma unroll
        for (int b = 0; b < NB; b++) {
            ss[b] = 0.0f;
            if (b < (int)p.nb) {
                const float* xr = (const float*)p.x + (uint64_t)b * p.x_stride;
                for (uint32_t k = tid; k < p.K; k += kGemvThreads) ss[b] = fmaf(xr[k], xr[k], ss[b]);
            }
            ss[b] = warp_sum(ss[b]);
            if (lane == 0) red[warp][b] = ss[b];
        }
        __syncthreads();
#pragma unroll
        for (int b = 0; b < NB; b++) {
            float t = 0.0f;
#pragma unroll
            for (int w = 0; w < kGemvWarps; w++) t += red[w][b];
            scale[b] = 1.0f / sqrtf(t / (float)p.K + p.eps);
        }
    }
#pragma unroll
    for (int b = 0; b < NB; b++) {
        XS* dst = xs + (size_t)b * Kpad;
        if (b < (int)p.nb) {
            for (uint32_t k = tid; k < Kpad; k += kGemvThreads) {
                float v = 0.0f;
                if (k < p.K) {
                    v = load_elem(p.x, p.x_dtype, (uint64_t)b * p.x_stride + k);
                    if (PRO == kProNorm) v = load_elem(p.norm_w, p.norm_dtype, k) * (scale[b] * v);
                }
                dst[k] = from_f32<XS>(v);
            }
        } else {
            for (uint32_t k = tid; k < Kpad; k += kGemvThreads) dst[k] = from_f32<XS>(0.0f);
        }
    }
    __syncthreads();

    // 4. Main loop over this warp's (unit, chunk) range.
    uint32_t idx = wa;
    while (idx < wb) {
        const uint32_t ul = idx / nc;
        const uint32_t c0 = idx - ul * nc;
        const uint32_t c1 = min(nc, c0 + (wb - idx));
        const WT *r0, *r1;
        unit_rows<WT, EPI>(p, u0 + ul, &r0, &r1);
        float acc0[NB], acc1[NB];
#pragma unroll
        for (int b = 0; b < NB; b++) acc0[b] = acc1[b] = 0.0f;
        for (uint32_t c = c0; c < c1; c += kGemvUnroll) {
            uint4 w0[kGemvUnroll], w1[kGemvUnroll];
#pragma unroll
            for (int j = 0; j < kGemvUnroll; j++) {
                const uint32_t e = (c + j) * CH + lane * V;
                if (c + j < c1 && e < p.K) {
                    w0[j] = ld_stream(r0 + e);
                    w1[j] = ld_stream(r1 + e);
                } else {
                    w0[j] = w1[j] = make_uint4(0, 0, 0, 0);
                }
            }
#pragma unroll
            for (int j = 0; j < kGemvUnroll; j++) {
                if (c + j < c1) {
                    const uint32_t e = (c + j) * CH + lane * V;
#pragma unroll
                    for (int b = 0; b < NB; b++) {
                        const uint4 xv = *reinterpret_cast<const uint4*>(xs + (size_t)b * Kpad + e);
                        acc0[b] = dot16(w0[j], xv, acc0[b], WT());
                        acc1[b] = dot16(w1[j], xv, acc1[b], WT());
                    }
                }
            }
        }
#pragma unroll
        for (int b = 0; b < NB; b++) {
            acc0[b] = warp_sum(acc0[b]);
            acc1[b] = warp_sum(acc1[b]);
        }
        if (lane == 0) {
            float* slot = part + (size_t)(ul + warp) * NB * 2;
#pragma unroll
            for (int b = 0; b < NB; b++) {
                slot[2 * b] = acc0[b];
                slot[2 * b + 1] = acc1[b];
            }
        }
        idx += c1 - c0;
    }
    __syncthreads();

    // The next kernel may launch now: letting it in earlier takes SM slots while this
    // kernel still streams (measured slower), so the trigger follows the main loop.
    pdl_trigger();

    // 5. Fold the warps' partial sums in warp order and apply the epilogue.
    for (uint32_t t = tid; t < ucta * NB; t += kGemvThreads) {
        const uint32_t ul = t / NB, b = t % NB;
        if (b >= p.nb) continue;
        const uint32_t lo = ul * nc, hi = lo + nc;
        float y0 = 0.0f, y1 = 0.0f;
#pragma unroll
        for (uint32_t w = 0; w < kGemvWarps; w++) {
            const uint32_t a = (uint32_t)((uint64_t)w * T / kGemvWarps);
            const uint32_t e = (uint32_t)((uint64_t)(w + 1) * T / kGemvWarps);
            if (a < e && a < hi && e > lo) {
                const float* slot = part + (size_t)(ul + w) * NB * 2;
                y0 += slot[2 * b];
                y1 += slot[2 * b + 1];
            }
        }
        const uint32_t u = u0 + ul;
        if (EPI == kEpiSwiglu) {
            store_elem(p.out, p.out_dtype, (uint64_t)b * p.out_stride + u, silu_mul(y0, y1));
        } else if (EPI == kEpiQkv) {
            const uint32_t r = 2 * u;
            const uint32_t pos = p.step[b].position;
            if (r < p.qd) {
                float c, s;
                rope_cos_sin(r, p.head, pos, p.theta, &c, &s);
                float* q = p.q + (uint64_t)b * p.qd + r;
                q[0] = y0 * c - y1 * s;
                q[1] = y0 * s + y1 * c;
            } else if (pos >= p.seq) {
                if (r == p.qd) atomicOr(p.flags, kFlagPositionRange);
            } else if (r < p.qd + p.kvd) {
                const uint32_t i = r - p.qd;
                float c, s;
                rope_cos_sin(i, p.head, pos, p.theta, &c, &s);
                const uint64_t o = (uint64_t)b * p.cache_stride + (uint64_t)pos * p.kvd + i;
                store_elem(p.kcache, p.kv_dtype, o, y0 * c - y1 * s);
                store_elem(p.kcache, p.kv_dtype, o + 1, y0 * s + y1 * c);
            } else {
                const uint32_t i = r - p.qd - p.kvd;
                const uint64_t o = (uint64_t)b * p.cache_stride + (uint64_t)pos * p.kvd + i;
                store_elem(p.vcache, p.kv_dtype, o, y0);
                store_elem(p.vcache, p.kv_dtype, o + 1, y1);
            }
        } else {
            const uint32_t r = 2 * u;
            const uint64_t o = (uint64_t)b * p.out_stride + r;
            if (EPI == kEpiResidual) {
                float* out = (float*)p.out;
                out[o] += y0;
                if (r + 1 < p.n_rows) out[o + 1] += y1;
            } else {
                if (p.addend) {
                    y0 += p.addend[o];
                    if (r + 1 < p.n_rows) y1 += p.addend[o + 1];
                }
                store_elem(p.out, p.out_dtype, o, y0);
                if (r + 1 < p.n_rows) store_elem(p.out, p.out_dtype, o + 1, y1);
            }
        }
    }
}

// Generic fallback for Linear shapes the vector kernel cannot take (K not a multiple of
// the 16-byte vector, unaligned views): one warp per output row.
template <typename WT>
__global__ void gemv_scalar_kernel(const WT* __restrict__ w, uint32_t n_rows, uint32_t K,
                                   const void* x, int32_t x_dtype, uint32_t batch, void* out,
                                   int32_t out_dtype) {
    pdl_wait();
    const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32;
    if (warp >= n_rows * batch) return;
    const uint32_t row = warp % n_rows, b = warp / n_rows;
    const WT* r = w + (uint64_t)row * K;
    float acc = 0.0f;
    for (uint32_t k = lane; k < K; k += 32)
        acc = fmaf(to_f32(r[k]), load_elem(x, x_dtype, (uint64_t)b * K + k), acc);
    acc = warp_sum(acc);
    if (lane == 0) store_elem(out, out_dtype, (uint64_t)b * n_rows + row, acc);
    pdl_trigger();
}

bool gemv_fusable(int32_t wdtype, uint32_t K, const void* const* segs, int nseg) {
    const uint32_t V = wdtype == AB_BF16 ? 8 : 4;
    if (K == 0 || K % V) return false;
    for (int i = 0; i < nseg; i++)
        if ((uintptr_t)segs[i] % 16) return false;
    return true;
}

template <typename WT, int NB, int PRO, int EPI>
static void add_gemv(ab_scheme* s, const char* label, const GemvParams& p, unsigned grid,
                     size_t smem) {
    auto kern = gemv_kernel<WT, NB, PRO, EPI>;
    s->add(label, [=](cudaStream_t st) {
        if (smem > 48 * 1024) {
            cudaError_t e =
                cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
        }
        return launch(st, dim3(grid), dim3(kGemvThreads), smem, true, kern, p);
    });
}

template <typename WT, int NB>
static void dispatch_epi(ab_scheme* s, const char* label, const GemvParams& p, int pro, int epi,
                         unsigned grid, size_t smem) {
    if (pro == kProNorm) {
        switch (epi) {
            case kEpiStore: return add_gemv<WT, NB, kProNorm, kEpiStore>(s, label, p, grid, smem);
            case kEpiQkv: return add_gemv<WT, NB, kProNorm, kEpiQkv>(s, label, p, grid, smem);
            case kEpiSwiglu: return add_gemv<WT, NB, kProNorm, kEpiSwiglu>(s, label, p, grid, smem);
            default: break;
        }
    } else {
        switch (epi) {
            case kEpiStore: return add_gemv<WT, NB, kProNone, kEpiStore>(s, label, p, grid, smem);
            case kEpiResidual:
                return add_gemv<WT, NB, kProNone, kEpiResidual>(s, label, p, grid, smem);
            default: break;
        }
    }
    fail(AB_ERR_ARGUMENT, "unsupported GEMV prologue/epilogue combination");
}

// Tuning parameters of the GEMV launch (the results do not change): CTAs per SM
// (AMMON_B200_GEMV_CTAS, 1-4, default 3: with programmatic dependent launch the next
// kernel's CTAs start their prologue in the register room a fourth would take, measured 1%
// faster per decode step) and the 512-byte chunks of its first weight rows each warp
// prefetches into L2 before its prologue (AMMON_B200_GEMV_PREFETCH, default 8).
static uint32_t env_u32(const char* name, uint32_t dflt, uint32_t lo, uint32_t hi) {
    const char* e = std::getenv(name);
    if (!e) return dflt;
    const long v = std::atol(e);
    return (uint32_t)std::min<long>(hi, std::max<long>(lo, v));
}
static uint32_t gemv_ctas_per_sm() {
    static const uint32_t v = env_u32("AMMON_B200_GEMV_CTAS", 3, 1, 4);
    return v;
}
static uint32_t gemv_prefetch_chunks() {
    static const uint32_t v = env_u32("AMMON_B200_GEMV_PREFETCH", 8, 0, 64);
    return v;
}

void record_gemv(ab_scheme* s, const char* label, GemvParams p, int32_t wdtype, uint32_t batch,
                 int pro, int epi) {
    p.prefetch_chunks = gemv_prefetch_chunks();
    const uint32_t V = wdtype == AB_BF16 ? 8 : 4;
    const uint32_t CH = 32 * V;
    p.nchunks = (p.K + CH - 1) / CH;
    const uint32_t Kpad = p.nchunks * CH;
    const int sms = s->rt ? s->rt->sm_count : 148;
    if (batch > kGemvMaxBatch && p.ws != nullptr) {
        // a dense contraction: tensor-core tiles read each weight once for the whole batch
        const bool f32 = wdtype == AB_F32;
        const bool inter = epi == kEpiSwiglu;
        int nseg = 0;
        bool segs_ok = true;
        for (int i = 0; i < 3; i++)
            if (p.seg_rows[i]) nseg = i + 1;
        // stacked segments must each fill whole 128-row tiles; a single one may end short
        for (int i = 0; i < nseg; i++)
            if (!inter && nseg > 1 && p.seg_rows[i] % 128) segs_ok = false;
        const uint32_t rows = inter ? p.seg_rows[0] : p.n_rows;
        // fp32: the activation is split into tf32 halves in the scratch (normalised or not)
        const bool x_ok =
            f32 ? p.x_dtype == AB_F32 && p.xn != nullptr &&
                      (uint64_t)batch * p.K * 8 <= p.xn_bytes
                : pro == kProNorm ? p.xn != nullptr : p.x_dtype == AB_BF16;
        if (segs_ok && x_ok && gemm_tc_fits(rows, p.K, batch, inter, f32)) {
            const void* xb = p.x;
            const void* xlo = nullptr;
            uint32_t xs = p.x_stride;
            if (f32) {
                float* hi = (float*)p.xn;
                float* lo = hi + (uint64_t)batch * p.K;
                record_split_rows_tf32(s, (std::string(label) + "_split").c_str(),
                                       (const float*)p.x, p.x_stride,
                                       pro == kProNorm ? p.norm_w : nullptr, p.norm_dtype, hi, lo,
                                       batch, p.K, p.eps);
                xb = hi;
                xlo = lo;
                xs = p.K;
            } else if (pro == kProNorm) {
                record_rmsnorm_rows_bf16(s, (std::string(label) + "_norm").c_str(),
                                         (const float*)p.x, p.norm_w, p.norm_dtype, p.xn, batch,
                                         p.K, p.eps);
                xb = p.xn;
                xs = p.K;
            }
            GemmTcParams g = {};
            g.K = p.K;
            g.nb = batch;
            g.interleave = inter ? 1 : 0;
            g.ws = p.ws;
            g.ws_floats = p.ws_floats;
            g.tickets = p.tickets;
            g.tickets_n = p.tickets_n;
            g.out = p.out;
            g.out_dtype = p.out_dtype;
            g.out_stride = p.out_stride;
            g.addend = p.addend;
            g.n_rows = p.n_rows;
            g.q = p.q;
            g.qd = p.qd;
            g.kvd = p.kvd;
            g.head = p.head;
            g.seq = p.seq;
            g.theta = p.theta;
            g.kcache = p.kcache;
            g.vcache = p.vcache;
            g.kv_dtype = p.kv_dtype;
            g.cache_stride = p.cache_stride;
            g.step = p.step;
            g.flags = p.flags;
            record_gemm_tc(s, label, g, wdtype, p.seg, p.seg_rows, nseg, xb, xlo, xs, epi);
            return;
        }
    }
    for (uint32_t b0 = 0; b0 < batch; b0 += 4) {
        const uint32_t nb = std::min(4u, batch - b0);
        const uint32_t NB = nb == 1 ? 1 : nb == 2 ? 2 : 4;
        GemvParams q = p;
        q.nb = nb;
        q.x = (const char*)p.x + (uint64_t)b0 * p.x_stride * dtype_size(p.x_dtype);
        if (epi == kEpiQkv) {
            q.q = p.q + (uint64_t)b0 * p.qd;
            q.step = p.step + b0;
            q.kcache = (char*)p.kcache + (uint64_t)b0 * p.cache_stride * dtype_size(p.kv_dtype);
            q.vcache = (char*)p.vcache + (uint64_t)b0 * p.cache_stride * dtype_size(p.kv_dtype);
        } else {
            q.out = (char*)p.out + (uint64_t)b0 * p.out_stride * dtype_size(p.out_dtype);
        }
        // 3 CTAs (24 warps) per SM keep enough 16-byte loads in flight to cover HBM latency
        unsigned grid = (unsigned)std::min<uint64_t>(p.units, (uint64_t)sms * gemv_ctas_per_sm());
        grid = std::max(1u, grid);
        const uint32_t ucta = (p.units + grid - 1) / grid;
        const size_t smem = (size_t)NB * Kpad * (wdtype == AB_BF16 ? 2 : 4) +
                            (size_t)(ucta + kGemvWarps) * NB * 2 * sizeof(float);
        if (smem > 220 * 1024)
            invalid(std::string(label) + ": activation row of " + std::to_string(p.K) +
                    " elements does not fit the GEMV's shared-memory stage");
        if (wdtype == AB_BF16) {
            if (NB == 1) dispatch_epi<bf16, 1>(s, label, q, pro, epi, grid, smem);
            else if (NB == 2) dispatch_epi<bf16, 2>(s, label, q, pro, epi, grid, smem);
            else dispatch_epi<bf16, 4>(s, label, q, pro, epi, grid, smem);
        } else {
            if (NB == 1) dispatch_epi<float, 1>(s, label, q, pro, epi, grid, smem);
            else if (NB == 2) dispatch_epi<float, 2>(s, label, q, pro, epi, grid, smem);
            else dispatch_epi<float, 4>(s, label, q, pro, epi, grid, smem);
        }
    }
}

// Linear::record / TensorKernels::matmul_into: out[b, :] = weight @ x[b, :].
void record_linear(ab_scheme* s, const char* label, ab_tensor weight, ab_tensor x, ab_tensor out) {
    expect_data("weight", weight);
    expect_data("x", x);
    expect_data("out", out);
    expect_rank("weight", weight, 2);
    expect_rank_in("x", x, 1, 2);
    expect_rank_in("out", out, 1, 2);
    expect_float("weight", weight);
    expect_float("x", x);
    expect_float("out", out);
    const uint32_t d_out = weight.dims[0], d_in = weight.dims[1];
    const uint32_t batch = x.rank == 2 ? x.dims[0] : 1;
    expect_dim("x", x, x.rank - 1, "d_in", d_in);
    expect_dim("out", out, out.rank - 1, "d_out", d_out);
    if ((out.rank == 2 ? out.dims[0] : 1) != batch)
        invalid("parameter `out`: dim `batch` must match x " + shape_str(x));
    if (weight.dtype == AB_F32 && x.dtype == AB_BF16)
        invalid("parameter `x`: f32 weights take f32 activations");
    const void* seg = weight.data;
    if (gemv_fusable(weight.dtype, d_in, &seg, 1) && (uintptr_t)x.data % 4 == 0) {
        GemvParams p = {};
        p.seg[0] = weight.data;
        p.seg_rows[0] = d_out;
        p.n_rows = d_out;
        p.units = (d_out + 1) / 2;
        p.K = d_in;
        p.x = x.data;
        p.x_dtype = x.dtype;
        p.x_stride = d_in;
        p.out = out.data;
        p.out_dtype = out.dtype;
        p.out_stride = d_out;
        record_gemv(s, label, p, weight.dtype, batch, kProNone, kEpiStore);
        return;
    }
    const void* xp = x.data;
    void* op = out.data;
    const int32_t xdt = x.dtype, odt = out.dtype;
    const uint64_t warps = (uint64_t)d_out * batch;
    const unsigned grid = (unsigned)((warps * 32 + 255) / 256);
    if (weight.dtype == AB_F32) {
        const float* wp = (const float*)weight.data;
        s->add(label, [=](cudaStream_t st) {
            return launch(st, dim3(grid), dim3(256), 0, true, gemv_scalar_kernel<float>, wp, d_out,
                          d_in, xp, xdt, batch, op, odt);
        });
    } else {
        const bf16* wp = (const bf16*)weight.data;
        s->add(label, [=](cudaStream_t st) {
            return launch(st, dim3(grid), dim3(256), 0, true, gemv_scalar_kernel<bf16>, wp, d_out,
                          d_in, xp, xdt, batch, op, odt);
        });
    }
}

}  // namespace ab

using namespace ab;

extern "C" {

int ab_tensor_matmul_into(ab_scheme* s, ab_tensor a, ab_tensor b, ab_tensor out) {
    return guard([&] {
        if (!s) fail(AB_ERR_ARGUMENT, "null scheme");
        record_linear(s, "matmul", a, b, out);
    });
}

int ab_linear_record(ab_scheme* s, ab_tensor weight, ab_tensor x, ab_tensor out) {
    return guard([&] {
        if (!s) fail(AB_ERR_ARGUMENT, "null scheme");
        record_linear(s, "linear", weight, x, out);
    });
}

}  // extern "C"
