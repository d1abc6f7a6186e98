// Persistent decode step: the whole batch-1 bf16 decode step of the Llama-shaped model --
// embedding, every layer's CausalAttentionBlock and SwiGluBlock (src/blocks.rs:178-278 op
// order), final RMSNorm, classifier, greedy pick (src/tokenizer.rs:179-189) and, in the device
// loop, the next DecodeStep -- as ONE cooperative launch of one CTA per SM.
//
// Why (B200): at batch 1 every projection is a bandwidth-bound GEMV of 4-235 MB. Run as
// separate launches, each one pays a fixed ramp and tail (launch, prologue, last wave) of
// several microseconds while HBM idles; ~160 of them per token cost about a quarter of the
// step. Here the weights of every phase stream through a per-SM shared-memory ring that one
// producer thread keeps full across phase boundaries. Weights never depend on activations, so
// while the consumer warps wait at a grid barrier for the previous phase's outputs, the
// producer is already loading the next phase's rows: the dependency chain
// (norm -> QKV -> attention -> wo -> norm -> gate/up -> down -> ...) costs barrier latency,
// not idle HBM, as long as a barrier plus the activation staging takes less than the ring's
// depth at the per-SM share of HBM bandwidth (192 KB at ~44 GB/s per SM = ~4.4 us).
//
// Layout of the work:
//  - Every GEMV phase splits its output rows (row pairs; (w1, w3) row pairs for gate/up) into
//    one balanced contiguous range per CTA. A CTA's rows stream as chunks of up to 32 KB
//    (four 4096-element bf16 rows, one 14336-element w2 row, or up to four of the shorter w2
//    rows of a tensor-parallel shard) by cp.async.bulk row copies into ring slot g % 6;
//    consumer warp w takes every chunk with g % 6 == w, computes its rows' dot products from
//    shared memory (weights and the staged bf16 activation) and applies the epilogue of the
//    phase: RoPE + K/V append (QKV), residual add (wo, w2), SwiGLU (gate/up), logits + running
//    first maximum (classifier).
//  - Tensor parallelism (world > 1): the same kernel on every rank over its shards; wo and w2
//    push their partial rows into every rank's exchange block as flag-carrying pairs, and CTA
//    c sums, for the rows it produced (the same rows on every rank), the ranks' partials in
//    rank order (tp_site_reduce) before a grid barrier publishes the new residual.
//  - Attention (between QKV and wo) is flash-decoding over positions 0..pos: items of
//    (kv head, block of 32-position tiles) sized to one wave of CTAs (see ps_attention).
//  - Staging (the normalised activation, the attention output, the SwiGLU output, K/V tiles)
//    goes through cp.async with every copy in flight: the data was written in this launch by
//    other CTAs and is read through L2.
//  - Grid barriers: one counter, monotonic within a launch, reset by the last CTA to leave.
//    Every wait (ring barriers, grid barrier) is bounded by %globaltimer; a wait that runs out
//    raises kFlagWaitTimeout and an abort word that every other wait checks, so all CTAs
//    return; the producer first waits (bounded) for the copies it has in flight.
#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "internal.h"
#include "ops.h"
#include "tma.cuh"

namespace ab {

namespace {

constexpr int kPsConsumers = 6;                      // consumer warps (one ring slot each)
constexpr int kPsThreads = (kPsConsumers + 1) * 32;  // + the producer warp
constexpr int kPsSlots = kPsConsumers;
constexpr uint32_t kPsSlotBytes = 32 * 1024;
constexpr uint32_t kPsActBytes = 32 * 1024;  // staged activation / attention tiles
constexpr uint32_t kPsMaxRows = 4;           // rows per chunk
constexpr uint32_t kPsMaxG = 8;              // query heads per kv head
constexpr size_t kPsSmem = (size_t)kPsSlots * kPsSlotBytes + kPsActBytes + 1024;
// inside the activation region: the norm stages x (f32) and its gain (bf16) behind the
// staged operand (dim <= 4096)
constexpr uint32_t kPsXOff = 8 * 1024;
constexpr uint32_t kPsGainOff = 24 * 1024;

enum : uint32_t { kPhQkv = 0, kPhWo = 1, kPhGateUp = 2, kPhDown = 3, kPhCls = 4 };

// dot of eight bf16 weights with eight bf16 activations (one 16-byte vector each) over two
// accumulators: even elements into a0, odd into a1
__device__ __forceinline__ void dot_bf16x8_2(const uint4& w, const uint4& x, float& a0,
                                             float& a1) {
    a0 = fmaf(bf16lo(w.x), bf16lo(x.x), a0);
    a1 = fmaf(bf16hi(w.x), bf16hi(x.x), a1);
    a0 = fmaf(bf16lo(w.y), bf16lo(x.y), a0);
    a1 = fmaf(bf16hi(w.y), bf16hi(x.y), a1);
    a0 = fmaf(bf16lo(w.z), bf16lo(x.z), a0);
    a1 = fmaf(bf16hi(w.z), bf16hi(x.z), a1);
    a0 = fmaf(bf16lo(w.w), bf16lo(x.w), a0);
    a1 = fmaf(bf16hi(w.w), bf16hi(x.w), a1);
}

struct PsLayer {
    const bf16 *wq, *wk, *wv, *wo, *w1, *w3, *w2;
    const bf16 *rms_att, *rms_ffn;
    bf16 *kcache, *vcache;  // this layer's [seq, kv_heads, head]
};

struct PsParams {
    const PsLayer* layers;
    uint32_t L;
    const bf16* embed;
    const bf16* wcls;
    const bf16* rms_final;
    uint32_t d, qd, kvd, hd, H, KV, F, V, seq;
    uint32_t upc_qkv, upc_wo, upc_gu, upc_cls;  // units (row pairs) per chunk
    uint32_t upc_down;                          // w2 rows per chunk
    float theta, eps;
    Step* step;
    float* x;         // [d] residual stream
    float* q;         // [qd] rotated queries
    bf16* o;          // [qd] attention output (feeds wo)
    bf16* h;          // [F] SwiGLU output (feeds w2)
    float* logits;    // [V]
    float* part;      // attention block partials O [KV][grid][G][hd]
    float* part_ml;   // and their (max, sum) [KV][ml_stride] ([grid][G][2] used)
    uint32_t ml_stride;  // floats per kv head in part_ml (a multiple of 4)
    uint32_t* tickets;  // [KV + 1]: attention folds, then the argmax merge
    float* cand_v;    // [grid] best logit of each CTA
    uint32_t* cand_i;
    int32_t* argmax;
    int32_t* history;  // [seq] (feedback)
    uint32_t feedback;
    uint32_t* bar;     // [0] grid barrier counter, [1] exit counter, [2] abort word
    uint32_t* flags;
    uint32_t stall_barrier;  // test hook: CTA 0 never arrives at this barrier (0 = none)
    uint64_t* trace;         // optional [barriers][kTrCols][grid] %globaltimer (trace_at)
    // tensor parallelism (world > 1): every rank's exchange block as this rank addresses it
    // (layout kXb*), the second residual buffer (all-reduce sites alternate x and x2), this
    // rank's counts (launches, all-reduce sites) and the first vocabulary id of its
    // classifier rows
    uint32_t world, rank, vocab_off;
    uint32_t vocab_all;  // rows of the (replicated) embedding table: V times the ranks
    unsigned char* xb[kTpMaxWorld];
    float* x2;
    unsigned long long* launch;  // [0] launches, [1] all-reduce sites
};

// Exchange block of one rank: [16] this rank's launch count (u64), [24] all-reduce sites run
// so far (u64), [64] argmax candidates [world] x two pairs (f32 value, u32 id), [256] partial
// projections
// [2 parities][world][d] of 8-byte pairs (f32 value, u32 site flag). A pair is written with
// one 8-byte store, so a reader that sees the site's flag sees that site's value: the
// all-reduce needs no fence or arrival counter (the flag-in-data scheme of low-latency
// collectives). The counts only grow, kept with the block for the communicator's life
// (models that share a communicator continue them): site k of a launch carries flag
// S + k + 1 for the S sites run before it, its argmax candidates S + 2L + 1 (32 bits: unique
// for 2^32 sites). A launch that ended early still advances both counts on every rank, so the
// ranks' flags stay in step after an error.
constexpr uint32_t kXbLaunch = 16, kXbSites = 24, kXbCand = 64, kXbPart = 256;

static_assert(kXbSites == kXbLaunch + 8, "the counts word pair: launches, then sites");

// rank `r`'s block as this rank addresses it: the pair slots of parity `par`, [world][d]; a
// pair is one u64 (low half the f32 value's bits, high half the flag), so one scalar 8-byte
// access moves both
__device__ __forceinline__ unsigned long long* xb_pairs(const PsParams& p, uint32_t r,
                                                        uint32_t par) {
    return reinterpret_cast<unsigned long long*>(p.xb[r] + kXbPart) +
           (size_t)par * p.world * p.d;
}
__device__ __forceinline__ unsigned long long mk_pair(float v, uint32_t flag) {
    return (unsigned long long)__float_as_uint(v) | ((unsigned long long)flag << 32);
}
__device__ __forceinline__ void st_pair(unsigned long long* dst, float v, uint32_t flag) {
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(dst), "l"(mk_pair(v, flag))
                 : "memory");
}
// two consecutive pairs in one 16-byte store (two 8-byte elements, each landing whole)
__device__ __forceinline__ void st_pair2(unsigned long long* dst, float v0, float v1,
                                         uint32_t flag) {
    asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(dst), "l"(mk_pair(v0, flag)),
                 "l"(mk_pair(v1, flag))
                 : "memory");
}
__device__ __forceinline__ unsigned long long ld_pair(const unsigned long long* src) {
    unsigned long long v;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(src) : "memory");
    return v;
}

// ---- shared-memory layout ------------------------------------------------------------------
struct PsSmem {
    unsigned char* ring;
    unsigned char* act;
    uint64_t* full;   // [kPsSlots]
    uint64_t* empty;  // [kPsSlots]
    float* red;       // [32] reductions
    uint32_t* misc;   // [32]: 0 barrier result, 1 fold ticket, 2 CTA aborting, 8.. warp ids
};

__device__ __forceinline__ PsSmem ps_smem(unsigned char* base) {
    PsSmem s;
    s.ring = base;
    s.act = base + (size_t)kPsSlots * kPsSlotBytes;
    unsigned char* tail = s.act + kPsActBytes;
    s.full = reinterpret_cast<uint64_t*>(tail);
    s.empty = s.full + kPsSlots;
    s.red = reinterpret_cast<float*>(s.empty + kPsSlots);
    s.misc = reinterpret_cast<uint32_t*>(s.red + 32);
    return s;
}

__device__ __forceinline__ void consumers_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kPsConsumers * 32) : "memory");
}

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar` (16-byte aligned
// addresses, size a multiple of 16).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

// 16-byte asynchronous copy global -> shared through L2 only (so data other CTAs wrote in
// this launch is seen), completed by cp_async_wait_all.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.wait_all;" ::: "memory");
}

// n 16-byte vectors src -> dst (shared) by the consumer threads, every copy in flight at once.
__device__ __forceinline__ void stage_async(void* dst, const void* src, uint32_t n16) {
    const uint4* g = reinterpret_cast<const uint4*>(src);
    uint4* d = reinterpret_cast<uint4*>(dst);
    for (uint32_t i = threadIdx.x; i < n16; i += kPsConsumers * 32) cp_async16(d + i, g + i);
}

__device__ __forceinline__ uint32_t ld_relaxed(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ bool aborted(const PsParams& p) { return ld_relaxed(p.bar + 2) != 0; }

__device__ __forceinline__ void raise_abort(const PsParams& p) {
    atomicOr(p.flags, kFlagWaitTimeout);
    atomicExch(p.bar + 2, 1u);
}

// Bounded wait on an mbarrier phase that also gives up when another CTA aborted.
__device__ __forceinline__ bool ps_wait(const PsParams& p, uint32_t bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    WaitClock clock;
    uint32_t n = 0;
    while (!mbar_try_wait(bar, parity)) {
        if ((++n & 63) == 0) {
            if (aborted(p)) return false;
            if (clock.expired(p.flags)) {
                raise_abort(p);
                return false;
            }
        }
    }
    return true;
}

// Phase geometry: units, rows per unit, units per chunk, K.
struct PsGeom {
    uint32_t units, rpu, upc, K;
};

__device__ __forceinline__ PsGeom ps_geom(const PsParams& p, uint32_t kind) {
    switch (kind) {
        case kPhQkv: return {(p.qd + 2 * p.kvd) / 2, 2, p.upc_qkv, p.d};
        case kPhWo: return {p.d / 2, 2, p.upc_wo, p.qd};
        case kPhGateUp: return {p.F, 2, p.upc_gu, p.d};
        case kPhDown: return {p.d, 1, p.upc_down, p.F};
        default: return {p.V / 2, 2, p.upc_cls, p.d};
    }
}

__device__ __forceinline__ const bf16* ps_row(const PsParams& p, const PsLayer& ly,
                                              uint32_t kind, uint32_t u, uint32_t r) {
    switch (kind) {
        case kPhQkv: {
            const uint32_t v = 2 * u + r;
            if (v < p.qd) return ly.wq + (uint64_t)v * p.d;
            if (v < p.qd + p.kvd) return ly.wk + (uint64_t)(v - p.qd) * p.d;
            return ly.wv + (uint64_t)(v - p.qd - p.kvd) * p.d;
        }
        case kPhWo: return ly.wo + (uint64_t)(2 * u + r) * p.qd;
        case kPhGateUp: return (r == 0 ? ly.w1 : ly.w3) + (uint64_t)u * p.d;
        case kPhDown: return ly.w2 + (uint64_t)u * p.F;
        default: return p.wcls + (uint64_t)(2 * u + r) * p.d;
    }
}

__device__ __forceinline__ void cta_range(uint32_t units, uint32_t* u0, uint32_t* u1) {
    *u0 = (uint32_t)((uint64_t)units * blockIdx.x / gridDim.x);
    *u1 = (uint32_t)((uint64_t)units * (blockIdx.x + 1) / gridDim.x);
}

// ---- producer ------------------------------------------------------------------------------
// Streams the CTA's rows of one phase into the ring; g counts chunks over the whole step. One
// thread: its reaction time (slot freed -> copies issued) is part of every ring round trip,
// so it keeps the layer's pointers in registers and does nothing else.
__device__ bool produce_phase(const PsParams& p, const PsSmem& s, uint32_t kind, uint32_t l,
                              uint32_t& g) {
    const PsGeom gm = ps_geom(p, kind);
    const PsLayer ly = kind == kPhCls ? PsLayer{} : p.layers[l];
    uint32_t u0, u1;
    cta_range(gm.units, &u0, &u1);
    const uint32_t row_bytes = gm.K * 2;
    for (uint32_t u = u0; u < u1; u += gm.upc, g++) {
        const uint32_t slot = g % kPsSlots, round = g / kPsSlots;
        if (round > 0 && !ps_wait(p, smem_u32(&s.empty[slot]), (round - 1) & 1)) return false;
        const uint32_t n = min(gm.upc, u1 - u);
        const uint32_t full = smem_u32(&s.full[slot]);
        mbar_arrive_expect_tx(full, n * gm.rpu * row_bytes);
        uint32_t dst = smem_u32(s.ring + (size_t)slot * kPsSlotBytes);
        for (uint32_t i = 0; i < n; i++)
            for (uint32_t r = 0; r < gm.rpu; r++) {
                bulk_load(dst, ps_row(p, ly, kind, u + i, r), row_bytes, full);
                dst += row_bytes;
            }
    }
    return true;
}

// ---- consumers: staging --------------------------------------------------------------------
// xs = bf16(gain * (ss * x)), ss = 1 / sqrt(mean(x^2) + eps): the RMSNorm of
// src/kernels.rs:75-101 (o = w * (ss * x)) with bf16 rounding of the operand of the next Linear.
// The norm of the x already staged (f32) in the activation region.
__device__ void norm_from_xf(const PsParams& p, const PsSmem& s, const bf16* gain) {
    const uint32_t tid = threadIdx.x, n = kPsConsumers * 32;
    float* xf = reinterpret_cast<float*>(s.act + kPsXOff);
    bf16* gs = reinterpret_cast<bf16*>(s.act + kPsGainOff);
    stage_async(gs, gain, p.d / 8);
    cp_async_wait_all();
    consumers_sync();
    float ss = 0.0f;
    for (uint32_t i = tid; i < p.d; i += n) ss = fmaf(xf[i], xf[i], ss);
    ss = warp_sum(ss);
    if (tid % 32 == 0) s.red[tid / 32] = ss;
    consumers_sync();
    float t = 0.0f;
#pragma unroll
    for (int w = 0; w < kPsConsumers; w++) t += s.red[w];
    const float scale = 1.0f / sqrtf(t / (float)p.d + p.eps);
    bf16* xs = reinterpret_cast<bf16*>(s.act);
    for (uint32_t i = tid; i < p.d; i += n)
        xs[i] = __float2bfloat16_rn(__bfloat162float(gs[i]) * (scale * xf[i]));
    consumers_sync();
}

__device__ void stage_norm(const PsParams& p, const PsSmem& s, const float* x, const bf16* gain) {
    stage_async(s.act + kPsXOff, x, p.d / 4);
    norm_from_xf(p, s, gain);
}

// Tensor parallelism, the all-reduce of one site: x_new = x_old + the ranks' partial rows,
// summed in rank order (every rank adds the same values in the same order, so the replicated
// residual stays bit-identical). Every rank splits a phase's rows over its CTAs the same way,
// so CTA c produced rows [r0, r1) on every rank: it waits for exactly those rows' pairs from
// every rank (the site's flag in each; one thread per pair, all polls in flight together),
// sums them and writes x_new[r0, r1). A grid barrier after it publishes the whole x_new on
// this rank. Bounded like every wait; false when this thread gave up.
__device__ bool tp_site_reduce(const PsParams& p, const PsSmem& s, uint32_t par, uint32_t r0,
                               uint32_t r1, uint32_t flag, const float* x_old, float* x_new) {
    consumers_sync();  // every warp is done with the phase's operand in the activation stage
    const uint32_t n = r1 - r0, total = n * p.world;
    float* vals = reinterpret_cast<float*>(s.act);  // [world][n]
    const unsigned long long* pairs = xb_pairs(p, p.rank, par);
    bool ok = true;
    for (uint32_t i = threadIdx.x; i < total && ok; i += kPsConsumers * 32) {
        const uint32_t r = i / n, u = r0 + i % n;
        const unsigned long long* src = pairs + (size_t)r * p.d + u;
        unsigned long long v = ld_pair(src);
        if ((uint32_t)(v >> 32) != flag) {
            WaitClock clock;
            uint32_t k = 0;
            while ((uint32_t)((v = ld_pair(src)) >> 32) != flag) {
                if ((++k & 15) == 0) {
                    if (aborted(p)) {
                        ok = false;
                        break;
                    }
                    if (clock.expired(p.flags)) {
                        raise_abort(p);
                        ok = false;
                        break;
                    }
                }
            }
        }
        vals[i] = __uint_as_float((uint32_t)v);
    }
    consumers_sync();
    for (uint32_t i = threadIdx.x; i < n; i += kPsConsumers * 32) {
        float a = __ldcg(x_old + r0 + i);
        for (uint32_t r = 0; r < p.world; r++) a += vals[r * n + i];
        x_new[r0 + i] = a;
    }
    return ok;
}

// xs = src[0 .. n) (bf16 produced earlier in this launch).
__device__ void stage_copy(const PsSmem& s, const bf16* src, uint32_t n) {
    stage_async(s.act, src, n / 8);
    cp_async_wait_all();
    consumers_sync();
}

// ---- consumers: one chunk ------------------------------------------------------------------
// R rows (row-major, nv 16-byte vectors each) against the staged vector: every lane takes
// vectors lane, lane + 32, ... with U of them (times R rows) in flight per iteration and two
// accumulator chains per row and in-flight vector; sums[r] gets row r's lane partial.
template <uint32_t R, uint32_t U>
__device__ __forceinline__ void dots_rows(const uint4* w, const uint4* xv, uint32_t nv,
                                          float* sums) {
    const uint32_t lane = threadIdx.x % 32;
    float a0[R][U], a1[R][U];
#pragma unroll
    for (uint32_t r = 0; r < R; r++)
#pragma unroll
        for (uint32_t u = 0; u < U; u++) a0[r][u] = a1[r][u] = 0.0f;
    uint32_t j = lane;
    for (; j + 32 * (U - 1) < nv; j += 32 * U) {
        uint4 xa[U], wa[R][U];
#pragma unroll
        for (uint32_t u = 0; u < U; u++) {
            xa[u] = xv[j + 32 * u];
#pragma unroll
            for (uint32_t r = 0; r < R; r++) wa[r][u] = w[r * nv + j + 32 * u];
        }
#pragma unroll
        for (uint32_t u = 0; u < U; u++)
#pragma unroll
            for (uint32_t r = 0; r < R; r++) dot_bf16x8_2(wa[r][u], xa[u], a0[r][u], a1[r][u]);
    }
    for (; j < nv; j += 32) {
        const uint4 x = xv[j];
#pragma unroll
        for (uint32_t r = 0; r < R; r++) dot_bf16x8_2(w[r * nv + j], x, a0[r][0], a1[r][0]);
    }
#pragma unroll
    for (uint32_t r = 0; r < R; r++) {
        float t = 0.0f;
#pragma unroll
        for (uint32_t u = 0; u < U; u++) t += a0[r][u] + a1[r][u];
        sums[r] = t;
    }
}

// Dot products of the chunk's rows (row-major, K elements each, back to back in the slot) with
// the staged activation; every lane ends with every row's sum.
__device__ __forceinline__ void chunk_dots(const unsigned char* slot, const unsigned char* act,
                                           uint32_t rows, uint32_t K, float acc[kPsMaxRows]) {
    const uint32_t nv = K / 8;
    const uint4* w = reinterpret_cast<const uint4*>(slot);
    const uint4* xv = reinterpret_cast<const uint4*>(act);
    float part[kPsMaxRows];
#pragma unroll
    for (uint32_t r = 0; r < kPsMaxRows; r++) part[r] = 0.0f;
    if (rows == 4) dots_rows<4, 2>(w, xv, nv, part);
    else if (rows == 2) dots_rows<2, 2>(w, xv, nv, part);
    else if (rows == 1) dots_rows<1, 4>(w, xv, nv, part);
    else dots_rows<3, 1>(w, xv, nv, part);
#pragma unroll
    for (uint32_t r = 0; r < kPsMaxRows; r++) acc[r] = warp_sum(part[r]);
}

struct PsBest {
    float v;
    uint32_t i;
};

__device__ __forceinline__ PsBest first_max2(PsBest a, PsBest b) {
    if (b.i == 0xffffffffu) return a;
    if (a.i == 0xffffffffu || b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
    return a;
}

// Consumes this warp's chunks of one phase (chunk g goes to warp g % kPsSlots).
// `flag`: the all-reduce site's flag (tensor parallelism, wo and w2 phases).
__device__ bool consume_phase(const PsParams& p, const PsSmem& s, uint32_t kind, uint32_t l,
                              uint32_t& g, uint32_t pos, bool pos_ok, PsBest* best,
                              uint32_t flag = 0) {
    const bool tp = p.world > 1;
    const uint32_t par = kind == kPhDown ? 1u : 0u;  // all-reduce site parity
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const PsGeom gm = ps_geom(p, kind);
    const PsLayer* ly = kind == kPhCls ? nullptr : p.layers + l;
    uint32_t u0, u1;
    cta_range(gm.units, &u0, &u1);
    for (uint32_t u = u0; u < u1; u += gm.upc, g++) {
        const uint32_t slot = g % kPsSlots;
        if (slot != warp) continue;
        const uint32_t n = min(gm.upc, u1 - u);
        const uint32_t rows = n * gm.rpu;
        // the residual rows this chunk adds to, loaded before the wait hide their latency
        float2 xr = make_float2(0.0f, 0.0f);
        if (!tp && kind == kPhWo && lane < n)
            xr = __ldcg(reinterpret_cast<const float2*>(p.x) + u + lane);
        if (!tp && kind == kPhDown && lane < n) xr.x = __ldcg(p.x + u + lane);
        // every lane waits; the warp agrees on one outcome before the full-mask shuffles below
        const bool landed = ps_wait(p, smem_u32(&s.full[slot]), (g / kPsSlots) & 1);
        if (!__all_sync(0xffffffffu, landed)) return false;
        float acc[kPsMaxRows];
        chunk_dots(s.ring + (size_t)slot * kPsSlotBytes, s.act, rows, gm.K, acc);
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&s.empty[slot]));
        // epilogue: lane i takes unit i (pairs) or row i (down)
        if (kind == kPhCls) {
            // every lane holds every sum: the running first maximum stays warp-uniform
#pragma unroll
            for (uint32_t r = 0; r < kPsMaxRows; r++) {
                if (r >= rows) break;
                const uint32_t row = 2 * u + r;
                if (lane == r) p.logits[row] = acc[r];
                if (acc[r] > best->v || (best->i == 0xffffffffu && acc[r] == best->v)) {
                    best->v = acc[r];
                    best->i = row + p.vocab_off;
                }
            }
            continue;
        }
        if (lane >= n) continue;
        if (kind == kPhDown) {  // lane i: w2 row u + i
            float y = acc[0];
#pragma unroll
            for (uint32_t r = 1; r < kPsMaxRows; r++)
                if (r == lane) y = acc[r];
            if (tp) {  // this rank's partial row, into every rank's exchange block
                for (uint32_t r = 0; r < p.world; r++)
                    st_pair(xb_pairs(p, r, par) + (size_t)p.rank * p.d + u + lane, y, flag);
            } else {
                p.x[u + lane] = xr.x + y;
            }
            continue;
        }
        float y0 = acc[0], y1 = acc[1];
#pragma unroll
        for (uint32_t i = 1; i < kPsMaxRows / 2; i++)
            if (lane == i) {
                y0 = acc[2 * i];
                y1 = acc[2 * i + 1];
            }
        const uint32_t unit = u + lane;
        if (kind == kPhGateUp) {
            p.h[unit] = __float2bfloat16_rn(silu_mul(y0, y1));
        } else if (kind == kPhWo) {
            if (tp) {
                for (uint32_t r = 0; r < p.world; r++)
                    st_pair2(xb_pairs(p, r, par) + (size_t)p.rank * p.d + 2 * unit, y0, y1, flag);
            } else {
                reinterpret_cast<float2*>(p.x)[unit] = make_float2(xr.x + y0, xr.y + y1);
            }
        } else {  // kPhQkv: RoPE (src/kernels.rs:174-210) and the K/V append (:212-226)
            const uint32_t r = 2 * unit;
            if (r < p.qd) {
                float c, sn;
                rope_cos_sin(r, p.hd, pos, p.theta, &c, &sn);
                p.q[r] = y0 * c - y1 * sn;
                p.q[r + 1] = y0 * sn + y1 * c;
            } else if (pos_ok && r < p.qd + p.kvd) {
                const uint32_t i = r - p.qd;
                float c, sn;
                rope_cos_sin(i, p.hd, pos, p.theta, &c, &sn);
                bf16* k = ly->kcache + (uint64_t)pos * p.kvd + i;
                k[0] = __float2bfloat16_rn(y0 * c - y1 * sn);
                k[1] = __float2bfloat16_rn(y0 * sn + y1 * c);
            } else if (pos_ok) {
                const uint32_t i = r - p.qd - p.kvd;
                bf16* v = ly->vcache + (uint64_t)pos * p.kvd + i;
                v[0] = __float2bfloat16_rn(y0);
                v[1] = __float2bfloat16_rn(y1);
            }
        }
    }
    return true;
}

// ---- trace ---------------------------------------------------------------------------------
// AMMON_B200_STEP_TRACE: [barriers][kTrCols][grid] %globaltimer nanoseconds per CTA and barrier.
enum : uint32_t { kTrArrive = 0, kTrRelease = 1, kTrStaged = 2, kTrSignal = 3, kTrCols = 4 };
__device__ __forceinline__ void trace_at(const PsParams& p, uint32_t barrier, uint32_t col) {
    p.trace[((uint64_t)barrier * kTrCols + col) * gridDim.x + blockIdx.x] = global_timer_ns();
}

// ---- grid barrier --------------------------------------------------------------------------
// All consumer threads call it; thread 0 arrives and waits for every CTA's arrival number
// `epoch`. ok_in false (any warp) makes the whole CTA leave. Returns false when aborting.
__device__ bool grid_barrier(const PsParams& p, const PsSmem& s, uint32_t& epoch,
                             bool ok_in = true) {
    if (!ok_in) s.misc[2] = 1;
    consumers_sync();
    epoch++;
    if (threadIdx.x == 0) {
        uint32_t ok = s.misc[2] == 0;
        if (p.stall_barrier == epoch && blockIdx.x == 0) ok = 0;  // test hook: never arrives
        if (ok && p.trace)
            trace_at(p, epoch - 1, kTrArrive);
        if (ok) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.bar) : "memory");
        const uint32_t target = epoch * gridDim.x;
        if (ok && ld_acquire(p.bar) < target) {
            WaitClock clock;
            uint32_t n = 0;
            while (ld_acquire(p.bar) < target) {
                if ((++n & 15) == 0) {
                    if (aborted(p)) {
                        ok = 0;
                        break;
                    }
                    if (clock.expired(p.flags)) {
                        raise_abort(p);
                        ok = 0;
                        break;
                    }
                }
            }
        }
        s.misc[0] = ok;
        if (ok && p.trace)
            trace_at(p, epoch - 1, kTrRelease);
    }
    consumers_sync();
    return s.misc[0] != 0;
}


// Trace point: the CTA has staged the operand of the phase that ends at barrier epoch + 1.
__device__ __forceinline__ void trace_staged(const PsParams& p, uint32_t epoch) {
    if (p.trace && threadIdx.x == 0) trace_at(p, epoch, kTrStaged);
}

// ---- attention -----------------------------------------------------------------------------
// Flash-decoding over positions [0, npos) of this layer for batch row 0 (src/kernels.rs:
// 228-410 semantics: scores q.k / sqrt(head), softmax over the positions, weighted V sum).
// Items of (kv head, block of 32-position tiles), at most one per CTA. The CTA stages a tile's
// K rows (16-byte chunks XOR-swizzled by row, so the lane-per-position reads spread over the
// banks) and V rows with every copy in flight; warp w owns query heads w and w + 6 of the
// group end to end (lanes own positions for q.K, head dimensions for P.V). With one item per
// kv head the warp writes the output; otherwise it leaves (O, m, l) and the last CTA of the kv
// head (atomic ticket) folds the blocks in block order.
constexpr uint32_t kPsTile = 32;  // attention positions per tile
// The K/V tiles live behind the staged projection operand (at most 8 KB while QKV runs).
constexpr uint32_t kPsTileOff = 8 * 1024;

// This CTA's attention item: kv head, block and its positions [t0, t1); false when it has none.
struct PsItem {
    uint32_t kvh, blk, Se, t0, t1;
};
__device__ __forceinline__ bool attn_item(const PsParams& p, uint32_t npos, PsItem* it) {
    uint32_t S = min(gridDim.x / p.KV, (npos + kPsTile - 1) / kPsTile);
    S = max(S, 1u);
    const uint32_t bl = ((npos + S - 1) / S + kPsTile - 1) / kPsTile * kPsTile;
    it->Se = npos ? (npos + bl - 1) / bl : 1;
    if (blockIdx.x >= p.KV * it->Se) return false;
    it->kvh = blockIdx.x / it->Se;
    it->blk = blockIdx.x % it->Se;
    it->t0 = min(npos, it->blk * bl);
    it->t1 = min(npos, it->t0 + bl);
    return true;
}

// Copies rows [tile, tile + n) of the item's K (16-byte chunks XOR-swizzled by row) and V into
// the tile stage, skipping row `skip` (written later in this launch).
template <int HD>
__device__ __forceinline__ void attn_load_tile(const PsParams& p, const PsSmem& s,
                                               const PsLayer& ly, uint32_t kvh, uint32_t tile,
                                               uint32_t n, uint32_t skip) {
    constexpr uint32_t NCH = HD * 2 / 16, ROWB = HD * 2;
    unsigned char* ks = s.act + kPsTileOff;
    unsigned char* vs = ks + kPsTile * ROWB;
    const bf16* kbase = ly.kcache + (uint64_t)kvh * HD;
    const bf16* vbase = ly.vcache + (uint64_t)kvh * HD;
    for (uint32_t c = threadIdx.x; c < n * NCH; c += kPsConsumers * 32) {
        const uint32_t row = c / NCH, ch = c % NCH;
        if (tile + row == skip) continue;
        const uint64_t off = (uint64_t)(tile + row) * p.kvd + ch * 8;
        cp_async16(ks + row * ROWB + ((ch ^ (row % NCH)) * 16), kbase + off);
        cp_async16(vs + row * ROWB + ch * 16, vbase + off);
    }
}

// Issued right after the QKV operand is staged: the item's first tile without the row at pos
// (that one is this step's, written by the QKV phase). Returns whether it issued.
template <int HD>
__device__ bool attn_prestage(const PsParams& p, const PsSmem& s, uint32_t l, uint32_t npos) {
    PsItem it;
    if (npos == 0 || !attn_item(p, npos, &it) || it.t0 >= it.t1) return false;
    attn_load_tile<HD>(p, s, p.layers[l], it.kvh, it.t0, min(kPsTile, it.t1 - it.t0), npos - 1);
    return true;
}

__device__ bool attn_prestage_any(const PsParams& p, const PsSmem& s, uint32_t l, uint32_t npos) {
    if (p.hd == 128) return attn_prestage<128>(p, s, l, npos);
    if (p.hd == 64) return attn_prestage<64>(p, s, l, npos);
    return attn_prestage<32>(p, s, l, npos);
}

template <int HD>
__device__ void ps_attention(const PsParams& p, const PsSmem& s, uint32_t l, uint32_t npos,
                             bool staged) {
    constexpr uint32_t DPL = HD / 32;      // head dims per lane
    constexpr uint32_t NCH = HD * 2 / 16;  // 16-byte chunks per row
    constexpr uint32_t TP = kPsTile;
    constexpr uint32_t ROWB = HD * 2;
    const uint32_t tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    const uint32_t G = p.H / p.KV;
    PsItem it;
    if (!attn_item(p, npos, &it)) return;  // CTA-uniform
    const uint32_t kvh = it.kvh, blk = it.blk, Se = it.Se, t0 = it.t0, t1 = it.t1;
    const PsLayer& ly = p.layers[l];
    unsigned char* ks = s.act + kPsTileOff;                       // [TP][ROWB], swizzled
    unsigned char* vs = ks + TP * ROWB;                           // [TP][ROWB]
    float* qs = reinterpret_cast<float*>(s.act);                  // [G][HD]
    stage_async(qs, p.q + (uint64_t)kvh * G * HD, G * HD / 4);
    const float scale = 1.0f / sqrtf((float)HD);
    const uint32_t h0 = warp, h1 = warp + kPsConsumers;  // this warp's heads (if < G)
    float m[2] = {-INFINITY, -INFINITY}, lsum[2] = {0.0f, 0.0f}, acc[2][DPL];
#pragma unroll
    for (int hs = 0; hs < 2; hs++)
#pragma unroll
        for (uint32_t d = 0; d < DPL; d++) acc[hs][d] = 0.0f;
    for (uint32_t tile = t0; tile < t1; tile += TP) {
        const uint32_t n = min(TP, t1 - tile);
        if (tile == t0 && staged) {
            // the rest of the first tile arrived during the QKV phase; add the row at pos
            if (npos - 1 >= tile && npos - 1 < tile + n) {
                const uint32_t row = npos - 1 - tile;
                for (uint32_t ch = tid; ch < NCH; ch += kPsConsumers * 32) {
                    const uint64_t off = (uint64_t)(npos - 1) * p.kvd + (uint64_t)kvh * HD + ch * 8;
                    cp_async16(ks + row * ROWB + ((ch ^ (row % NCH)) * 16), ly.kcache + off);
                    cp_async16(vs + row * ROWB + ch * 16, ly.vcache + off);
                }
            }
        } else {
            attn_load_tile<HD>(p, s, ly, kvh, tile, n, 0xffffffffu);
        }
        cp_async_wait_all();
        consumers_sync();
        const bool valid = lane < n;
#pragma unroll
        for (int hs = 0; hs < 2; hs++) {
            const uint32_t h = hs == 0 ? h0 : h1;
            if (h >= G) break;  // warp-uniform
            // q.K: lane = position
            float sc = 0.0f;
            if (valid) {
                const float* qh = qs + h * HD;
#pragma unroll
                for (uint32_t v = 0; v < NCH; v++) {
                    const uint4 kk = *reinterpret_cast<const uint4*>(
                        ks + lane * ROWB + ((v ^ (lane % NCH)) * 16));
                    const float4 qa = *reinterpret_cast<const float4*>(qh + v * 8);
                    const float4 qb = *reinterpret_cast<const float4*>(qh + v * 8 + 4);
                    sc = fmaf(qa.x, bf16lo(kk.x), sc);
                    sc = fmaf(qa.y, bf16hi(kk.x), sc);
                    sc = fmaf(qa.z, bf16lo(kk.y), sc);
                    sc = fmaf(qa.w, bf16hi(kk.y), sc);
                    sc = fmaf(qb.x, bf16lo(kk.z), sc);
                    sc = fmaf(qb.y, bf16hi(kk.z), sc);
                    sc = fmaf(qb.z, bf16lo(kk.w), sc);
                    sc = fmaf(qb.w, bf16hi(kk.w), sc);
                }
            }
            const float x = valid ? sc * scale : -INFINITY;
            const float mnew = fmaxf(m[hs], warp_max(x));
            const float alpha = m[hs] == -INFINITY ? 0.0f : expf(m[hs] - mnew);
            const float e = valid ? expf(x - mnew) : 0.0f;
            lsum[hs] = lsum[hs] * alpha + warp_sum(e);
            m[hs] = mnew;
#pragma unroll
            for (uint32_t d = 0; d < DPL; d++) acc[hs][d] *= alpha;
            // P.V: lane = head dimensions lane * DPL ..
            for (uint32_t j = 0; j < n; j++) {
                const float ej = __shfl_sync(0xffffffffu, e, j);
                const unsigned char* vr = vs + j * ROWB + lane * DPL * 2;
                float vv[DPL];
                if constexpr (DPL == 4) {
                    const uint2 w2 = *reinterpret_cast<const uint2*>(vr);
                    vv[0] = bf16lo(w2.x);
                    vv[1] = bf16hi(w2.x);
                    vv[2] = bf16lo(w2.y);
                    vv[3] = bf16hi(w2.y);
                } else if constexpr (DPL == 2) {
                    const uint32_t w1 = *reinterpret_cast<const uint32_t*>(vr);
                    vv[0] = bf16lo(w1);
                    vv[1] = bf16hi(w1);
                } else {
                    vv[0] = __bfloat162float(*reinterpret_cast<const bf16*>(vr));
                }
#pragma unroll
                for (uint32_t d = 0; d < DPL; d++) acc[hs][d] = fmaf(ej, vv[d], acc[hs][d]);
            }
        }
        consumers_sync();  // the next tile overwrites the stage
    }
    cp_async_wait_all();  // the q copies, when the item had no tile to wait for
    // this warp's heads: the output (one block) or the block's partial
#pragma unroll
    for (int hs = 0; hs < 2; hs++) {
        const uint32_t h = hs == 0 ? h0 : h1;
        if (h >= G) break;
        if (Se == 1) {
            const float inv = lsum[hs] > 0.0f ? 1.0f / lsum[hs] : 0.0f;
#pragma unroll
            for (uint32_t d = 0; d < DPL; d++)
                p.o[(uint64_t)(kvh * G + h) * HD + lane * DPL + d] =
                    __float2bfloat16_rn(acc[hs][d] * inv);
        } else {
            const uint64_t slot = ((uint64_t)kvh * gridDim.x + blk) * G + h;
#pragma unroll
            for (uint32_t d = 0; d < DPL; d++) p.part[slot * HD + lane * DPL + d] = acc[hs][d];
            if (lane == 0) {
                float* ml = p.part_ml + (uint64_t)kvh * p.ml_stride + ((uint64_t)blk * G + h) * 2;
                ml[0] = m[hs];
                ml[1] = lsum[hs];
            }
        }
    }
    if (Se == 1) return;
    consumers_sync();
    if (tid == 0) {
        __threadfence();
        s.misc[1] = atomicAdd(p.tickets + kvh, 1u) == Se - 1;
    }
    consumers_sync();
    if (!s.misc[1]) return;
    __threadfence();
    // fold: per head the blocks' weights exp(m_b - M) (shared), then O over the blocks in
    // block order with eight loads in flight per thread
    const uint64_t base = (uint64_t)kvh * gridDim.x * G;
    // every block's (m, l) in one round trip: [Se][G][2] floats, 16-byte pieces
    float* ml = reinterpret_cast<float*>(s.act + 16 * 1024);
    stage_async(ml, p.part_ml + (uint64_t)kvh * p.ml_stride, (Se * G * 2 + 3) / 4);
    cp_async_wait_all();
    consumers_sync();
    float* wts = reinterpret_cast<float*>(s.act);  // [G][Se] weights, then [G] 1 / L
    float* inv = wts + G * Se;
    if (tid < G) {
        const uint32_t h = tid;
        float M = -INFINITY;
        for (uint32_t b = 0; b < Se; b++) M = fmaxf(M, ml[(b * G + h) * 2]);
        float Lt = 0.0f;
        for (uint32_t b = 0; b < Se; b++) {
            const float mb = ml[(b * G + h) * 2];
            const float w = (M == -INFINITY || mb == -INFINITY) ? 0.0f : expf(mb - M);
            wts[h * Se + b] = w;
            Lt += ml[(b * G + h) * 2 + 1] * w;
        }
        inv[h] = Lt > 0.0f ? 1.0f / Lt : 0.0f;
    }
    consumers_sync();
    for (uint32_t i = tid; i < G * HD / 4; i += kPsConsumers * 32) {
        const uint32_t h = i / (HD / 4), d4 = i % (HD / 4);
        float4 o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (uint32_t b0 = 0; b0 < Se; b0 += 8) {
            float4 v[8];
#pragma unroll
            for (uint32_t k = 0; k < 8; k++)
                v[k] = b0 + k < Se
                           ? __ldcg(reinterpret_cast<const float4*>(
                                        p.part + (base + (uint64_t)(b0 + k) * G + h) * HD) +
                                    d4)
                           : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
            for (uint32_t k = 0; k < 8; k++) {
                if (b0 + k >= Se) break;
                const float w = wts[h * Se + b0 + k];
                o.x = fmaf(v[k].x, w, o.x);
                o.y = fmaf(v[k].y, w, o.y);
                o.z = fmaf(v[k].z, w, o.z);
                o.w = fmaf(v[k].w, w, o.w);
            }
        }
        bf16* dst = p.o + (uint64_t)(kvh * G + h) * HD + d4 * 4;
        dst[0] = __float2bfloat16_rn(o.x * inv[h]);
        dst[1] = __float2bfloat16_rn(o.y * inv[h]);
        dst[2] = __float2bfloat16_rn(o.z * inv[h]);
        dst[3] = __float2bfloat16_rn(o.w * inv[h]);
    }
    if (tid == 0) p.tickets[kvh] = 0;
}

__device__ void ps_attention_any(const PsParams& p, const PsSmem& s, uint32_t l, uint32_t npos,
                                 bool staged) {
    if (p.hd == 128) ps_attention<128>(p, s, l, npos, staged);
    else if (p.hd == 64) ps_attention<64>(p, s, l, npos, staged);
    else ps_attention<32>(p, s, l, npos, staged);
}

// ---- the kernel ----------------------------------------------------------------------------
__global__ void __launch_bounds__(kPsThreads, 1) decode_step_kernel(const PsParams p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const PsSmem s = ps_smem(smem_raw);
    const uint32_t tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    if (tid == 0) {
        for (int i = 0; i < kPsSlots; i++) {
            mbar_init(smem_u32(&s.full[i]), 1);
            mbar_init(smem_u32(&s.empty[i]), 1);
        }
        s.misc[2] = 0;
        fence_barrier_init();
    }
    __syncthreads();
    const Step st = p.step[0];

    if (warp == kPsConsumers) {  // producer
        if (lane != 0) return;
        uint32_t g = 0;
        bool ok = true;
        for (uint32_t l = 0; l < p.L && ok; l++)
            for (uint32_t kind = kPhQkv; kind <= kPhDown && ok; kind++)
                ok = produce_phase(p, s, kind, l, g);
        if (ok) ok = produce_phase(p, s, kPhCls, 0, g);
        if (!ok) {
            // aborting: wait (bounded) for the copies still in flight into the ring
            for (uint32_t k = g > kPsSlots ? g - kPsSlots : 0; k < g; k++)
                mbar_wait_bounded(smem_u32(&s.full[k % kPsSlots]), (k / kPsSlots) & 1, p.flags);
        }
        return;
    }

    // consumers
    const uint32_t pos = st.position;
    const bool pos_ok = pos < p.seq;
    uint32_t tok = st.token;
    if (tok >= p.vocab_all) {
        if (tid == 0 && blockIdx.x == 0) atomicOr(p.flags, kFlagTokenRange);
        tok = 0;
    }
    if (!pos_ok && tid == 0 && blockIdx.x == 0) atomicOr(p.flags, kFlagPositionRange);
    const uint32_t npos = pos_ok ? pos + 1 : 0;
    uint32_t epoch = 0, g = 0;
    bool ok = true;
    PsBest best = {-INFINITY, 0xffffffffu};

    // embedding row (src/kernels.rs:35-47) into this CTA's slice of the residual stream
    {
        const uint32_t i0 = (uint32_t)((uint64_t)p.d * blockIdx.x / gridDim.x);
        const uint32_t i1 = (uint32_t)((uint64_t)p.d * (blockIdx.x + 1) / gridDim.x);
        for (uint32_t i = i0 + tid; i < i1; i += kPsConsumers * 32)
            p.x[i] = __bfloat162float(p.embed[(uint64_t)tok * p.d + i]);
    }
    // ok stays uniform over the CTA's consumer warps: every phase ends in a grid barrier
    ok = grid_barrier(p, s, epoch);
    const bool tp = p.world > 1;
    // tensor parallelism: all-reduce site k of this launch (wo of layer l is 2l, w2 is 2l + 1)
    const unsigned long long sites = tp ? p.launch[1] : 0ull;  // kXbSites follows kXbLaunch
    auto site_flag = [&](uint32_t k) { return (uint32_t)(sites + k + 1); };
    for (uint32_t l = 0; l < p.L && ok; l++) {
        const PsLayer& ly = p.layers[l];
        stage_norm(p, s, p.x, ly.rms_att);
        trace_staged(p, epoch);
        // this CTA's attention item's first tile (rows before pos) lands during the QKV phase
        const bool staged = attn_prestage_any(p, s, l, npos);
        ok = grid_barrier(p, s, epoch, consume_phase(p, s, kPhQkv, l, g, pos, pos_ok, &best));
        if (!ok) break;
        trace_staged(p, epoch);
        ps_attention_any(p, s, l, npos, staged);
        ok = grid_barrier(p, s, epoch);
        if (!ok) break;
        stage_copy(s, p.o, p.qd);
        trace_staged(p, epoch);
        if (tp) {
            const uint32_t f = site_flag(2 * l);
            bool mine = consume_phase(p, s, kPhWo, l, g, pos, pos_ok, &best, f);
            uint32_t u0, u1;
            cta_range(p.d / 2, &u0, &u1);
            if (p.trace && threadIdx.x == 0) trace_at(p, epoch, kTrSignal);
            mine = tp_site_reduce(p, s, 0, 2 * u0, 2 * u1, f, p.x, p.x2) && mine;
            ok = grid_barrier(p, s, epoch, mine);
            if (!ok) break;
            stage_norm(p, s, p.x2, ly.rms_ffn);
        } else {
            ok = grid_barrier(p, s, epoch, consume_phase(p, s, kPhWo, l, g, pos, pos_ok, &best));
            if (!ok) break;
            stage_norm(p, s, p.x, ly.rms_ffn);
        }
        trace_staged(p, epoch);
        ok = grid_barrier(p, s, epoch,
                          consume_phase(p, s, kPhGateUp, l, g, pos, pos_ok, &best));
        if (!ok) break;
        stage_copy(s, p.h, p.F);
        trace_staged(p, epoch);
        if (tp) {
            const uint32_t f = site_flag(2 * l + 1);
            bool mine = consume_phase(p, s, kPhDown, l, g, pos, pos_ok, &best, f);
            uint32_t u0, u1;
            cta_range(p.d, &u0, &u1);
            if (p.trace && threadIdx.x == 0) trace_at(p, epoch, kTrSignal);
            mine = tp_site_reduce(p, s, 1, u0, u1, f, p.x2, p.x) && mine;
            ok = grid_barrier(p, s, epoch, mine);
        } else {
            ok = grid_barrier(p, s, epoch,
                              consume_phase(p, s, kPhDown, l, g, pos, pos_ok, &best));
        }
    }
    cp_async_wait_all();  // an aborted layer may leave a prestaged tile in flight
    if (ok) {
        stage_norm(p, s, p.x, p.rms_final);
        if (!consume_phase(p, s, kPhCls, 0, g, pos, pos_ok, &best)) s.misc[2] = 1;
    }
    // the CTA's first maximum, then the last CTA keeps the first maximum of all CTAs
    if (lane == 0) {
        s.red[warp] = best.v;
        s.misc[8 + warp] = best.i;
    }
    consumers_sync();
    if (ok && s.misc[2] == 0 && tid == 0) {
        PsBest b = {-INFINITY, 0xffffffffu};
        for (int w = 0; w < kPsConsumers; w++) b = first_max2(b, PsBest{s.red[w], s.misc[8 + w]});
        p.cand_v[blockIdx.x] = b.v;
        p.cand_i[blockIdx.x] = b.i;
        __threadfence();
        if (atomicAdd(p.tickets + p.KV, 1u) == gridDim.x - 1) {
            __threadfence();
            PsBest a = {-INFINITY, 0xffffffffu};
            for (uint32_t c = 0; c < gridDim.x; c++)
                a = first_max2(a, PsBest{__ldcg(p.cand_v + c), __ldcg(p.cand_i + c)});
            bool merged = true;
            if (tp) {
                // every rank's best (value, id) into every rank's block as two flagged pairs
                // (this launch's flag: one past its last all-reduce site), then the first
                // maximum over the ranks in rank order: all ranks pick the same id
                const uint32_t f = site_flag(2 * p.L);
                for (uint32_t r = 0; r < p.world; r++) {
                    unsigned long long* c =
                        reinterpret_cast<unsigned long long*>(p.xb[r] + kXbCand) + 2 * p.rank;
                    asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(c),
                                 "l"(mk_pair(a.v, f)),
                                 "l"((unsigned long long)a.i | ((unsigned long long)f << 32))
                                 : "memory");
                }
                const unsigned long long* cand =
                    reinterpret_cast<const unsigned long long*>(p.xb[p.rank] + kXbCand);
                a = PsBest{-INFINITY, 0xffffffffu};
                for (uint32_t r = 0; merged && r < p.world; r++) {
                    unsigned long long v = ld_pair(cand + 2 * r), i = ld_pair(cand + 2 * r + 1);
                    WaitClock clock;
                    while ((uint32_t)(v >> 32) != f || (uint32_t)(i >> 32) != f) {
                        if (clock.expired(p.flags)) {
                            raise_abort(p);
                            merged = false;
                            break;
                        }
                        v = ld_pair(cand + 2 * r);
                        i = ld_pair(cand + 2 * r + 1);
                    }
                    a = first_max2(a, PsBest{__uint_as_float((uint32_t)v), (uint32_t)i});
                }
            }
            const int32_t id = a.i == 0xffffffffu ? 0 : (int32_t)a.i;
            p.argmax[0] = id;
            p.tickets[p.KV] = 0;
            if (p.feedback) {  // the next DecodeStep {argmax, position + 1}
                const uint32_t next = pos + 1;
                if (next >= p.seq) {
                    atomicOr(p.flags, kFlagPositionRange);
                } else {
                    p.history[next] = id;
                    p.step[0].token = (uint32_t)id;
                    p.step[0].position = next;
                }
            }
        }
    }
    // the last CTA to leave resets the barrier words (and, after an abort, the tickets that
    // CTAs which left early never drew) for the next launch
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(p.bar + 1, 1u) == gridDim.x - 1) {
            if (ld_relaxed(p.bar + 2))
                for (uint32_t k = 0; k <= p.KV; k++) p.tickets[k] = 0;
            if (tp) {
                p.launch[0] += 1;
                p.launch[1] += 2ull * p.L;
            }
            p.bar[0] = 0;
            p.bar[1] = 0;
            p.bar[2] = 0;
            __threadfence();
        }
    }
}

}  // namespace

// ---- host side -----------------------------------------------------------------------------
struct FusedStep {
    Runtime* rt = nullptr;
    PsParams p = {};
    void* scratch = nullptr;
    uint32_t grid = 0;
    uint32_t barriers = 0;  // grid barriers per launch (trace rows)
};

// Read at each model creation, so one process can build models of either kind.
bool fused_step_enabled() {
    const char* e = std::getenv("AMMON_B200_FUSED_STEP");
    return !(e && e[0] == '0');
}

// Test hook for the error path (AMMON_B200_TEST_STALL_BARRIER=n, read at model creation): CTA 0
// does not arrive at grid barrier n (1 = the first), so every other CTA's wait there runs out
// and the launch ends with kFlagWaitTimeout, as it would if a CTA stopped making progress.
static uint32_t env_stall_barrier() {
    if (const char* e = std::getenv("AMMON_B200_TEST_STALL_BARRIER")) {
        const long v = std::atol(e);
        if (v > 0) return (uint32_t)v;
    }
    return 0;
}

size_t fused_step_xblock_bytes(uint32_t world, uint32_t dim) {
    return kXbPart + 2ull * world * dim * sizeof(unsigned long long);
}

// Why the fused step cannot run this model ("" when it can).
std::string fused_step_unsupported(const FusedStepModel& m, int sms) {
    if (m.world > kTpMaxWorld) return "more than 8 ranks";
    if (m.batch != 1) return "batch is not 1";
    if (m.dtype != AB_BF16) return "weights are not bf16";
    const uint32_t qd = m.heads * m.head_dim, kvd = m.kv_heads * m.head_dim;
    if (m.head_dim != 32 && m.head_dim != 64 && m.head_dim != 128) return "head_dim not 32/64/128";
    if (m.kv_heads == 0 || m.heads % m.kv_heads || m.heads / m.kv_heads > kPsMaxG)
        return "query heads per kv head above 8";
    if (m.kv_heads > (uint32_t)sms) return "more kv heads than SMs";
    if (m.dim % 8 || qd % 8 || kvd % 8 || m.hidden % 8) return "dims not multiples of 8";
    if (m.dim % 2 || m.vocab % 2) return "odd dim or vocab";
    if (m.dim > 4096) return "dim above 4096 (the norm stages x and its gain in 24 KB)";
    if (m.world > 1 && m.dim % 4) return "dim not a multiple of 4";
    const uint64_t pair = 2ull * 2 * std::max(m.dim, qd);
    if (pair > kPsSlotBytes) return "a row pair exceeds the 32 KB ring slot";
    if ((uint64_t)m.hidden * 2 > kPsSlotBytes) return "a w2 row exceeds the 32 KB ring slot";
    if ((uint64_t)std::max({m.dim, qd, m.hidden}) * 2 > kPsActBytes)
        return "activation exceeds the 32 KB stage";
    return "";
}

FusedStep* fused_step_create(Runtime* rt, const FusedStepModel& m) {
    rt->activate();
    auto* f = new FusedStep();
    f->rt = rt;
    PsParams& p = f->p;
    const uint32_t G = m.heads / m.kv_heads;
    f->grid = (uint32_t)rt->sm_count;
    p.L = m.layers;
    p.d = m.dim;
    p.qd = m.heads * m.head_dim;
    p.kvd = m.kv_heads * m.head_dim;
    p.hd = m.head_dim;
    p.H = m.heads;
    p.KV = m.kv_heads;
    p.F = m.hidden;
    p.V = m.vocab;
    p.seq = m.seq;
    p.theta = m.rope_theta;
    p.eps = m.norm_eps;
    auto upc = [](uint32_t K) { return std::max(1u, std::min(2u, kPsSlotBytes / (2u * 2u * K))); };
    p.upc_qkv = upc(p.d);
    p.upc_wo = upc(p.qd);
    p.upc_gu = upc(p.d);
    p.upc_cls = upc(p.d);
    // w2 rows per chunk (tensor-parallel shards have short rows: several fill a slot)
    p.upc_down = std::max(1u, std::min(kPsMaxRows, kPsSlotBytes / (2u * p.F)));
    p.embed = (const bf16*)m.embed;
    p.wcls = (const bf16*)m.wcls;
    p.rms_final = (const bf16*)m.rms_final;
    p.step = (Step*)m.step;
    p.x = m.x;
    p.logits = m.logits;
    p.argmax = m.argmax;
    p.history = m.history;
    p.flags = rt->flags;
    p.world = m.world;
    p.rank = m.rank;
    p.vocab_off = m.rank * m.vocab;
    p.vocab_all = m.vocab * m.world;
    for (uint32_t r = 0; r < kTpMaxWorld; r++) p.xb[r] = r < m.world ? m.xblock[r] : nullptr;
    p.launch = m.world > 1 ? (unsigned long long*)(m.xblock[m.rank] + kXbLaunch) : nullptr;
    p.stall_barrier = env_stall_barrier();
    // one scratch allocation: layer table, q, o, h, attention partials, tickets, candidates,
    // barrier words, trace
    f->barriers = 1 + 5 * m.layers;
    const bool trace = std::getenv("AMMON_B200_STEP_TRACE") != nullptr;
    auto al = [](size_t n) { return (n + 255) / 256 * 256; };
    const size_t b_layers = al(sizeof(PsLayer) * m.layers);
    const size_t b_q = al(4ull * p.qd), b_o = al(2ull * p.qd), b_h = al(2ull * p.F);
    const size_t b_x2 = m.world > 1 ? al(4ull * p.d) : 0;
    const size_t b_part = al(4ull * p.KV * f->grid * G * p.hd);
    p.ml_stride = (f->grid * G * 2 + 3) / 4 * 4;
    const size_t b_ml = al(4ull * p.KV * p.ml_stride);
    const size_t b_tk = al(4ull * (p.KV + 1));
    const size_t b_cand = al(8ull * f->grid);
    const size_t b_bar = 256;
    const size_t b_trace = trace ? al(8ull * kTrCols * f->barriers * f->grid) : 0;
    const size_t total =
        b_layers + b_q + b_o + b_h + b_x2 + b_part + b_ml + b_tk + b_cand + b_bar + b_trace;
    try {
        cuda_check(cudaMalloc(&f->scratch, total), "fused step scratch");
        cuda_check(cudaMemset(f->scratch, 0, total), "fused step scratch");
        char* c = (char*)f->scratch;
        PsLayer* layers = (PsLayer*)c;
        c += b_layers;
        p.layers = layers;
        p.q = (float*)c;
        c += b_q;
        p.o = (bf16*)c;
        c += b_o;
        p.h = (bf16*)c;
        c += b_h;
        p.x2 = b_x2 ? (float*)c : nullptr;
        c += b_x2;
        p.part = (float*)c;
        c += b_part;
        p.part_ml = (float*)c;
        c += b_ml;
        p.tickets = (uint32_t*)c;
        c += b_tk;
        p.cand_v = (float*)c;
        p.cand_i = (uint32_t*)(c + 4ull * f->grid);
        c += b_cand;
        p.bar = (uint32_t*)c;
        c += b_bar;
        p.trace = trace ? (uint64_t*)c : nullptr;
        std::vector<PsLayer> host(m.layers);
        for (uint32_t l = 0; l < m.layers; l++) {
            PsLayer& ly = host[l];
            ly.wq = (const bf16*)m.wq[l];
            ly.wk = (const bf16*)m.wk[l];
            ly.wv = (const bf16*)m.wv[l];
            ly.wo = (const bf16*)m.wo[l];
            ly.w1 = (const bf16*)m.w1[l];
            ly.w3 = (const bf16*)m.w3[l];
            ly.w2 = (const bf16*)m.w2[l];
            ly.rms_att = (const bf16*)m.rms_att[l];
            ly.rms_ffn = (const bf16*)m.rms_ffn[l];
            ly.kcache = (bf16*)m.kcache[l];
            ly.vcache = (bf16*)m.vcache[l];
        }
        cuda_check(cudaMemcpy(layers, host.data(), sizeof(PsLayer) * m.layers,
                              cudaMemcpyHostToDevice),
                   "fused step layer table");
        cuda_check(cudaFuncSetAttribute(decode_step_kernel,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)kPsSmem),
                   "fused step shared memory");
        int per_sm = 0;
        cuda_check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_step_kernel,
                                                                 kPsThreads, kPsSmem),
                   "fused step occupancy");
        if (per_sm < 1) fail(AB_ERR_CUDA, "fused step: one CTA per SM does not fit");
    } catch (...) {
        fused_step_destroy(f);
        throw;
    }
    return f;
}

void fused_step_destroy(FusedStep* f) {
    if (!f) return;
    if (f->scratch) cudaFree(f->scratch);
    delete f;
}

void record_fused_step(ab_scheme* s, FusedStep* f, bool feedback) {
    // (the tensor-parallel step() scheme adds the logits all-gather after this node)
    PsParams p = f->p;
    p.feedback = feedback ? 1u : 0u;
    const uint32_t grid = f->grid;
    // one cooperative launch per step: launched directly on each submit, no graph around it
    s->use_graph = false;
    s->add("decode_step", [=](cudaStream_t st) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(grid);
        cfg.blockDim = dim3(kPsThreads);
        cfg.dynamicSmemBytes = kPsSmem;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeCooperative;
        attr[0].val.cooperative = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, decode_step_kernel, p);
    });
}

// Per-barrier times of the last launch (AMMON_B200_STEP_TRACE set): [barriers][4][grid]
// nanoseconds of %globaltimer -- arrival, release, when the CTA had staged the operand of the
// phase that ends at that barrier, and (the barriers after an all-reduce site) when it had
// pushed its partial rows and began to wait for the other ranks'; false when tracing is off.
bool fused_step_trace(FusedStep* f, std::vector<uint64_t>* out, uint32_t* barriers,
                      uint32_t* grid) {
    if (!f || !f->p.trace) return false;
    out->resize((size_t)kTrCols * f->barriers * f->grid);
    cuda_check(cudaMemcpy(out->data(), f->p.trace, out->size() * 8, cudaMemcpyDeviceToHost),
               "fused step trace");
    *barriers = f->barriers;
    *grid = f->grid;
    return true;
}

}  // namespace ab
