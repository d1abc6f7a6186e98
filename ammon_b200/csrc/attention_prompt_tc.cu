// Prompt attention on the 5th-generation tensor cores: the rows of a batched prefill pass are
// consecutive positions of one stream over one shared [seq, kv_heads, head] cache, so every
// K/V tile serves every query row of a kv head (src/kernels.rs:228-410 semantics: scores
// q.k / sqrt(head), causal softmax over positions 0..pos, weighted V sum; the reference feeds
// a prompt one token per step, src/generate.rs:60-66, and this is the batched replacement).
//
// One CTA takes 128 query rows of kv head blockIdx.y -- 128 / G consecutive batch rows times
// the G query heads of the group -- one row per TMEM lane:
//  - warp 4 (one thread) streams 64-position K and V tiles with TMA (128-byte swizzle) into a
//    ring guarded by full/empty mbarriers;
//  - warp 5 (one thread) issues tcgen05.mma (kind::f16, f32 accumulate): S = Q.K^T into one of
//    two 64-column TMEM buffers (the next tile's scores are computed while the softmax warps
//    work on the current one), and O += P.V into a 128-column TMEM accumulator with V as an
//    MN-major operand straight from its TMA tile;
//  - warps 0-3 (thread = row = TMEM lane) stage Q, then per tile read S with tcgen05.ld, apply
//    the row's causal limit, keep the running max and sum, write P to shared memory as the A
//    operand of the next P.V, and rescale O in TMEM (tcgen05.ld/st) only when the row's max
//    grew by more than kPtRescale since the reference it was last scaled to (exact either way:
//    P and the sum use the same reference; scores in base 2, exp2f); at the end they read O,
//    divide by the sum and store the row.
// Q is fp32 and P carries values up to e^kPtRescale, so both go to the tensor core as bf16
// high + low pairs (two MMAs each), keeping the scores and the weighted sums near fp32
// precision; K and V are the bf16 cache itself.
// Every wait is bounded; a wait that runs out raises the device flag, the CTA drains its
// copies and MMAs and still frees its TMEM.
#include <cuda_bf16.h>

#include "common.cuh"
#include "internal.h"
#include "ops.h"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace ab {

namespace {

constexpr uint32_t kPtRows = 128;      // query rows per CTA (TMEM lanes)
constexpr uint32_t kPtTile = 64;       // positions per K/V tile
constexpr uint32_t kPtSoftmax = 256;   // softmax threads: two per row (warps 0-7)
constexpr uint32_t kPtThreads = 352;   // + the K TMA warp 8, the MMA warp 9, the V TMA warp 10
constexpr uint32_t kPtTmemCols = 256;  // S buffers at columns 0 and 64, O from column 128
// Scores are kept in base 2 (Q is pre-scaled by log2(e) / sqrt(head)), so P = 2^(s - m) is
// e^(score - max) exactly as the softmax defines it; O is rescaled when a row's max grows by
// more than kPtRescale (in base-2 units: P stays below 2^kPtRescale).
constexpr float kPtLog2e = 1.4426950408889634f;
constexpr float kPtRescale = 11.5f;

// K and V tiles stream through separate rings: a K tile is free once its scores are computed,
// long before the P.V that frees its V tile, so the next K tiles never wait behind a softmax.
template <int HD>
struct AttnPtLayout {
    static constexpr uint32_t kQBytes = kPtRows * HD * 2;        // Q hi, then Q lo
    static constexpr uint32_t kPBytes = kPtRows * kPtTile * 2;   // P hi, then P lo (16 KB)
    static constexpr uint32_t kTile = kPtTile * HD * 2;          // one K or V tile
    // a K tile is needed one tile ahead of its V tile and freed a softmax earlier: V gets the
    // deeper ring
    static constexpr uint32_t kKStages = HD == 128 ? 2 : 4;
    static constexpr uint32_t kVStages = HD == 128 ? 3 : 4;
    static constexpr uint32_t kQOff = 0;
    static constexpr uint32_t kPOff = 2 * kQBytes;               // [2 buffers][hi, lo]
    static constexpr uint32_t kKOff = kPOff + 4 * kPBytes;
    static constexpr uint32_t kVOff = kKOff + kKStages * kTile;
    static constexpr uint32_t kRedOff = kVOff + kVStages * kTile;   // [6][128] f32
    static constexpr size_t smem() { return (size_t)kRedOff + 6 * kPtRows * 4 + 1024; }
};

// Byte offset of 16-byte chunk c (0..7) of row r in a K-major 128-byte-swizzled operand block
// of 128 rows (8-row groups 1024 bytes apart): the CU_TENSOR_MAP_SWIZZLE_128B pattern.
__device__ __forceinline__ uint32_t sw_row_chunk(uint32_t r, uint32_t c) {
    return (r / 8) * 1024 + (r % 8) * 128 + ((c ^ (r % 8)) * 16);
}

// Two floats as a bf16 pair (first in the low half) and the pair of what rounding left.
__device__ __forceinline__ void pt_split(float a, float b, uint32_t* hi, uint32_t* lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    const float2 hf = __bfloat1622float2(h);
    const __nv_bfloat162 l = __floats2bfloat162_rn(a - hf.x, b - hf.y);
    *hi = *reinterpret_cast<const uint32_t*>(&h);
    *lo = *reinterpret_cast<const uint32_t*>(&l);
}

__device__ __forceinline__ void st_shared16(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                            uint32_t d) {
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
                 "r"(d)
                 : "memory");
}

// Named barrier 1 of the 256 softmax threads that also ANDs a predicate over them: every
// softmax thread takes the same barriers, and a failed wait anywhere stops all of them together.
__device__ __forceinline__ bool softmax_sync_and(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\t"
        "bar.red.and.pred p, 1, %2, q;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(kPtSoftmax)
        : "memory");
    return r != 0;
}

template <typename OT>
__device__ __forceinline__ void pt_store16(OT* dst, const float* v, float scale);
template <>
__device__ __forceinline__ void pt_store16<float>(float* dst, const float* v, float scale) {
#pragma unroll
    for (int k = 0; k < 16; k += 4)
        *reinterpret_cast<float4*>(dst + k) =
            make_float4(v[k] * scale, v[k + 1] * scale, v[k + 2] * scale, v[k + 3] * scale);
}
template <>
__device__ __forceinline__ void pt_store16<bf16>(bf16* dst, const float* v, float scale) {
    uint32_t w[8];
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * k] * scale, v[2 * k + 1] * scale);
        w[k] = *reinterpret_cast<const uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
    *reinterpret_cast<uint4*>(dst + 8) = make_uint4(w[4], w[5], w[6], w[7]);
}

template <typename OT, int G, int HD>
__global__ void __launch_bounds__(kPtThreads, 1)
    attn_prompt_tc_kernel(const AttnParams p, const __grid_constant__ CUtensorMap kmap,
                          const __grid_constant__ CUtensorMap vmap) {
    using LY = AttnPtLayout<HD>;
    constexpr uint32_t SK = LY::kKStages, SV = LY::kVStages;
    constexpr uint32_t NBOX = HD / 64;     // 64-dimension boxes of a K or V row
    constexpr uint32_t QP = kPtRows / G;   // batch rows per CTA
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t k_full[SK], k_empty[SK], v_full[SV], v_empty[SV];
    __shared__ __align__(8) uint64_t s_full[2], s_free[2], p_full[2], pv_done[2], done_bar;
    __shared__ uint32_t sm_tmem, sm_end;
    __shared__ int sm_fail, sm_last;
    unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    const uint32_t kvh = blockIdx.y, b0 = blockIdx.x * QP;

    pdl_wait();
    if (tid == 0) {
        uint32_t e = 0;
        for (uint32_t j = 0; j < QP && b0 + j < p.batch; j++) {
            const uint32_t pos = p.step[b0 + j].position;
            if (pos < p.seq) e = max(e, pos + 1);
        }
        sm_end = e;
        for (uint32_t i = 0; i < SK; i++) {
            mbar_init(smem_u32(&k_full[i]), 1);
            mbar_init(smem_u32(&k_empty[i]), 1);
        }
        for (uint32_t i = 0; i < SV; i++) {
            mbar_init(smem_u32(&v_full[i]), 1);
            mbar_init(smem_u32(&v_empty[i]), 1);
        }
        for (uint32_t i = 0; i < 2; i++) {
            mbar_init(smem_u32(&s_full[i]), 1);
            mbar_init(smem_u32(&s_free[i]), kPtSoftmax);
            mbar_init(smem_u32(&p_full[i]), kPtSoftmax);
            mbar_init(smem_u32(&pv_done[i]), 1);
        }
        mbar_init(smem_u32(&done_bar), 1);
        fence_barrier_init();
        sm_fail = 0;
    }
    if (warp == 0) tmem_alloc(smem_u32(&sm_tmem), kPtTmemCols);

    // row r = tid (warps 0-3): batch row b0 + r / G, query head kvh * G + r % G
    int32_t lim = -1;  // last visible position (-1: no query)
    uint64_t orow = 0;
    const float* q = nullptr;
    if (tid < kPtSoftmax) {  // both softmax threads of a row need its limit and output row
        const uint32_t r = tid % kPtRows, b = b0 + r / G;
        if (b < p.batch) {
            const uint32_t pos = p.step[b].position;
            if (pos < p.seq) {
                lim = (int32_t)pos;
                orow = (uint64_t)b * p.heads + (uint64_t)kvh * G + r % G;
                q = p.q + orow * HD;
            }
        }
    }
    if (tid < kPtRows) {
        // Q (pre-scaled) as the K-major A operand, bf16 high and low parts
        const float qs = kPtLog2e / sqrtf((float)HD);
#pragma unroll
        for (uint32_t kb = 0; kb < NBOX; kb++) {
#pragma unroll
            for (uint32_t c = 0; c < 8; c++) {
                float v[8];
                if (q) {
                    const float4 a = *reinterpret_cast<const float4*>(q + kb * 64 + c * 8);
                    const float4 d = *reinterpret_cast<const float4*>(q + kb * 64 + c * 8 + 4);
                    v[0] = a.x * qs; v[1] = a.y * qs; v[2] = a.z * qs; v[3] = a.w * qs;
                    v[4] = d.x * qs; v[5] = d.y * qs; v[6] = d.z * qs; v[7] = d.w * qs;
                } else {
#pragma unroll
                    for (int k = 0; k < 8; k++) v[k] = 0.0f;
                }
                uint32_t hi[4], lo[4];
#pragma unroll
                for (int k = 0; k < 4; k++) pt_split(v[2 * k], v[2 * k + 1], &hi[k], &lo[k]);
                const uint32_t off = LY::kQOff + kb * (kPtRows * 128) + sw_row_chunk(tid, c);
                st_shared16(sbase + off, hi[0], hi[1], hi[2], hi[3]);
                st_shared16(sbase + off + LY::kQBytes, lo[0], lo[1], lo[2], lo[3]);
            }
        }
        fence_proxy_async_smem();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm_tmem;
    // gridDim.z CTAs (1 or 2) split the row block's tiles: this one takes [t_lo, t_lo + ntiles)
    const uint32_t halves = gridDim.z, nt_all = (sm_end + kPtTile - 1) / kPtTile;
    const uint32_t h_tiles = (nt_all + halves - 1) / halves;
    const uint32_t t_lo = min(nt_all, blockIdx.z * h_tiles);
    const uint32_t ntiles = min(nt_all, t_lo + h_tiles) - t_lo;
    float m_ref = -INFINITY, l = 0.0f;        // softmax rows: running max (base 2) and sum
    const uint32_t lane_base = (warp * 32u) << 16;

    if (warp == 8 || warp == 10) {
        // ---- TMA: warp 8 streams the K tiles, warp 10 the V tiles (64 positions each) ----
        if (lane == 0) {
            const bool kside = warp == 8;
            const uint32_t S = kside ? SK : SV;
            uint64_t* full = kside ? k_full : v_full;
            uint64_t* empty = kside ? k_empty : v_empty;
            const CUtensorMap* map = kside ? &kmap : &vmap;
            const uint32_t ring = sbase + (kside ? LY::kKOff : LY::kVOff);
            uint32_t issued = 0;
            for (uint32_t i = 0; i < ntiles; i++) {
                const uint32_t s = i % S;
                if (i >= S &&
                    !mbar_wait_bounded(smem_u32(&empty[s]), ((i - S) / S) & 1, p.flags)) {
                    sm_fail = 1;
                    break;
                }
                if (*(volatile int*)&sm_fail) break;
                const uint32_t bar = smem_u32(&full[s]);
                mbar_arrive_expect_tx(bar, LY::kTile);
#pragma unroll
                for (uint32_t j = 0; j < NBOX; j++) {
                    // whole tiles: rows past seq read the zero fill, rows past a query's
                    // position are masked by its causal limit
                    const int32_t x = (int32_t)(kvh * HD + j * 64);
                    const int32_t y = (int32_t)((t_lo + i) * kPtTile);
                    tma_load_2d(ring + s * LY::kTile + j * kPtTile * 128, map, x, y, bar);
                }
                issued++;
            }
            // the copies still in flight land before the CTA can leave
            for (uint32_t j = issued > S ? issued - S : 0; j < issued; j++)
                mbar_wait_bounded(smem_u32(&full[j % S]), (j / S) & 1, p.flags);
        }
    } else if (warp == 9) {
        // ---- MMA: S(i + 1) = Q.K^T ahead of O += P(i).V ----
        if (lane == 0 && ntiles > 0) {
            const uint32_t idesc_s = tc_idesc_bf16(kPtRows, kPtTile);
            const uint32_t idesc_o = tc_idesc_bf16(kPtRows, HD) | kIdescBMajorMN;
            const uint32_t qhi = sbase + LY::kQOff, qlo = qhi + LY::kQBytes;
            auto issue_s = [&](uint32_t i) {
                const uint32_t s = i % SK;
                if (!mbar_wait_bounded(smem_u32(&k_full[s]), (i / SK) & 1, p.flags)) return false;
                // the softmax warps have read this S buffer's previous tile
                if (i >= 2 &&
                    !mbar_wait_bounded(smem_u32(&s_free[i % 2]), ((i - 2) / 2) & 1, p.flags))
                    return false;
                tc_fence_after();
                const uint32_t kst = sbase + LY::kKOff + s * LY::kTile;
                const uint32_t d = tmem + (i % 2) * kPtTile;
#pragma unroll
                for (uint32_t kb = 0; kb < NBOX; kb++) {
                    const uint64_t dh = sw128_desc(qhi + kb * kPtRows * 128);
                    const uint64_t dl = sw128_desc(qlo + kb * kPtRows * 128);
                    const uint64_t dk = sw128_desc(kst + kb * kPtTile * 128);
#pragma unroll
                    for (uint32_t k = 0; k < 4; k++)
                        tc_mma_bf16(d, dh + 2 * k, dk + 2 * k, idesc_s, (kb | k) != 0);
#pragma unroll
                    for (uint32_t k = 0; k < 4; k++) tc_mma_bf16(d, dl + 2 * k, dk + 2 * k, idesc_s, 1);
                }
                tc_commit(smem_u32(&s_full[i % 2]));
                tc_commit(smem_u32(&k_empty[s]));  // the K tile is free once S is computed
                return true;
            };
            bool ok = issue_s(0);
            for (uint32_t i = 0; i < ntiles && ok; i++) {
                if (i + 1 < ntiles && !issue_s(i + 1)) {
                    ok = false;
                    break;
                }
                if (!mbar_wait_bounded(smem_u32(&v_full[i % SV]), (i / SV) & 1, p.flags) ||
                    !mbar_wait_bounded(smem_u32(&p_full[i % 2]), (i / 2) & 1, p.flags)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t pb = sbase + LY::kPOff + (i % 2) * 2 * LY::kPBytes;
                const uint32_t vst = sbase + LY::kVOff + (i % SV) * LY::kTile;
                const uint64_t ph = sw128_desc(pb), pl = sw128_desc(pb + LY::kPBytes);
#pragma unroll
                for (uint32_t k = 0; k < kPtTile / 16; k++) {
                    // V rows 16k .. 16k + 15 (two 8-row groups), every head dimension
                    const uint64_t dv = sw128_desc_mn(vst + k * 16 * 128, kPtTile * 128);
                    tc_mma_bf16(tmem + 128, ph + 2 * k, dv, idesc_o, (i | k) != 0);
                    tc_mma_bf16(tmem + 128, pl + 2 * k, dv, idesc_o, 1);
                }
                tc_commit(smem_u32(&pv_done[i % 2]));
                tc_commit(smem_u32(&v_empty[i % SV]));
            }
            if (!ok) sm_fail = 1;
        }
        if (lane == 0) tc_commit(smem_u32(&done_bar));  // every MMA this thread issued
    } else if (warp < 8) {
        // ---- softmax: two threads per query row (TMEM lane = row); half 0 (warps 0-3) owns
        // score columns 0-31 and O columns [0, HD/2), half 1 (warps 4-7) the rest ----
        const uint32_t row = tid % kPtRows, hf = tid / kPtRows;
        float* red = reinterpret_cast<float*>(smem + LY::kRedOff);  // [2 tiles][2 halves][128]
        bool ok = true, failed = false;
        float lh = 0.0f;  // this half's part of the row sum
        for (uint32_t i = 0; i < ntiles; i++) {
            // every wait happens before the tile's barrier, which ANDs the outcomes: the
            // softmax threads leave together (and the warps stay converged for tcgen05.ld/st)
            bool w = mbar_wait_bounded(smem_u32(&s_full[i % 2]), (i / 2) & 1, p.flags);
            // this tile's P buffer is free once P.V of tile i - 2 finished
            if (i >= 2)
                w = mbar_wait_bounded(smem_u32(&pv_done[i % 2]), ((i - 2) / 2) & 1, p.flags) &&
                    w;
            tc_fence_after();
            float sv[kPtTile / 2];
#pragma unroll
            for (uint32_t c = 0; c < kPtTile / 32; c++)
                tmem_ld16(tmem + lane_base + (i % 2) * kPtTile + hf * 32 + 16 * c, sv + 16 * c);
            tc_fence_before();
            mbar_arrive(smem_u32(&s_free[i % 2]));
            const int32_t t0 = (int32_t)((t_lo + i) * kPtTile + hf * 32);
            // only a tile that reaches past the row's position needs the causal mask
            if (t0 + (int32_t)(kPtTile / 2) - 1 > lim) {
#pragma unroll
                for (uint32_t j = 0; j < kPtTile / 2; j++)
                    if (t0 + (int32_t)j > lim) sv[j] = -INFINITY;
            }
            float pmx = sv[0];
#pragma unroll
            for (uint32_t j = 1; j < kPtTile / 2; j++) pmx = fmaxf(pmx, sv[j]);
            red[((i & 1) * 2 + hf) * kPtRows + row] = pmx;
            ok = softmax_sync_and(w && !failed);
            if (!ok) break;
            const float mx = fmaxf(pmx, red[((i & 1) * 2 + (hf ^ 1)) * kPtRows + row]);
            float alpha = 1.0f;
            bool rescale = false;
            if (mx != -INFINITY && (m_ref == -INFINITY || mx > m_ref + kPtRescale)) {
                if (m_ref != -INFINITY) {
                    alpha = exp2f(m_ref - mx);
                    rescale = true;
                }
                m_ref = mx;
            }
            float sum = 0.0f;
            if (m_ref == -INFINITY) {  // nothing visible yet: P = 0
#pragma unroll
                for (uint32_t j = 0; j < kPtTile / 2; j++) sv[j] = 0.0f;
            } else {
#pragma unroll
                for (uint32_t j = 0; j < kPtTile / 2; j++) {
                    sv[j] = exp2f(sv[j] - m_ref);  // a masked score (-inf) gives 0
                    sum += sv[j];
                }
            }
            lh = lh * alpha + sum;
            // O holds every earlier tile's P.V before it is scaled: the rare tile that rescales
            // waits for P.V of tile i - 1 (a warp whose wait runs out skips the scaling and
            // fails the launch at the next barrier, so no softmax thread is left behind)
            bool scale = __any_sync(0xffffffffu, rescale);
            if (scale && i >= 1) {
                scale = __all_sync(0xffffffffu,
                                   mbar_wait_bounded(smem_u32(&pv_done[(i - 1) % 2]),
                                                     ((i - 1) / 2) & 1, p.flags));
                failed |= !scale;
                tc_fence_after();
            }
            if (scale) {
                // this half's O columns (alpha = 1 for rows that keep their reference)
#pragma unroll
                for (uint32_t c = 0; c < HD / 32; c++) {
                    float o[16];
                    const uint32_t col = 128 + hf * (HD / 2) + 16 * c;
                    tmem_ld16(tmem + lane_base + col, o);
#pragma unroll
                    for (int k = 0; k < 16; k++) o[k] *= alpha;
                    tmem_st16(tmem + lane_base + col, o);
                }
                tmem_wait_st();
            }
            // this half's P columns (bf16 high and low parts) as the K-major A operand
            const uint32_t pb = sbase + LY::kPOff + (i % 2) * 2 * LY::kPBytes;
#pragma unroll
            for (uint32_t c = 0; c < kPtTile / 16; c++) {
                uint32_t hi[4], lo[4];
#pragma unroll
                for (int k = 0; k < 4; k++)
                    pt_split(sv[8 * c + 2 * k], sv[8 * c + 2 * k + 1], &hi[k], &lo[k]);
                const uint32_t off = sw_row_chunk(row, hf * (kPtTile / 16) + c);
                st_shared16(pb + off, hi[0], hi[1], hi[2], hi[3]);
                st_shared16(pb + LY::kPBytes + off, lo[0], lo[1], lo[2], lo[3]);
            }
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(smem_u32(&p_full[i % 2]));
        }
        // the row sum from both halves; the last tile's P.V
        bool w = true;
        if (ok && ntiles > 0) {
            const uint32_t last = ntiles - 1;
            w = mbar_wait_bounded(smem_u32(&pv_done[last % 2]), (last / 2) & 1, p.flags);
        }
        red[(4 + hf) * kPtRows + row] = lh;
        ok = softmax_sync_and(ok && w && !failed);
        l = red[4 * kPtRows + row] + red[5 * kPtRows + row];
        if (ok) tc_fence_after();
        const uint32_t c0 = hf * (HD / 32);  // this half's 16-column chunks of O
        if (ok && halves == 1 && ntiles > 0) {
            const float inv = (lim >= 0 && l > 0.0f) ? 1.0f / l : 0.0f;
            OT* dst = (OT*)p.out + orow * HD;
#pragma unroll
            for (uint32_t c = c0; c < c0 + HD / 32; c++) {
                float o[16];
                tmem_ld16(tmem + lane_base + 128 + 16 * c, o);
                if (lim >= 0) pt_store16<OT>(dst + 16 * c, o, inv);
            }
        } else if (ok && halves > 1) {
            // this half's partial (O relative to its reference m_ref, m_ref, l) for the merge
            float* po = p.part_o + (orow * halves + blockIdx.z) * HD;
            float* pm = p.part_o + (uint64_t)p.batch * p.heads * halves * HD +
                        (orow * halves + blockIdx.z) * 2;
#pragma unroll
            for (uint32_t c = c0; c < c0 + HD / 32; c++) {
                float o[16];
                if (ntiles > 0) {
                    tmem_ld16(tmem + lane_base + 128 + 16 * c, o);
                } else {
#pragma unroll
                    for (int k = 0; k < 16; k++) o[k] = 0.0f;
                }
                if (lim >= 0) pt_store16<float>(po + 16 * c, o, 1.0f);
            }
            if (lim >= 0 && hf == 0) {
                pm[0] = m_ref;
                pm[1] = l;
            }
            __threadfence();
        }
        if (!ok) sm_fail = 1;
    }
    __syncthreads();
    if (halves > 1) {
        // the second CTA of the row block to finish merges both halves
        if (tid == 0) {
            int last = 0;
            if (!sm_fail) {
                __threadfence();
                last = atomicAdd(p.counters + blockIdx.x * p.kv_heads + kvh, 1u) == halves - 1;
            }
            sm_last = last;
        }
        __syncthreads();
        if (sm_last && warp < 8) {
            __threadfence();
            const uint32_t other = blockIdx.z ^ 1;
            const float* po = p.part_o + (orow * halves + other) * HD;
            const float* pm = p.part_o + (uint64_t)p.batch * p.heads * halves * HD +
                              (orow * halves + other) * 2;
            float m2 = -INFINITY, l2 = 0.0f;
            if (lim >= 0) {
                m2 = __ldcg(pm);
                l2 = __ldcg(pm + 1);
            }
            const float m = fmaxf(m_ref, m2);
            const float w1 = m_ref == -INFINITY ? 0.0f : exp2f(m_ref - m);
            const float w2 = m2 == -INFINITY ? 0.0f : exp2f(m2 - m);
            const float lt = l * w1 + l2 * w2;
            const float inv = (lim >= 0 && lt > 0.0f) ? 1.0f / lt : 0.0f;
            OT* dst = (OT*)p.out + orow * HD;
            const uint32_t c0 = (tid / kPtRows) * (HD / 32);  // this half's chunks of O
#pragma unroll
            for (uint32_t c = c0; c < c0 + HD / 32; c++) {
                float o[16];
                if (ntiles > 0) {
                    tmem_ld16(tmem + lane_base + 128 + 16 * c, o);
                } else {
#pragma unroll
                    for (int k = 0; k < 16; k++) o[k] = 0.0f;
                }
                if (lim >= 0) {
#pragma unroll
                    for (int k = 0; k < 16; k += 4) {
                        const float4 b = __ldcg(reinterpret_cast<const float4*>(po + 16 * c + k));
                        o[k] = o[k] * w1 + b.x * w2;
                        o[k + 1] = o[k + 1] * w1 + b.y * w2;
                        o[k + 2] = o[k + 2] * w1 + b.z * w2;
                        o[k + 3] = o[k + 3] * w1 + b.w * w2;
                    }
                    pt_store16<OT>(dst + 16 * c, o, inv);
                }
            }
        }
        if (sm_last && tid == 0) p.counters[blockIdx.x * p.kv_heads + kvh] = 0;
        __syncthreads();
    }
    if (warp == 0) {
        if (sm_fail && lane == 0) atomicOr(p.flags, kFlagWaitTimeout);
        // every MMA has completed before the TMEM goes back
        mbar_wait_bounded(smem_u32(&done_bar), 0, p.flags);
        tc_fence_after();
        tmem_dealloc(tmem, kPtTmemCols);
    }
    pdl_trigger();
}

cudaError_t pt_set_smem(const void* kern, size_t smem) {
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
}

template <typename OT, int G, int HD>
void pt_add(ab_scheme* s, const char* label, const AttnParams& p, const CUtensorMap& kmap,
            const CUtensorMap& vmap) {
    auto kern = attn_prompt_tc_kernel<OT, G, HD>;
    const size_t smem = AttnPtLayout<HD>::smem();
    const uint32_t qp = kPtRows / G;
    // two CTAs per row block (each half of the positions, merged by the second to finish)
    // when the block's split scratch can hold the halves' partials
    const uint64_t need = (uint64_t)p.batch * p.heads * 2 * (HD + 2);
    const uint32_t halves = (p.part_o && p.counters && p.part_cap >= need) ? 2 : 1;
    const dim3 grid((p.batch + qp - 1) / qp, p.kv_heads, halves);
    s->add(label, [=](cudaStream_t st) {
        cudaError_t e = pt_set_smem((const void*)kern, smem);
        if (e != cudaSuccess) return e;
        return launch(st, grid, dim3(kPtThreads), smem, true, kern, p, kmap, vmap);
    });
}

template <typename OT, int G>
void pt_add_hd(ab_scheme* s, const char* label, const AttnParams& p, const CUtensorMap& kmap,
               const CUtensorMap& vmap) {
    if (p.head == 128) pt_add<OT, G, 128>(s, label, p, kmap, vmap);
    else pt_add<OT, G, 64>(s, label, p, kmap, vmap);
}

template <typename OT>
bool pt_add_g(ab_scheme* s, const char* label, const AttnParams& p, const CUtensorMap& kmap,
              const CUtensorMap& vmap) {
    switch (p.heads / p.kv_heads) {
        case 1: pt_add_hd<OT, 1>(s, label, p, kmap, vmap); return true;
        case 2: pt_add_hd<OT, 2>(s, label, p, kmap, vmap); return true;
        case 4: pt_add_hd<OT, 4>(s, label, p, kmap, vmap); return true;
        case 8: pt_add_hd<OT, 8>(s, label, p, kmap, vmap); return true;
        default: return false;
    }
}

}  // namespace

// Records the prompt attention of a pass whose rows share one bf16 cache (cache_rows == 0)
// with head 64 or 128; false when the shape is not one this kernel takes.
bool record_prompt_attention_tc(ab_scheme* s, const char* label, const AttnParams& p) {
    if (p.kv_dtype != AB_BF16 || (p.head != 64 && p.head != 128) || p.cache_rows != 0)
        return false;
    CUtensorMap kmap, vmap;
    const uint64_t inner = (uint64_t)p.kv_heads * p.head;
    encode_tmap_2d(&kmap, AB_BF16, p.kcache, inner, p.seq, inner * 2, 64, kPtTile, 128);
    encode_tmap_2d(&vmap, AB_BF16, p.vcache, inner, p.seq, inner * 2, 64, kPtTile, 128);
    if (p.out_dtype == AB_BF16) return pt_add_g<bf16>(s, label, p, kmap, vmap);
    return pt_add_g<float>(s, label, p, kmap, vmap);
}

}  // namespace ab
