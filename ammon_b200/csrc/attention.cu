// Fused flash-decoding attention for the block path, replacing the reference's
// attention_partial + attention_combine pair (src/kernels.rs:228-410).
//
// Design (B200):
//  - Grid (splits, kv_heads, batch). One CTA serves every query head of its GQA group
//    from one staged K/V tile, so K/V bytes are read once per kv head rather than once
//    per query head.
//  - K/V tiles of 64 positions are staged in shared memory by TMA (2-D tensor maps over
//    the cache, CTA-local copies), double-buffered on mbarriers, in the 32/64/128-byte
//    swizzle that lets row-parallel lanes read distinct banks. Head sizes TMA cannot tile
//    use the same algorithm with plain 16-byte loads into padded rows.
//  - The position range [0, pos] is cut into `nsplit` chunks (multiples of the 64-row
//    tile) computed on the device from the step's position, so a graph recorded once
//    serves every position. Only the splits that hold positions do work.
//  - Scores, the online softmax (running max m, sum l) and the P.V accumulation happen
//    in one pass over each tile.
//  - The last active CTA of a (batch, kv head) to finish (atomic ticket) folds the
//    partials in split order and writes the output, so no second kernel runs; it resets
//    the ticket for the next replay.
#include <algorithm>
#include <mutex>
#include <string>

#include "common.cuh"
#include "internal.h"
#include "ops.h"
#include "tma.cuh"

namespace ab {

constexpr int kAttnThreads = 128;
constexpr int kAttnTile = 64;
constexpr int kAttnStages = 2;

// 16-byte vector of K/V elements converted to floats (4 for f32, 8 for bf16).
__device__ __forceinline__ void unpack(const uint4& v, float* f, float) {
    f[0] = __uint_as_float(v.x);
    f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z);
    f[3] = __uint_as_float(v.w);
}
__device__ __forceinline__ void unpack(const uint4& v, float* f, bf16) {
    f[0] = bf16lo(v.x);
    f[1] = bf16hi(v.x);
    f[2] = bf16lo(v.y);
    f[3] = bf16hi(v.y);
    f[4] = bf16lo(v.z);
    f[5] = bf16hi(v.z);
    f[6] = bf16lo(v.w);
    f[7] = bf16hi(v.w);
}

// Shared state after the K/V stage buffers (both kernels).
struct AttnTail {
    size_t q_off, s_off, p_off, st_off, fold_off, w_off, end;
};

__host__ __device__ inline AttnTail attn_tail(size_t o, uint32_t head, uint32_t G, uint32_t nsplit) {
    AttnTail T;
    o = (o + 15) & ~(size_t)15;
    T.q_off = o;
    o += (size_t)G * head * 4;
    T.s_off = o;
    o += (size_t)G * kAttnTile * 4;
    T.p_off = o;
    o += (size_t)kAttnTile * (G < 4 ? 4 : G) * 4;
    T.st_off = o;
    o += 3 * 8 * 4 + 16;
    T.fold_off = o;
    o += (size_t)kAttnThreads * G * 4;
    T.w_off = o;
    o += (size_t)nsplit * G * 4;
    T.end = (o + 15) & ~(size_t)15;
    return T;
}

// Plain-load layout: K rows padded to a stride of 4 (mod 8) words so that lanes reading
// different rows at the same column hit distinct banks.
struct AttnLayout {
    uint32_t row_words, kstride_words;
    size_t k_off, v_off;
    AttnTail t;
    size_t total;
};

__host__ __device__ inline AttnLayout attn_layout(uint32_t head, uint32_t esz, uint32_t G,
                                                  uint32_t nsplit) {
    AttnLayout L;
    L.row_words = head * esz / 4;
    L.kstride_words = L.row_words + ((12 - L.row_words % 8) % 8);
    L.k_off = 0;
    L.v_off = (size_t)kAttnTile * L.kstride_words * 4;
    L.t = attn_tail(L.v_off + (size_t)kAttnTile * L.row_words * 4, head, G, nsplit);
    L.total = L.t.end;
    return L;
}

// Online-softmax update of one tile: scores sc[G][64] -> probabilities pt[64][PS],
// running m/l and the rescale factor alpha per head. Warp w takes heads w, w + 4.
template <int G>
__device__ __forceinline__ void attn_softmax_tile(const float* sc, float* pt, float* sm_m,
                                                  float* sm_l, float* sm_a, uint32_t warp,
                                                  uint32_t lane) {
    constexpr int PS = G < 4 ? 4 : G;
    for (int h = warp; h < G; h += 4) {
        const float s0 = sc[h * kAttnTile + lane], s1 = sc[h * kAttnTile + lane + 32];
        const float tmax = warp_max(fmaxf(s0, s1));
        const float mold = sm_m[h];
        const float mnew = fmaxf(mold, tmax);
        const float alpha = expf(mold - mnew);
        const float e0 = expf(s0 - mnew), e1 = expf(s1 - mnew);
        const float lsum = warp_sum(e0 + e1);
        pt[lane * PS + h] = e0;
        pt[(lane + 32) * PS + h] = e1;
        if (lane == 0) {
            sm_m[h] = mnew;
            sm_l[h] = sm_l[h] * alpha + lsum;
            sm_a[h] = alpha;
        }
    }
}

// After the last tile: fold the ways, then either write the output (one active split) or
// publish this split's partial and, in the last CTA of the group, combine the partials.
template <typename OT, int G>
__device__ __forceinline__ void attn_finish(const AttnParams& p, float* acc, uint32_t way,
                                            uint32_t ways, uint32_t di, float* fold, float* wts,
                                            float* sm_m, float* sm_l, int* sm_last,
                                            uint32_t split, uint32_t active, uint32_t kvh,
                                            uint32_t b, uint32_t tid) {
    const uint32_t hd = p.head;
    if (way < ways) {
#pragma unroll
        for (int h = 0; h < G; h++) fold[((size_t)way * G + h) * hd + di] = acc[h];
    }
    __syncthreads();
    if (way == 0) {
        for (uint32_t w = 1; w < ways; w++) {
#pragma unroll
            for (int h = 0; h < G; h++) acc[h] += fold[((size_t)w * G + h) * hd + di];
        }
    }
    const uint64_t orow = (uint64_t)b * p.heads * hd + (uint64_t)kvh * G * hd;
    if (active == 1) {
        if (way == 0) {
#pragma unroll
            for (int h = 0; h < G; h++) {
                const float l = sm_l[h];
                const float v = l > 0.0f ? acc[h] / l : 0.0f;
                ((OT*)p.out)[orow + (uint64_t)h * hd + di] = from_f32<OT>(v);
            }
        }
        return;
    }
    const uint64_t grp = (uint64_t)b * p.kv_heads + kvh;
    float* po = p.part_o + (grp * p.nsplit + split) * G * hd;
    float* pml = p.part_ml + (grp * p.nsplit + split) * G * 2;
    if (way == 0) {
#pragma unroll
        for (int h = 0; h < G; h++) po[(size_t)h * hd + di] = acc[h];
    }
    if (tid < (uint32_t)G) {
        pml[tid * 2] = sm_m[tid];
        pml[tid * 2 + 1] = sm_l[tid];
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const uint32_t prev = atomicAdd(p.counters + grp, 1u);
        *sm_last = prev == active - 1;
    }
    __syncthreads();
    if (!*sm_last) return;
    __threadfence();
    const float* go = p.part_o + grp * p.nsplit * G * hd;
    const float* gml = p.part_ml + grp * p.nsplit * G * 2;
    // per-head maximum over the active splits (threads stride the splits)
    float red[G];
#pragma unroll
    for (int h = 0; h < G; h++) red[h] = -INFINITY;
    for (uint32_t s = tid; s < active; s += kAttnThreads) {
#pragma unroll
        for (int h = 0; h < G; h++) red[h] = fmaxf(red[h], __ldcg(gml + (s * G + h) * 2));
    }
#pragma unroll
    for (int h = 0; h < G; h++) fold[tid * G + h] = red[h];
    __syncthreads();
    if (tid < (uint32_t)G) {
        float M = -INFINITY;
        for (uint32_t t = 0; t < kAttnThreads; t++) M = fmaxf(M, fold[t * G + tid]);
        sm_m[tid] = M;
    }
    __syncthreads();
    // split weights exp(m_s - M) and the normaliser sum_s w_s l_s
#pragma unroll
    for (int h = 0; h < G; h++) red[h] = 0.0f;
    for (uint32_t s = tid; s < active; s += kAttnThreads) {
#pragma unroll
        for (int h = 0; h < G; h++) {
            const float w = expf(__ldcg(gml + (s * G + h) * 2) - sm_m[h]);
            wts[s * G + h] = w;
            red[h] += w * __ldcg(gml + (s * G + h) * 2 + 1);
        }
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < G; h++) fold[tid * G + h] = red[h];
    __syncthreads();
    if (tid < (uint32_t)G) {
        float L = 0.0f;
        for (uint32_t t = 0; t < kAttnThreads; t++) L += fold[t * G + tid];
        sm_l[tid] = L;
    }
    __syncthreads();
    // each thread folds all of its outputs at once with four independent sums apiece, so
    // NO * 4 partial loads are in flight per step instead of one dependent chain
    constexpr int NO = (G * 128 + kAttnThreads - 1) / kAttnThreads;
    float v[NO][4];
#pragma unroll
    for (int k = 0; k < NO; k++) v[k][0] = v[k][1] = v[k][2] = v[k][3] = 0.0f;
    uint32_t s = 0;
    for (; s + 4 <= active; s += 4) {
#pragma unroll
        for (int u = 0; u < 4; u++) {
#pragma unroll
            for (int k = 0; k < NO; k++) {
                const uint32_t o = tid + k * kAttnThreads;
                if (o < G * hd)
                    v[k][u] += wts[(s + u) * G + o / hd] *
                               __ldcg(go + (size_t)(s + u) * G * hd + o);
            }
        }
    }
    for (; s < active; s++) {
#pragma unroll
        for (int k = 0; k < NO; k++) {
            const uint32_t o = tid + k * kAttnThreads;
            if (o < G * hd) v[k][0] += wts[s * G + o / hd] * __ldcg(go + (size_t)s * G * hd + o);
        }
    }
#pragma unroll
    for (int k = 0; k < NO; k++) {
        const uint32_t o = tid + k * kAttnThreads;
        if (o < G * hd) {
            const float L = sm_l[o / hd];
            const float tot = (v[k][0] + v[k][1]) + (v[k][2] + v[k][3]);
            ((OT*)p.out)[orow + o] = from_f32<OT>(L > 0.0f ? tot / L : 0.0f);
        }
    }
    if (tid == 0) p.counters[grp] = 0;
}

// Merges the four warps' partial results of a CTA (per-head max wm, sum wl and unnormalised
// output wo[warp][head][dim], all in shared memory) and hands the CTA's result to
// attn_finish. Called by every thread after the warps wrote their parts.
template <typename OT, int G>
__device__ __forceinline__ void attn_merge_finish(const AttnParams& p, const float* wo,
                                                  float (*wm)[8], float (*wl)[8], float* run_m,
                                                  float* run_l, uint32_t hd, float* fold,
                                                  float* wts, int* sm_last, uint32_t split,
                                                  uint32_t active, uint32_t kvh, uint32_t b,
                                                  uint32_t tid) {
    __syncthreads();
    if (tid < (uint32_t)G) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < 4; w++) M = fmaxf(M, wm[w][tid]);
        float L = 0.0f;
#pragma unroll
        for (int w = 0; w < 4; w++)
            if (wm[w][tid] != -INFINITY) L += wl[w][tid] * expf(wm[w][tid] - M);
        run_m[tid] = M;
        run_l[tid] = L;
    }
    __syncthreads();
    const uint32_t di = tid % hd;
    float acc[G];
#pragma unroll
    for (int h = 0; h < G; h++) {
        float a = 0.0f;
#pragma unroll
        for (int w = 0; w < 4; w++) {
            const float mw = wm[w][h];
            if (mw != -INFINITY) a += wo[(w * G + h) * hd + di] * expf(mw - run_m[h]);
        }
        acc[h] = a;
    }
    attn_finish<OT, G>(p, acc, tid / hd, 1, di, fold, wts, run_m, run_l, sm_last, split, active,
                       kvh, b, tid);
}

// The split's position range [start, end) and the number of splits holding positions.
__device__ __forceinline__ void attn_split_range(const AttnParams& p, uint32_t split, uint32_t b,
                                                 uint32_t* start, uint32_t* end, uint32_t* active) {
    const uint32_t pos = p.step[b].position;
    const bool bad = pos >= p.seq;
    if (bad && split == 0 && blockIdx.y == 0 && threadIdx.x == 0)
        atomicOr(p.flags, kFlagPositionRange);
    const uint32_t total = bad ? 0u : pos + 1;
    uint32_t chunk = (total + p.nsplit - 1) / p.nsplit;
    chunk = max(1u, (chunk + kAttnTile - 1) / kAttnTile) * kAttnTile;
    chunk = max(chunk, p.min_chunk);
    *active = max(1u, (total + chunk - 1) / chunk);
    *start = min(split * chunk, total);
    *end = min(*start + chunk, total);
}

// ---- warp-independent SIMT kernel (f32 K/V; bf16 heads other than 64 and 128) ------------
// The pipeline of the tensor-core kernel below with CUDA-core arithmetic: K/V tiles of 64
// positions in a TMA ring (32/64/128-byte swizzle), each warp owning 16 positions of every
// tile. For q.K lane l takes position l % 16 and half l / 16 of the head dims (the halves
// meet in one shuffle); the warp's online softmax runs per head over its 16 positions; for
// P.V lane l owns head dims l, l + 32, ... and each position's weights come by shuffle from
// the lane that scored it. Warps release stages with one arrival each; thread 0 refills.
constexpr uint32_t kWarpMaxStages = 4;

struct AttnWarpLayout {
    uint32_t stage_bytes, stages;
    size_t q_off, fold_off, w_off, last_off, total;
};

__host__ __device__ inline AttnWarpLayout attn_warp_layout(uint32_t head, uint32_t esz, uint32_t G,
                                                           uint32_t nsplit) {
    AttnWarpLayout L;
    L.stage_bytes = 2u * kAttnTile * head * esz;
    // about 64 KB of stages: three CTAs per SM at f32 head 64, whose splits are short
    uint32_t st = (64u * 1024) / L.stage_bytes;
    L.stages = st < 2 ? 2 : st > kWarpMaxStages ? kWarpMaxStages : st;
    size_t o = (size_t)L.stages * L.stage_bytes;
    L.q_off = o;
    o += (size_t)G * head * 4;
    L.fold_off = o;
    o += (size_t)kAttnThreads * G * 4;
    L.w_off = o;
    o += (size_t)nsplit * G * 4;
    L.last_off = o;
    o += 16;
    L.total = o + 1024;
    return L;
}

template <typename KT, typename OT, int G, int SWZ>
__global__ void __launch_bounds__(kAttnThreads)
    attn_decode_warp_kernel(const AttnParams p, const __grid_constant__ CUtensorMap kmap,
                            const __grid_constant__ CUtensorMap vmap,
                            const __grid_constant__ CUtensorMap kmap16,
                            const __grid_constant__ CUtensorMap vmap16) {
    constexpr uint32_t ESZ = sizeof(KT);
    constexpr uint32_t VE = 16 / ESZ;     // elements per 16-byte chunk
    constexpr uint32_t BOXE = SWZ / ESZ;  // elements per box row
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t full_bar[kWarpMaxStages];
    __shared__ __align__(8) uint64_t empty_bar[kWarpMaxStages];
    __shared__ float wm[4][8], wl[4][8], run_m[8], run_l[8];
    __shared__ int sm_fail;
    const uint32_t hd = p.head;
    const AttnWarpLayout L = attn_warp_layout(hd, ESZ, G, p.nsplit);
    const uint32_t S = L.stages;
    unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    float* qs = (float*)(smem + L.q_off);  // [G][hd], pre-scaled by 1/sqrt(hd)
    float* fold = (float*)(smem + L.fold_off);
    float* wts = (float*)(smem + L.w_off);
    int* sm_last = (int*)(smem + L.last_off);

    const uint32_t split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const uint32_t tid = threadIdx.x, lane = tid % 32, warp = tid / 32;
    const uint32_t nbox = hd * ESZ / SWZ;

    pdl_wait();
    uint32_t start, end, active;
    attn_split_range(p, split, b, &start, &end, &active);
    if (split >= active) {
        pdl_trigger();
        return;
    }
    const uint32_t ntiles = (end - start + kAttnTile - 1) / kAttnTile;
    const int32_t ybase = (int32_t)(b * p.cache_rows + start);
    auto issue = [&](uint32_t i) {
        const uint32_t s = i % S;
        const uint32_t bar = smem_u32(&full_bar[s]);
        unsigned char* kst = smem + (size_t)s * L.stage_bytes;
        unsigned char* vst = kst + L.stage_bytes / 2;
        const int32_t y = ybase + (int32_t)(i * kAttnTile);
        const uint32_t rows = min((uint32_t)kAttnTile, end - (start + i * kAttnTile));
        if (rows == kAttnTile) {
            mbar_arrive_expect_tx(bar, L.stage_bytes);
            for (uint32_t j = 0; j < nbox; j++) {
                const int32_t x = (int32_t)(kvh * hd + j * BOXE);
                tma_load_2d(smem_u32(kst + (size_t)j * kAttnTile * SWZ), &kmap, x, y, bar);
                tma_load_2d(smem_u32(vst + (size_t)j * kAttnTile * SWZ), &vmap, x, y, bar);
            }
        } else {
            // the split's last tile: only the 16-row groups that hold positions
            const uint32_t groups = (rows + 15) / 16;
            mbar_arrive_expect_tx(bar, groups * 16 * 2 * hd * ESZ);
            for (uint32_t q = 0; q < groups; q++) {
                for (uint32_t j = 0; j < nbox; j++) {
                    const int32_t x = (int32_t)(kvh * hd + j * BOXE);
                    const size_t off = (size_t)j * kAttnTile * SWZ + (size_t)q * 16 * SWZ;
                    tma_load_2d(smem_u32(kst + off), &kmap16, x, y + 16 * q, bar);
                    tma_load_2d(smem_u32(vst + off), &vmap16, x, y + 16 * q, bar);
                }
            }
        }
    };
    uint32_t issued = 0;  // meaningful in thread 0
    if (tid == 0) {
        for (uint32_t s = 0; s < S; s++) {
            mbar_init(smem_u32(&full_bar[s]), 1);
            mbar_init(smem_u32(&empty_bar[s]), 4);
        }
        fence_barrier_init();
        sm_fail = 0;
        // the first tiles are in flight while q is staged
        for (; issued < ntiles && issued < S; issued++) issue(issued);
    }
    const float qscale = 1.0f / sqrtf((float)hd);
    const float* qsrc = p.q + ((uint64_t)b * p.heads + (uint64_t)kvh * G) * hd;
    for (uint32_t i = tid; i < G * hd; i += kAttnThreads) qs[i] = qsrc[i] * qscale;
    __syncthreads();

    const uint32_t pl = lane % 16, half = lane / 16, hh = hd / 2;
    float acc[G][4];
    float m[G], lp[G];
#pragma unroll
    for (int h = 0; h < G; h++) {
        acc[h][0] = acc[h][1] = acc[h][2] = acc[h][3] = 0.0f;
        m[h] = -INFINITY;
        lp[h] = 0.0f;
    }
    for (uint32_t i = 0; i < ntiles; i++) {
        if (tid == 0 && i >= 1 && issued < ntiles) {
            const uint32_t r = i - 1;
            if (mbar_wait_bounded(smem_u32(&empty_bar[r % S]), (r / S) & 1, p.flags)) issue(issued++);
            else sm_fail = 1;
        }
        __syncwarp();
        if (__any_sync(0xffffffffu, *(volatile int*)&sm_fail != 0)) break;
        const uint32_t s = i % S;
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&full_bar[s]), (i / S) & 1, p.flags))) {
            sm_fail = 1;
            break;
        }
        const uint32_t rows = min((uint32_t)kAttnTile, end - (start + i * kAttnTile));
        const unsigned char* kst = smem + (size_t)s * L.stage_bytes;
        const unsigned char* vst = kst + L.stage_bytes / 2;
        // a warp whose 16 positions all lie past the split's end has nothing in this tile
        if (warp * 16 < rows) {
            // q.K: position 16 * warp + pl over half `half` of the head dims
            const uint32_t row = warp * 16 + pl;
            float d[G];
#pragma unroll
            for (int h = 0; h < G; h++) d[h] = 0.0f;
            for (uint32_t c = 0; c < hh / VE; c++) {
                const uint32_t e0 = half * hh + c * VE;
                const uint32_t byte = e0 * ESZ;
                const uint32_t off =
                    swizzle_off<SWZ>((byte / SWZ) * kAttnTile * SWZ + row * SWZ + byte % SWZ);
                float kf[VE];
                unpack(*reinterpret_cast<const uint4*>(kst + off), kf, KT());
#pragma unroll
                for (int h = 0; h < G; h++) {
                    const float* qh = qs + h * hd + e0;
#pragma unroll
                    for (uint32_t e = 0; e < VE; e++) d[h] = fmaf(qh[e], kf[e], d[h]);
                }
            }
            const bool valid = row < rows;
            float e[G];
#pragma unroll
            for (int h = 0; h < G; h++) {
                // every lane takes part in the shuffle; invalid positions are masked after it
                const float other = __shfl_xor_sync(0xffffffffu, d[h], 16);
                const float sc = valid ? d[h] + other : -INFINITY;
                float t = sc;
#pragma unroll
                for (int off = 1; off < 16; off <<= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, off));
                const float n = fmaxf(m[h], t);
                const float alpha = n == -INFINITY ? 1.0f : expf(m[h] - n);
                e[h] = n == -INFINITY ? 0.0f : expf(sc - n);
                m[h] = n;
                lp[h] = lp[h] * alpha + e[h];
#pragma unroll
                for (int k = 0; k < 4; k++) acc[h][k] *= alpha;
            }
            // P.V: lane owns dims lane + 32k; the weight of position q comes from lane q
            for (uint32_t q = 0; q < 16; q++) {
                const uint32_t vrow = warp * 16 + q;
                float w[G];
#pragma unroll
                for (int h = 0; h < G; h++) w[h] = __shfl_sync(0xffffffffu, e[h], q);
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const uint32_t dd = lane + 32 * k;
                    if (dd < hd) {
                        const uint32_t byte = dd * ESZ;
                        const uint32_t off = swizzle_off<SWZ>((byte / SWZ) * kAttnTile * SWZ +
                                                              vrow * SWZ + byte % SWZ);
                        const float v = to_f32(*reinterpret_cast<const KT*>(vst + off));
#pragma unroll
                        for (int h = 0; h < G; h++) acc[h][k] = fmaf(w[h], v, acc[h][k]);
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&empty_bar[s]));
    }
    __syncthreads();
    if (sm_fail) {
        if (tid == 0) {
            atomicOr(p.flags, kFlagWaitTimeout);
            for (uint32_t j = issued > S ? issued - S : 0; j < issued; j++)
                mbar_wait_bounded(smem_u32(&full_bar[j % S]), (j / S) & 1, p.flags);
        }
        __syncthreads();
        pdl_trigger();
        return;
    }
    pdl_trigger();
    // per-warp sums over the 16 scoring lanes (lanes 16-31 hold copies)
    float* wo = (float*)smem;  // [4 warps][G][hd] over the drained stages
#pragma unroll
    for (int h = 0; h < G; h++) {
        float l = lane < 16 ? lp[h] : 0.0f;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
        if (lane == 0) {
            wm[warp][h] = m[h];
            wl[warp][h] = l;
        }
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const uint32_t dd = lane + 32 * k;
            if (dd < hd) wo[(warp * G + h) * hd + dd] = acc[h][k];
        }
    }
    attn_merge_finish<OT, G>(p, wo, wm, wl, run_m, run_l, hd, fold, wts, sm_last, split, active,
                             kvh, b, tid);
}

// ---- tensor-core kernel (bf16 K/V, head 64 or 128) --------------------------------------------
// Each of the four warps owns 16 positions of every 64-position tile end to end, so warps
// never wait for one another inside the loop:
//   S[16 pos x 8 heads]   = K[16 x head] . Q^T[head x 8]        (mma.sync m16n8k16)
//   online softmax per head over the warp's positions (its own running max and sum)
//   O^T[head x 8 heads]  += V^T[head x 16 pos] . P^T[16 pos x 8] (P^T formed in registers by
//                                                                 movmatrix.trans)
// Q and P are split into bf16 high and low parts (two MMAs each), so scores and weights
// keep close to fp32 precision; K and V are bf16 already. Operand fragments come from the
// swizzled TMA tiles through ldmatrix (V transposed). Thread 0 refills a stage once all
// four warps have released it (one arrival each on its empty barrier); the warps' partial
// (max, sum, O) are merged through shared memory after the loop. Positions past the
// current one inside the last tile are masked out of the softmax; they must hold finite
// values (caches start zeroed), as their zero weights multiply them.
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t* r) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t* r) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void mma_16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// Two floats as a bf16 pair (first in the low half) and the pair of what rounding left.
__device__ __forceinline__ void split_bf16x2(float a, float b, uint32_t* hi, uint32_t* lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    const float2 hf = __bfloat1622float2(h);
    const __nv_bfloat162 l = __floats2bfloat162_rn(a - hf.x, b - hf.y);
    *hi = *reinterpret_cast<const uint32_t*>(&h);
    *lo = *reinterpret_cast<const uint32_t*>(&l);
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

template <int HD>
struct AttnMmaLayout {
    static constexpr uint32_t kRowBytes = HD * 2;
    static constexpr uint32_t kStage = 2 * kAttnTile * kRowBytes;  // K tile | V tile
    static constexpr uint32_t kStages = HD == 128 ? 3 : 4;
    static constexpr uint32_t kTail = kStages * kStage;  // then fold, split weights, ticket
    static size_t smem(uint32_t G, uint32_t nsplit) {
        return (size_t)kTail + (size_t)kAttnThreads * G * 4 + (size_t)nsplit * G * 4 + 16 + 1024;
    }
};

template <typename OT, int G, int HD>
__global__ void __launch_bounds__(kAttnThreads)
    attn_decode_mma_kernel(const AttnParams p, const __grid_constant__ CUtensorMap kmap,
                           const __grid_constant__ CUtensorMap vmap,
                           const __grid_constant__ CUtensorMap kmap16,
                           const __grid_constant__ CUtensorMap vmap16) {
    using LY = AttnMmaLayout<HD>;
    constexpr uint32_t S = LY::kStages;
    constexpr uint32_t NBOX = LY::kRowBytes / 128;
    constexpr int KS = HD / 16;  // k-steps of K.Q^T, m-tiles of V^T.P^T
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t full_bar[S];
    __shared__ __align__(8) uint64_t empty_bar[S];
    __shared__ float wm[4][8], wl[4][8], run_m[8], run_l[8];
    __shared__ int sm_fail;
    unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    float* fold = (float*)(smem + LY::kTail);  // [kAttnThreads][G]
    float* wts = fold + kAttnThreads * G;      // [nsplit][G]
    int* sm_last = (int*)(wts + p.nsplit * G);

    const uint32_t split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const uint32_t tid = threadIdx.x, lane = tid % 32, warp = tid / 32;
    const uint32_t g = lane / 4, t = lane % 4;

    pdl_wait();
    uint32_t start, end, active;
    attn_split_range(p, split, b, &start, &end, &active);
    if (split >= active) {
        pdl_trigger();
        return;
    }
    const uint32_t ntiles = (end - start + kAttnTile - 1) / kAttnTile;
    const int32_t ybase = (int32_t)(b * p.cache_rows + start);
    auto issue = [&](uint32_t i) {
        const uint32_t s = i % S;
        const uint32_t bar = smem_u32(&full_bar[s]);
        unsigned char* kst = smem + (size_t)s * LY::kStage;
        unsigned char* vst = kst + LY::kStage / 2;
        const int32_t y = ybase + (int32_t)(i * kAttnTile);
        const uint32_t rows = min((uint32_t)kAttnTile, end - (start + i * kAttnTile));
        if (rows == kAttnTile) {
            mbar_arrive_expect_tx(bar, LY::kStage);
#pragma unroll
            for (uint32_t j = 0; j < NBOX; j++) {
                const int32_t x = (int32_t)(kvh * HD + j * 64);
                tma_load_2d(smem_u32(kst + j * kAttnTile * 128), &kmap, x, y, bar);
                tma_load_2d(smem_u32(vst + j * kAttnTile * 128), &vmap, x, y, bar);
            }
        } else {
            // the split's last tile: only the 16-row groups that hold positions
            const uint32_t groups = (rows + 15) / 16;
            mbar_arrive_expect_tx(bar, groups * 16 * 2 * LY::kRowBytes);
            for (uint32_t q = 0; q < groups; q++) {
#pragma unroll
                for (uint32_t j = 0; j < NBOX; j++) {
                    const int32_t x = (int32_t)(kvh * HD + j * 64);
                    const uint32_t off = j * kAttnTile * 128 + q * 16 * 128;
                    tma_load_2d(smem_u32(kst + off), &kmap16, x, y + 16 * q, bar);
                    tma_load_2d(smem_u32(vst + off), &vmap16, x, y + 16 * q, bar);
                }
            }
        }
    };
    uint32_t issued = 0;  // meaningful in thread 0
    if (tid == 0) {
        for (uint32_t s = 0; s < S; s++) {
            mbar_init(smem_u32(&full_bar[s]), 1);
            mbar_init(smem_u32(&empty_bar[s]), 4);
        }
        fence_barrier_init();
        sm_fail = 0;
        // the first tiles are in flight while the Q fragments load
        for (; issued < ntiles && issued < S; issued++) issue(issued);
    }
    // Q^T fragments (k = head dim, n = query head), pre-scaled, bf16 high + low parts
    uint32_t qh[KS][2], ql[KS][2];
    {
        const float qscale = 1.0f / sqrtf((float)HD);
        const float* qsrc = p.q + ((uint64_t)b * p.heads + (uint64_t)kvh * G) * HD;
#pragma unroll
        for (int ks = 0; ks < KS; ks++) {
#pragma unroll
            for (int h2 = 0; h2 < 2; h2++) {
                const uint32_t d = ks * 16 + 2 * t + 8 * h2;
                float a = 0.0f, c = 0.0f;
                if (g < (uint32_t)G) {
                    a = qsrc[g * HD + d] * qscale;
                    c = qsrc[g * HD + d + 1] * qscale;
                }
                split_bf16x2(a, c, &qh[ks][h2], &ql[ks][h2]);
            }
        }
    }
    __syncthreads();

    float o[KS][4];
#pragma unroll
    for (int m = 0; m < KS; m++) o[m][0] = o[m][1] = o[m][2] = o[m][3] = 0.0f;
    float mA = -INFINITY, mB = -INFINITY, lA = 0.0f, lB = 0.0f;  // heads 2t, 2t + 1
    const uint32_t mi = lane / 8, r8 = lane % 8;
    for (uint32_t i = 0; i < ntiles; i++) {
        // thread 0 refills the stage of tile i - 1 once all four warps released it
        if (tid == 0 && i >= 1 && issued < ntiles) {
            const uint32_t r = i - 1;
            if (mbar_wait_bounded(smem_u32(&empty_bar[r % S]), (r / S) & 1, p.flags)) issue(issued++);
            else sm_fail = 1;
        }
        __syncwarp();
        if (__any_sync(0xffffffffu, *(volatile int*)&sm_fail != 0)) break;
        const uint32_t s = i % S;
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&full_bar[s]), (i / S) & 1, p.flags))) {
            sm_fail = 1;
            break;
        }
        const uint32_t rows = min((uint32_t)kAttnTile, end - (start + i * kAttnTile));
        const uint32_t kst = smem_u32(smem + (size_t)s * LY::kStage);
        const uint32_t vst = kst + LY::kStage / 2;
        // a warp whose 16 positions all lie past the split's end has nothing in this tile
        if (warp * 16 < rows) {
            // S for positions 16 * warp + (g, g + 8), heads (2t, 2t + 1)
            float sh[4] = {0.0f, 0.0f, 0.0f, 0.0f}, sl[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            {
                const uint32_t row = warp * 16 + (lane % 16);
#pragma unroll
                for (int ks = 0; ks < KS; ks++) {
                    const uint32_t colb = (ks % 4) * 32 + (lane / 16) * 16;
                    uint32_t a[4];
                    ldsm_x4(kst + swizzle_off<128>((ks / 4) * kAttnTile * 128 + row * 128 + colb), a);
                    mma_16816(sh, a, qh[ks][0], qh[ks][1]);
                    mma_16816(sl, a, ql[ks][0], ql[ks][1]);
                }
            }
            float sc[4] = {sh[0] + sl[0], sh[1] + sl[1], sh[2] + sl[2], sh[3] + sl[3]};
            const uint32_t p0 = warp * 16 + g;
            if (p0 >= rows) sc[0] = sc[1] = -INFINITY;
            if (p0 + 8 >= rows) sc[2] = sc[3] = -INFINITY;
            float ta = fmaxf(sc[0], sc[2]), tb = fmaxf(sc[1], sc[3]);
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) {
                ta = fmaxf(ta, __shfl_xor_sync(0xffffffffu, ta, off));
                tb = fmaxf(tb, __shfl_xor_sync(0xffffffffu, tb, off));
            }
            const float nA = fmaxf(mA, ta), nB = fmaxf(mB, tb);
            // a warp whose positions were all masked so far keeps m = -inf and weight 0
            const float aA = nA == -INFINITY ? 1.0f : expf(mA - nA);
            const float aB = nB == -INFINITY ? 1.0f : expf(mB - nB);
            const float e0 = nA == -INFINITY ? 0.0f : expf(sc[0] - nA);
            const float e1 = nB == -INFINITY ? 0.0f : expf(sc[1] - nB);
            const float e2 = nA == -INFINITY ? 0.0f : expf(sc[2] - nA);
            const float e3 = nB == -INFINITY ? 0.0f : expf(sc[3] - nB);
            mA = nA;
            mB = nB;
            lA = lA * aA + (e0 + e2);
            lB = lB * aB + (e1 + e3);
#pragma unroll
            for (int m = 0; m < KS; m++) {
                o[m][0] *= aA;
                o[m][1] *= aB;
                o[m][2] *= aA;
                o[m][3] *= aB;
            }
            // P^T fragments: the S accumulator holds (pos g / g + 8, heads 2t / 2t + 1); the
            // transposed 8x8 blocks hold (head g, pos 2t / 2t + 1 and 8 + ...)
            uint32_t h01, l01, h23, l23;
            split_bf16x2(e0, e1, &h01, &l01);
            split_bf16x2(e2, e3, &h23, &l23);
            const uint32_t bh0 = movmatrix_trans(h01), bh1 = movmatrix_trans(h23);
            const uint32_t bl0 = movmatrix_trans(l01), bl1 = movmatrix_trans(l23);
            const uint32_t pos = warp * 16 + r8 + (mi >= 2 ? 8 : 0);
#pragma unroll
            for (int m = 0; m < KS; m++) {
                const uint32_t byte = (m * 16 + ((mi & 1) ? 8 : 0)) * 2;
                uint32_t a[4];
                ldsm_x4_t(vst + swizzle_off<128>((byte / 128) * kAttnTile * 128 + pos * 128 +
                                                 byte % 128),
                          a);
                mma_16816(o[m], a, bh0, bh1);
                mma_16816(o[m], a, bl0, bl1);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&empty_bar[s]));
    }
    __syncthreads();
    if (sm_fail) {
        // a bounded wait ran out: flag it, let the copies in flight land, and stop (only the
        // last S issued tiles can still be in flight, each on the newest phase of its stage)
        if (tid == 0) {
            atomicOr(p.flags, kFlagWaitTimeout);
            for (uint32_t j = issued > S ? issued - S : 0; j < issued; j++)
                mbar_wait_bounded(smem_u32(&full_bar[j % S]), (j / S) & 1, p.flags);
        }
        __syncthreads();
        pdl_trigger();
        return;
    }
    pdl_trigger();
    // merge the four warps: per-head max, rescaled sums and outputs (stage memory is free)
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
        lA += __shfl_xor_sync(0xffffffffu, lA, off);
        lB += __shfl_xor_sync(0xffffffffu, lB, off);
    }
    if (g == 0) {
        wm[warp][2 * t] = mA;
        wm[warp][2 * t + 1] = mB;
        wl[warp][2 * t] = lA;
        wl[warp][2 * t + 1] = lB;
    }
    float* wo = (float*)smem;  // [4 warps][G][HD]
#pragma unroll
    for (int m = 0; m < KS; m++) {
        const uint32_t d0 = m * 16 + g;
        if (2 * t < (uint32_t)G) {
            wo[(warp * G + 2 * t) * HD + d0] = o[m][0];
            wo[(warp * G + 2 * t) * HD + d0 + 8] = o[m][2];
        }
        if (2 * t + 1 < (uint32_t)G) {
            wo[(warp * G + 2 * t + 1) * HD + d0] = o[m][1];
            wo[(warp * G + 2 * t + 1) * HD + d0 + 8] = o[m][3];
        }
    }
    attn_merge_finish<OT, G>(p, wo, wm, wl, run_m, run_l, HD, fold, wts, sm_last, split, active,
                             kvh, b, tid);
}

// Rows of one sequence over one shared cache (a prefill pass) take the tcgen05 prompt kernel
// (attention_prompt_tc.cu) from this many rows on; fewer take the split decode kernel.
constexpr uint32_t kPfMinBatch = 16;

// ---- plain-load kernel (head sizes the TMA boxes cannot tile) --------------------------------
template <typename KT, typename OT, int G>
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const AttnParams p) {
    extern __shared__ __align__(16) unsigned char smem[];
    constexpr int VE = 16 / sizeof(KT);  // elements per 16-byte vector
    constexpr int PS = G < 4 ? 4 : G;
    const uint32_t hd = p.head;
    const AttnLayout L = attn_layout(hd, sizeof(KT), G, p.nsplit);
    uint32_t* ks = (uint32_t*)(smem + L.k_off);  // [TP][kstride_words]
    uint32_t* vs = (uint32_t*)(smem + L.v_off);  // [TP][row_words]
    float* qs = (float*)(smem + L.t.q_off);      // [G][hd], pre-scaled by 1/sqrt(hd)
    float* sc = (float*)(smem + L.t.s_off);      // [G][TP] scores
    float* pt = (float*)(smem + L.t.p_off);      // [TP][max(G,4)] probabilities
    float* st = (float*)(smem + L.t.st_off);     // m[8], l[8], alpha[8], flag
    float* fold = (float*)(smem + L.t.fold_off);
    float* wts = (float*)(smem + L.t.w_off);
    float* sm_m = st;
    float* sm_l = st + 8;
    float* sm_a = st + 16;
    int* sm_last = (int*)(st + 24);

    const uint32_t split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const uint32_t tid = threadIdx.x, lane = tid % 32, warp = tid / 32;
    const uint32_t kvd = p.kv_heads * hd;
    const uint32_t nvec = hd / VE;  // 16-byte vectors per K/V row

    pdl_wait();
    uint32_t start, end, active;
    attn_split_range(p, split, b, &start, &end, &active);
    if (split >= active) {
        pdl_trigger();
        return;
    }
    const float qscale = 1.0f / sqrtf((float)hd);
    const float* qsrc = p.q + ((uint64_t)b * p.heads + (uint64_t)kvh * G) * hd;
    for (uint32_t i = tid; i < G * hd; i += kAttnThreads) qs[i] = qsrc[i] * qscale;
    if (tid < 8) {
        sm_m[tid] = -INFINITY;
        sm_l[tid] = 0.0f;
    }
    const uint32_t ways = kAttnThreads / hd;
    const uint32_t way = tid / hd, di = tid % hd;
    float acc[G];
#pragma unroll
    for (int h = 0; h < G; h++) acc[h] = 0.0f;
    __syncthreads();

    const KT* kbase = (const KT*)p.kcache + (uint64_t)b * p.cache_stride + (uint64_t)kvh * hd;
    const KT* vbase = (const KT*)p.vcache + (uint64_t)b * p.cache_stride + (uint64_t)kvh * hd;

    for (uint32_t t0 = start; t0 < end; t0 += kAttnTile) {
        const uint32_t rows = min((uint32_t)kAttnTile, end - t0);
        for (uint32_t v = tid; v < kAttnTile * nvec; v += kAttnThreads) {
            const uint32_t r = v / nvec, c = v % nvec;
            uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
            if (r < rows) {
                const uint64_t off = (uint64_t)(t0 + r) * kvd + (uint64_t)c * VE;
                kv = ld_stream(kbase + off);
                vv = ld_stream(vbase + off);
            }
            *reinterpret_cast<uint4*>(ks + (size_t)r * L.kstride_words + c * 4) = kv;
            *reinterpret_cast<uint4*>(vs + (size_t)r * L.row_words + c * 4) = vv;
        }
        __syncthreads();
        {
            const uint32_t pp = tid % kAttnTile, hg = tid / kAttnTile;
            float d[G];
#pragma unroll
            for (int h = 0; h < G; h++) d[h] = 0.0f;
            if (hg < (uint32_t)G) {
                const uint32_t* kr = ks + (size_t)pp * L.kstride_words;
                for (uint32_t c = 0; c < nvec; c++) {
                    float kf[VE];
                    unpack(*reinterpret_cast<const uint4*>(kr + c * 4), kf, KT());
#pragma unroll
                    for (int h = 0; h < G; h++) {
                        if ((h % 2) != (int)hg && G > 1) continue;
                        const float* qh = qs + h * hd + c * VE;
#pragma unroll
                        for (int e = 0; e < VE; e++) d[h] = fmaf(qh[e], kf[e], d[h]);
                    }
                }
#pragma unroll
                for (int h = 0; h < G; h++) {
                    if ((h % 2) != (int)hg && G > 1) continue;
                    sc[h * kAttnTile + pp] = pp < rows ? d[h] : -INFINITY;
                }
            }
        }
        __syncthreads();
        attn_softmax_tile<G>(sc, pt, sm_m, sm_l, sm_a, warp, lane);
        __syncthreads();
        if (way < ways) {
#pragma unroll
            for (int h = 0; h < G; h++) acc[h] *= sm_a[h];
            for (uint32_t r = way; r < rows; r += ways) {
                const KT* vr = reinterpret_cast<const KT*>(vs + (size_t)r * L.row_words);
                const float v = to_f32(vr[di]);
                const float* pr = pt + r * PS;
#pragma unroll
                for (int h = 0; h < G; h++) acc[h] = fmaf(pr[h], v, acc[h]);
            }
        }
        __syncthreads();
    }
    pdl_trigger();
    attn_finish<OT, G>(p, acc, way, ways, di, fold, wts, sm_m, sm_l, sm_last, split, active, kvh,
                       b, tid);
}

bool attention_fusable(uint32_t heads, uint32_t kv_heads, uint32_t head, int32_t kv_dtype) {
    if (kv_heads == 0 || heads % kv_heads) return false;
    const uint32_t G = heads / kv_heads;
    if (G != 1 && G != 2 && G != 4 && G != 8) return false;
    if (head == 0 || head > kAttnThreads || head % 2) return false;
    const uint32_t esz = kv_dtype == AB_BF16 ? 2 : 4;
    return (head * esz) % 16 == 0;
}

uint32_t attention_choose_splits(uint32_t batch, uint32_t kv_heads, uint32_t seq, int sm_count,
                                 uint32_t max_splits) {
    // The kernels keep two CTAs per SM resident. Split the positions so the (batch, kv
    // head, split) grid fills whole waves of those slots -- the first split count whose last
    // wave is at least 90% full, else the fullest -- with at least four 64-position tiles
    // per split. A grid with a group per slot or more is not split.
    const uint64_t slots = (uint64_t)std::max(sm_count, 1) * 2;
    const uint64_t groups = std::max<uint64_t>(1, (uint64_t)batch * kv_heads);
    const uint64_t tiles = (seq + kAttnTile - 1) / kAttnTile;
    const uint64_t cap = std::min<uint64_t>(std::max<uint32_t>(max_splits, 1),
                                            std::max<uint64_t>(1, tiles / 4));
    if (groups >= slots || cap <= 1) return 1;
    uint64_t best = 1;
    double best_fill = 0.0;
    for (uint64_t ns = 1; ns <= cap; ns++) {
        const uint64_t ctas = groups * ns;
        const uint64_t waves = (ctas + slots - 1) / slots;
        const double fill = (double)ctas / (double)(waves * slots);
        if (fill >= 0.9) return (uint32_t)ns;
        if (fill > best_fill) {
            best_fill = fill;
            best = ns;
        }
    }
    return (uint32_t)best;
}

// Smallest split, in positions (a multiple of the 64-position tile): 256 by default;
// AMMON_B200_ATTN_MIN_CHUNK overrides it (a tuning parameter: the results do not change).
uint32_t attention_min_chunk() {
    static const uint32_t v = [] {
        const char* e = std::getenv("AMMON_B200_ATTN_MIN_CHUNK");
        long n = e ? std::atol(e) : 256;
        if (n < kAttnTile) n = kAttnTile;
        if (n > 1 << 20) n = 1 << 20;
        return (uint32_t)(n / kAttnTile * kAttnTile);
    }();
    return v;
}

// Largest split count attention_choose_splits picks for any grid of up to `max_groups`
// (batch, kv head) groups: the scratch bound of a block whose kv head count is not yet known.
uint32_t attention_max_splits(uint32_t max_groups, uint32_t seq, int sm_count,
                              uint32_t max_splits) {
    uint32_t m = 1;
    for (uint32_t g = 1; g <= max_groups; g++)
        m = std::max(m, attention_choose_splits(g, 1, seq, sm_count, max_splits));
    return m;
}

void attention_scratch_size(uint32_t batch, uint32_t heads, uint32_t head, uint32_t nsplit,
                            uint64_t* floats, uint64_t* counters) {
    *floats = (uint64_t)batch * heads * nsplit * (head + 2);
    *counters = (uint64_t)batch * heads;
}

static cudaError_t set_smem(const void* kern, size_t smem) {
    if (smem <= 48 * 1024) return cudaSuccess;
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
}

template <typename KT, typename OT, int G>
static void add_attn(ab_scheme* s, const char* label, const AttnParams& p) {
    const int esz = sizeof(KT);
    const uint32_t rowbytes = p.head * esz;
    dim3 grid(p.nsplit, p.kv_heads, p.batch);
    const int swz = rowbytes % 128 == 0 ? 128 : rowbytes % 64 == 0 ? 64 : 0;
    // the rows share one cache (a prompt's positions): 128 queries per staged K/V tile on the
    // 5th-generation tensor cores (attention_prompt_tc.cu)
    if (esz == 2 && p.cache_rows == 0 && p.batch >= kPfMinBatch &&
        record_prompt_attention_tc(s, label, p))
        return;
    if (esz == 2 && (p.head == 128 || p.head == 64)) {
        // bf16 K/V: both products on the tensor cores
        CUtensorMap kmap, vmap;
        const uint64_t inner = (uint64_t)p.kv_heads * p.head;
        const uint64_t rows = (uint64_t)(p.batch - 1) * p.cache_rows + p.seq;
        encode_tmap_2d(&kmap, AB_BF16, p.kcache, inner, rows, inner * 2, 64, kAttnTile, 128);
        encode_tmap_2d(&vmap, AB_BF16, p.vcache, inner, rows, inner * 2, 64, kAttnTile, 128);
        CUtensorMap kmap16, vmap16;  // 16-row boxes for a split's partial last tile
        encode_tmap_2d(&kmap16, AB_BF16, p.kcache, inner, rows, inner * 2, 64, 16, 128);
        encode_tmap_2d(&vmap16, AB_BF16, p.vcache, inner, rows, inner * 2, 64, 16, 128);
        const size_t smem = p.head == 128 ? AttnMmaLayout<128>::smem(G, p.nsplit)
                                          : AttnMmaLayout<64>::smem(G, p.nsplit);
        if (smem > 220 * 1024) invalid("attention: shared-memory stage too large");
        if (p.head == 128) {
            auto kern = attn_decode_mma_kernel<OT, G, 128>;
            s->add(label, [=](cudaStream_t st) {
                cudaError_t e = set_smem((const void*)kern, smem);
                if (e != cudaSuccess) return e;
                return launch(st, grid, dim3(kAttnThreads), smem, true, kern, p, kmap, vmap, kmap16,
                              vmap16);
            });
        } else {
            auto kern = attn_decode_mma_kernel<OT, G, 64>;
            s->add(label, [=](cudaStream_t st) {
                cudaError_t e = set_smem((const void*)kern, smem);
                if (e != cudaSuccess) return e;
                return launch(st, grid, dim3(kAttnThreads), smem, true, kern, p, kmap, vmap, kmap16,
                              vmap16);
            });
        }
        return;
    }
    if (swz) {
        CUtensorMap kmap, vmap;
        const uint64_t inner = (uint64_t)p.kv_heads * p.head;
        const uint64_t rows = (uint64_t)(p.batch - 1) * p.cache_rows + p.seq;
        encode_tmap_2d(&kmap, esz == 2 ? AB_BF16 : AB_F32, p.kcache, inner, rows, inner * esz,
                       swz / esz, kAttnTile, swz);
        encode_tmap_2d(&vmap, esz == 2 ? AB_BF16 : AB_F32, p.vcache, inner, rows, inner * esz,
                       swz / esz, kAttnTile, swz);
        CUtensorMap kmap16, vmap16;  // 16-row boxes for a split's partial last tile
        encode_tmap_2d(&kmap16, esz == 2 ? AB_BF16 : AB_F32, p.kcache, inner, rows, inner * esz,
                       swz / esz, 16, swz);
        encode_tmap_2d(&vmap16, esz == 2 ? AB_BF16 : AB_F32, p.vcache, inner, rows, inner * esz,
                       swz / esz, 16, swz);
        const size_t smem = attn_warp_layout(p.head, esz, G, p.nsplit).total;
        if (smem > 220 * 1024) invalid("attention: shared-memory stage too large");
        if (swz == 128) {
            auto kern = attn_decode_warp_kernel<KT, OT, G, 128>;
            s->add(label, [=](cudaStream_t st) {
                cudaError_t e = set_smem((const void*)kern, smem);
                if (e != cudaSuccess) return e;
                return launch(st, grid, dim3(kAttnThreads), smem, true, kern, p, kmap, vmap, kmap16,
                              vmap16);
            });
        } else {
            auto kern = attn_decode_warp_kernel<KT, OT, G, 64>;
            s->add(label, [=](cudaStream_t st) {
                cudaError_t e = set_smem((const void*)kern, smem);
                if (e != cudaSuccess) return e;
                return launch(st, grid, dim3(kAttnThreads), smem, true, kern, p, kmap, vmap, kmap16,
                              vmap16);
            });
        }
        return;
    }
    const size_t smem = attn_layout(p.head, esz, G, p.nsplit).total;
    if (smem > 200 * 1024) invalid("attention: shared-memory stage too large");
    auto kern = attn_decode_kernel<KT, OT, G>;
    s->add(label, [=](cudaStream_t st) {
        cudaError_t e = set_smem((const void*)kern, smem);
        if (e != cudaSuccess) return e;
        return launch(st, grid, dim3(kAttnThreads), smem, true, kern, p);
    });
}

template <typename KT, typename OT>
static void dispatch_g(ab_scheme* s, const char* label, const AttnParams& p) {
    switch (p.heads / p.kv_heads) {
        case 1: return add_attn<KT, OT, 1>(s, label, p);
        case 2: return add_attn<KT, OT, 2>(s, label, p);
        case 4: return add_attn<KT, OT, 4>(s, label, p);
        case 8: return add_attn<KT, OT, 8>(s, label, p);
        default: invalid("attention: heads per kv head must be 1, 2, 4 or 8");
    }
}

void record_attention(ab_scheme* s, const char* label, AttnParams p) {
    if (!attention_fusable(p.heads, p.kv_heads, p.head, p.kv_dtype))
        invalid("attention: shape not supported by the fused kernel");
    // the tiled loads address the cache as [(batch - 1) * cache_rows + seq] rows of
    // kv_heads * head elements: cache_rows is seq for a cache per batch row, 0 when every
    // row reads the same cache (consecutive positions of one sequence)
    const uint64_t row = (uint64_t)p.kv_heads * p.head;
    if (p.cache_stride % row || p.cache_stride / row > p.seq)
        invalid("attention: the cache stride must be 0 or a whole number of positions <= seq");
    p.cache_rows = (uint32_t)(p.cache_stride / row);
    if (p.kv_dtype == AB_BF16) {
        if (p.out_dtype == AB_BF16) dispatch_g<bf16, bf16>(s, label, p);
        else dispatch_g<bf16, float>(s, label, p);
    } else {
        if (p.out_dtype == AB_BF16) dispatch_g<float, bf16>(s, label, p);
        else dispatch_g<float, float>(s, label, p);
    }
}

}  // namespace ab

// ---- allocation-free variant ------------------------------------------------------------
// ab_attention_decode_noalloc runs attn_decode_kernel with its split partials and tickets in
// one fixed array of device memory that is part of the library image, so the call itself
// allocates nothing. Layout of the array: kNoAllocFloats floats of partials, then
// kNoAllocTickets 32-bit tickets, then one flag word.
namespace ab {

constexpr uint64_t kNoAllocFloats = 1ull << 20;  // 4 MiB of split partials
constexpr uint32_t kNoAllocTickets = 16384;      // 64 KiB of tickets (batch * kv_heads)
constexpr uint64_t kNoAllocBytes = kNoAllocFloats * 4 + (uint64_t)kNoAllocTickets * 4 + 256;
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) unsigned char g_attn_noalloc_scratch[kNoAllocBytes];

static std::mutex g_noalloc_mu;
static void* g_noalloc_addr[kNoAllocMaxDevices] = {};

// Device address of the scratch array on the current device, looked up once per device.
static unsigned char* noalloc_scratch(int* device) {
    cuda_check(cudaGetDevice(device), "cudaGetDevice");
    if (*device < 0 || *device >= kNoAllocMaxDevices)
        fail(AB_ERR_ARGUMENT, "device index out of range for the static scratch table");
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_addr[*device]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
        if (e != cudaSuccess || !p)
            fail(AB_ERR_CUDA, std::string("cudaGetSymbolAddress of the attention scratch: ") +
                                  cudaGetErrorString(e));
        g_noalloc_addr[*device] = p;
    }
    return (unsigned char*)g_noalloc_addr[*device];
}

}  // namespace ab

using namespace ab;

// Validates the operands of the fused attention entry points and fills every AttnParams
// field except the scratch (part_o, part_ml, counters, flags).
static AttnParams attention_decode_operands(ab_tensor q, ab_tensor key_cache,
                                            ab_tensor value_cache, ab_tensor out, ab_tensor step,
                                            int sms) {
    expect_data("q", q);
    expect_data("key_cache", key_cache);
    expect_data("value_cache", value_cache);
    expect_data("out", out);
    expect_dtype("q", q, AB_F32);
    expect_rank_in("q", q, 2, 3);
    const uint32_t batch = q.rank == 3 ? q.dims[0] : 1;
    const uint32_t heads = q.dims[q.rank - 2], head = q.dims[q.rank - 1];
    expect_float("key_cache", key_cache);
    expect_dtype("value_cache", value_cache, key_cache.dtype);
    // [B, seq, kv, head] (a cache per row) or [seq, kv, head] (one cache: at batch 1, or
    // shared by rows that are positions of one sequence)
    const int cr = q.rank == 3 && key_cache.rank != 3 ? 4 : 3;
    expect_rank("key_cache", key_cache, cr);
    expect_rank("value_cache", value_cache, cr);
    for (int a = 0; a < cr; a++)
        if (value_cache.dims[a] != key_cache.dims[a])
            invalid("parameter `value_cache`: dims must match key_cache " + shape_str(key_cache));
    const int o = cr - 3;
    if (cr == 4 && key_cache.dims[0] < batch) expect_dim("key_cache", key_cache, 0, "batch", batch);
    const uint32_t seq = key_cache.dims[o], kv_heads = key_cache.dims[o + 1];
    expect_dim("key_cache", key_cache, o + 2, "head", head);
    expect_float("out", out);
    if (numel(out) != (uint64_t)batch * heads * head)
        invalid("parameter `out`: expected " + std::to_string((uint64_t)batch * heads * head) +
                " elements ([batch, heads * head]), got " + shape_str(out));
    expect_step(step, batch);
    if (!attention_fusable(heads, kv_heads, head, key_cache.dtype))
        invalid("attention: needs query_heads / kv_heads in {1, 2, 4, 8} and head * element "
                "size a multiple of 16 bytes, head <= 128");
    AttnParams p = {};
    p.q = (const float*)q.data;
    p.kcache = key_cache.data;
    p.vcache = value_cache.data;
    p.kv_dtype = key_cache.dtype;
    p.cache_stride = cr == 3 ? 0 : (uint64_t)seq * kv_heads * head;
    p.out = out.data;
    p.out_dtype = out.dtype;
    p.heads = heads;
    p.kv_heads = kv_heads;
    p.head = head;
    p.seq = seq;
    p.batch = batch;
    p.nsplit = attention_choose_splits(batch, kv_heads, seq, sms, 256);
    p.min_chunk = attention_min_chunk();
    p.step = (const Step*)step.data;
    return p;
}

extern "C" int ab_kernel_attention_decode(ab_scheme* s, ab_tensor q, ab_tensor key_cache,
                                          ab_tensor value_cache, ab_tensor out, ab_tensor step) {
    return guard([&] {
        if (!s) fail(AB_ERR_ARGUMENT, "null scheme");
        if (!s->rt) fail(AB_ERR_ARGUMENT, "attention_decode: the scheme needs a runtime (it "
                                          "allocates the split scratch)");
        AttnParams p = attention_decode_operands(q, key_cache, value_cache, out, step,
                                                 s->rt->sm_count);
        uint64_t floats = 0, tickets = 0;
        attention_scratch_size(p.batch, p.heads, p.head, p.nsplit, &floats, &tickets);
        // room for the prompt kernel's two halves too (rows over one shared cache)
        floats = std::max<uint64_t>(floats, (uint64_t)p.batch * p.heads * 2 * (p.head + 2));
        tickets = (uint64_t)p.batch * p.kv_heads;
        s->rt->activate();
        void* part = nullptr;
        void* counters = nullptr;
        cuda_check(cudaMalloc(&part, std::max<uint64_t>(floats, 1) * 4), "cudaMalloc");
        if (cudaMalloc(&counters, tickets * 4) != cudaSuccess ||
            cudaMemset(counters, 0, tickets * 4) != cudaSuccess) {
            cudaGetLastError();
            cudaFree(part);
            if (counters) cudaFree(counters);
            fail(AB_ERR_CUDA, "attention_decode: scratch allocation failed");
        }
        s->owned.push_back(part);
        s->owned.push_back(counters);
        p.part_o = (float*)part;
        p.part_ml = (float*)part + (uint64_t)p.batch * p.heads * p.nsplit * p.head;
        p.counters = (uint32_t*)counters;
        p.part_cap = floats;
        p.flags = s->rt->flags;
        record_attention(s, "attn_decode", p);
    });
}

extern "C" int ab_attention_decode_noalloc(void* stream, ab_tensor q, ab_tensor key_cache,
                                           ab_tensor value_cache, ab_tensor out, ab_tensor step) {
    return guard([&] {
        int device = 0;
        cuda_check(cudaGetDevice(&device), "query device");
        int sms = 148;
        cuda_check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device),
                   "query SM count");
        AttnParams p = attention_decode_operands(q, key_cache, value_cache, out, step, sms);

        // this entry launches directly: refuse anything that is not device memory first
        for (const ab_tensor* t : {&q, &key_cache, &value_cache, &out, &step}) {
            cudaPointerAttributes attr;
            if (cudaPointerGetAttributes(&attr, t->data) != cudaSuccess ||
                (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged)) {
                cudaGetLastError();
                fail(AB_ERR_ARGUMENT, "ab_attention_decode_noalloc: a tensor pointer is not "
                                      "device memory");
            }
        }
        unsigned char* base = noalloc_scratch(&device);
        uint64_t floats = 0, tickets = 0;
        attention_scratch_size(p.batch, p.heads, p.head, p.nsplit, &floats, &tickets);
        tickets = (uint64_t)p.batch * p.kv_heads;
        if (floats > kNoAllocFloats || tickets > kNoAllocTickets)
            fail(AB_ERR_ARGUMENT,
                 "ab_attention_decode_noalloc: this shape needs " + std::to_string(floats * 4) +
                     " bytes of split partials and " + std::to_string(tickets) +
                     " tickets; the static scratch holds " + std::to_string(kNoAllocFloats * 4) +
                     " bytes and " + std::to_string(kNoAllocTickets) + " tickets");
        p.part_o = (float*)base;
        p.part_ml = (float*)base + (uint64_t)p.batch * p.heads * p.nsplit * p.head;
        p.counters = (uint32_t*)(base + kNoAllocFloats * 4);
        p.flags = (uint32_t*)(base + kNoAllocFloats * 4 + (uint64_t)kNoAllocTickets * 4);

        cudaStream_t st = (cudaStream_t)stream;
        // tickets must start at zero; the kernel resets them, but a failed earlier call
        // could have left them set
        cuda_check(cudaMemsetAsync(p.counters, 0, tickets * 4, st), "clear tickets");
        // record into a throw-away list of launch closures, then launch them directly
        ab_scheme tmp;
        record_attention(&tmp, "attn_decode_noalloc", p);
        for (auto& n : tmp.nodes) cuda_check(n.launch(st), "attention launch");
    });
}

// The flag word the allocation-free attention raises (a position >= seq, a bounded wait that
// ran out) is sticky across calls: this reads it after `stream` drains, clears it, and turns
// a raised flag into AB_ERR_DEVICE. Copies through host stack memory; allocates nothing.
extern "C" int ab_attention_decode_noalloc_status(void* stream, uint32_t* flags_out) {
    return guard([&] {
        if (flags_out) *flags_out = 0;
        int device = 0;
        unsigned char* base = noalloc_scratch(&device);
        uint32_t* flags = (uint32_t*)(base + kNoAllocFloats * 4 + (uint64_t)kNoAllocTickets * 4);
        cudaStream_t st = (cudaStream_t)stream;
        uint32_t f = 0;
        cuda_check(cudaMemcpyAsync(&f, flags, 4, cudaMemcpyDeviceToHost, st), "read flags");
        cuda_check(cudaMemsetAsync(flags, 0, 4, st), "clear flags");
        cuda_check(cudaStreamSynchronize(st), "synchronize");
        if (flags_out) *flags_out = f;
        if (f) fail(AB_ERR_DEVICE, "ab_attention_decode_noalloc: " + device_flag_message(f));
    });
}
