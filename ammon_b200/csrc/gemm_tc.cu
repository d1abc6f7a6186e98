// Tensor-core decode GEMM for batches above the GEMV's range: out[b, r] = W[r, :] . X[b, :]
// with W the (virtual) weight matrix and X the batch of bf16 activations. It replaces
// Goldy's matmul_into (src/kernels.rs:518-528) at batch >= 5 and keeps the GEMV's fused
// epilogues (RoPE + K/V append, SwiGLU, residual add).
//
// Design (B200, sm_100a):
//  - One CTA computes a 128-row tile of W against all (padded) batch columns BN over a
//    range of 64-element k-blocks; tiles x k-splits cover the matrix, sized to one wave.
//  - Warp-specialised: thread 0 issues TMA loads (W tile 128 x 64, X tile BN x 64, both
//    K-major with the 128-byte swizzle, each CTA loading its own copy) into a
//    multi-stage ring guarded by full/empty mbarriers; thread 32 issues
//    tcgen05.mma.cta_group::1.kind::f16 (bf16 x bf16 -> f32) into a TMEM accumulator of BN
//    columns and commits each stage back to its empty barrier; all four warps then read
//    their 32 TMEM lanes with tcgen05.ld.
//  - TMEM is allocated only after griddepcontrol.wait, so a successor launched early by
//    programmatic dependent launch never holds TMEM that this kernel's later CTAs need.
//  - Split-K partials go to an L2-resident fp32 workspace; a second kernel folds them in
//    split order and applies the epilogue.
//  - fp32 weights take the same path on the tf32 tensor cores with three products per
//    k-step (3xTF32): every value v is split exactly into hi = v with its low 13 mantissa
//    bits cleared and lo = v - hi, and D += Wlo.Xhi + Whi.Xlo + Whi.Xhi keeps the error of
//    each product near 2^-22 relative, inside the fp32 parity bar. Activations are split
//    once per launch by the kernel that normalises them; weight tiles are split in shared
//    memory after they land, so the weights stay plain fp32 tensors in HBM.
//  - Every mbarrier wait is bounded (%globaltimer); a wait that runs out raises the device
//    flag, and the CTA still releases its TMEM.
#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "internal.h"
#include "ops.h"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace ab {

constexpr int kTcThreads = 128;
constexpr int kTcBM = 128;
constexpr int kTcBK = 64;  // bf16 elements per k-block: one 128-byte swizzled row
constexpr int kTcMaxStages = 8;
constexpr int kTfBK = 32;          // fp32 elements per k-block: one 128-byte swizzled row
constexpr int kTfThreads = 192;    // producer warp, MMA warp, 4 split/epilogue warps

// High part of the exact split v = hi + lo: v with its 13 low mantissa bits cleared (a
// tf32 value). lo = v - hi is exact in fp32 and carries the cleared bits.
__device__ __forceinline__ float tf32_hi(float v) {
    return __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
}

// Named barrier of the 128 epilogue threads (the four warps that own the TMEM lanes).
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// ---- epilogue on a chunk of 16 batch columns held by the thread of TMEM lane `row` ------------
template <int EPI>
__device__ __forceinline__ void tc_epilogue_chunk(const GemmTcParams& p, uint32_t tile,
                                                  uint32_t row, uint32_t c0, const float* v,
                                                  float* xch) {
    const uint32_t live = p.nb > c0 ? min(16u, p.nb - c0) : 0u;
    if (EPI == kEpiSwiglu) {
        // tile rows 0-63 are w1 rows tile*64 + row, rows 64-127 the matching w3 rows. Both
        // halves go through shared memory so that all 128 threads share the SwiGLU math:
        // thread `row` finishes unit row % 64 for 8 of the 16 columns.
        float* x0 = xch;            // [16][64] w1 products
        float* x1 = xch + 16 * 64;  // [16][64] w3 products
        float* xs = row < 64 ? x0 + row : x1 + (row - 64);
#pragma unroll
        for (int j = 0; j < 16; j++) xs[j * 64] = v[j];
        epi_sync();
        const uint32_t uu = row % 64, jb = (row / 64) * 8;
        const uint32_t u = tile * 64 + uu;
#pragma unroll
        for (int jj = 0; jj < 8; jj++) {
            const uint32_t j = jb + jj;
            if (j >= live) break;
            const float y0 = x0[j * 64 + uu], y1 = x1[j * 64 + uu];
            const float h = silu_mul(y0, y1);
            const uint64_t o = (uint64_t)(c0 + j) * p.out_stride + u;
            if (p.out_dtype == AB_F32) ((float*)p.out)[o] = h;
            else ((bf16*)p.out)[o] = __float2bfloat16_rn(h);
        }
        epi_sync();
        return;
    }
    float partner[16];
#pragma unroll
    for (int j = 0; j < 16; j++) partner[j] = __shfl_xor_sync(0xffffffffu, v[j], 1);
    const uint32_t r = tile * kTcBM + row;
    if (r >= p.n_rows) return;
    if (EPI == kEpiStore || EPI == kEpiResidual) {
#pragma unroll
        for (int j = 0; j < 16; j++) {
            if ((uint32_t)j >= live) break;
            const uint64_t o = (uint64_t)(c0 + j) * p.out_stride + r;
            if (EPI == kEpiResidual) ((float*)p.out)[o] += v[j];
            else if (p.out_dtype == AB_F32)
                ((float*)p.out)[o] = p.addend ? p.addend[o] + v[j] : v[j];
            else ((bf16*)p.out)[o] = __float2bfloat16_rn(v[j]);
        }
        return;
    }
    // kEpiQkv: the even row of each pair rotates / stores both
    if (r & 1) return;
#pragma unroll 4
    for (int j = 0; j < 16; j++) {
        if ((uint32_t)j >= live) break;
        const uint32_t b = c0 + j;
        const float y0 = v[j], y1 = partner[j];
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
            if (p.kv_dtype == AB_F32) {
                ((float*)p.kcache)[o] = y0 * c - y1 * s;
                ((float*)p.kcache)[o + 1] = y0 * s + y1 * c;
            } else {
                ((bf16*)p.kcache)[o] = __float2bfloat16_rn(y0 * c - y1 * s);
                ((bf16*)p.kcache)[o + 1] = __float2bfloat16_rn(y0 * s + y1 * c);
            }
        } else {
            const uint32_t i = r - p.qd - p.kvd;
            const uint64_t o = (uint64_t)b * p.cache_stride + (uint64_t)pos * p.kvd + i;
            if (p.kv_dtype == AB_F32) {
                ((float*)p.vcache)[o] = y0;
                ((float*)p.vcache)[o + 1] = y1;
            } else {
                ((bf16*)p.vcache)[o] = __float2bfloat16_rn(y0);
                ((bf16*)p.vcache)[o + 1] = __float2bfloat16_rn(y1);
            }
        }
    }
}

template <int EPI>
__global__ void __launch_bounds__(kTcThreads, 1)
    gemm_tc_kernel(const GemmTcParams p, const __grid_constant__ CUtensorMap ta0,
                   const __grid_constant__ CUtensorMap ta1, const __grid_constant__ CUtensorMap ta2,
                   const __grid_constant__ CUtensorMap tb) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t full_bar[kTcMaxStages];
    __shared__ __align__(8) uint64_t empty_bar[kTcMaxStages];
    __shared__ __align__(8) uint64_t done_bar;
    __shared__ uint32_t tmem_slot;
    __shared__ int sm_last;
    __shared__ int sm_ok;
    unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const uint32_t a_bytes = kTcBM * 128;
    const uint32_t stage_bytes = a_bytes + p.bn * 128;
    float* xch = (float*)(smem + (size_t)p.stages * stage_bytes);  // [2][16][64]
    const uint32_t tile = blockIdx.x, split = blockIdx.y;
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t kb0 = (uint32_t)((uint64_t)split * p.kblocks / p.ksplit);
    const uint32_t kb1 = (uint32_t)((uint64_t)(split + 1) * p.kblocks / p.ksplit);
    const uint32_t nk = kb1 - kb0;
    // each tile walks its k-blocks from its own starting block, so the CTAs of a launch
    // read different activation blocks at any moment instead of all the same L2 lines
    const uint32_t rot = nk ? (tile * p.krot) % nk : 0;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < p.stages; s++) {
            mbar_init(smem_u32(&full_bar[s]), 1);
            mbar_init(smem_u32(&empty_bar[s]), 1);
        }
        mbar_init(smem_u32(&done_bar), 1);
        fence_barrier_init();
        sm_ok = 1;
    }
    // activations come from the previous kernel, and TMEM is taken only after it finished
    pdl_wait();
    if (warp == 0) tmem_alloc(smem_u32(&tmem_slot), p.tmem_cols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;

    // Roles: lane 0 of warp 0 issues the TMA loads, lane 0 of warp 1 the MMAs. The other lanes
    // of those warps park at __syncwarp until their lane 0 is done: spinning on the done
    // barrier in the same warp would take issue turns (and mbarrier suspends) from it.
    if (warp == 0) {
        if (lane == 0) {
        // TMA producer: the W map and row of this tile are fixed; stage, phase and k-block
        // advance as counters (no divisions in the loop)
        const CUtensorMap* wmap = &ta0;
        int32_t wy = (int32_t)(tile * kTcBM);
        if (p.interleave) {
            wy = (int32_t)(tile * 64);
        } else if (tile >= p.seg_tiles[0] + p.seg_tiles[1]) {
            wmap = &ta2;
            wy = (int32_t)((tile - p.seg_tiles[0] - p.seg_tiles[1]) * kTcBM);
        } else if (tile >= p.seg_tiles[0]) {
            wmap = &ta1;
            wy = (int32_t)((tile - p.seg_tiles[0]) * kTcBM);
        }
        const uint32_t smem0 = smem_u32(smem);
        uint32_t s = 0, ph = 0, kb = kb0 + rot;
        for (uint32_t i = 0; i < nk; i++) {
            if (i >= p.stages && !mbar_wait_bounded(smem_u32(&empty_bar[s]), ph ^ 1, p.flags)) {
                sm_ok = 0;
                break;
            }
            const int32_t kx = (int32_t)(kb * kTcBK);
            const uint32_t bar = smem_u32(&full_bar[s]);
            const uint32_t a = smem0 + s * stage_bytes;
            mbar_arrive_expect_tx(bar, stage_bytes);
            tma_load_2d(a, wmap, kx, wy, bar);
            if (p.interleave) tma_load_2d(a + 64 * 128, &ta1, kx, wy, bar);
            tma_load_2d(a + a_bytes, &tb, kx, 0, bar);
            if (++kb == kb1) kb = kb0;
            if (++s == p.stages) {
                s = 0;
                ph ^= 1;
            }
        }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
        // MMA issuer: descriptors of a stage's operands advance by 32 bytes (2 in the
        // descriptor's address field) per 16-element k-step
        const uint32_t idesc = tc_idesc_bf16(kTcBM, p.bn);
        const uint32_t smem0 = smem_u32(smem);
        uint32_t s = 0, ph = 0;
        for (uint32_t i = 0; i < nk; i++) {
            if (!mbar_wait_bounded(smem_u32(&full_bar[s]), ph, p.flags)) {
                sm_ok = 0;
                break;
            }
            tc_fence_after();
            const uint32_t a = smem0 + s * stage_bytes;
            const uint64_t da = sw128_desc(a), db = sw128_desc(a + a_bytes);
#pragma unroll
            for (uint32_t k = 0; k < kTcBK / 16; k++)
                tc_mma_bf16(tmem, da + 2 * k, db + 2 * k, idesc, (i | k) != 0);
            tc_commit(smem_u32(&empty_bar[s]));
            if (++s == p.stages) {
                s = 0;
                ph ^= 1;
            }
        }
        tc_commit(smem_u32(&done_bar));
        }
        __syncwarp();
    }
    const bool got = mbar_wait_bounded(smem_u32(&done_bar), 0, p.flags);
    tc_fence_after();
    __syncthreads();
    const bool ok = __syncthreads_and(got && sm_ok != 0);
    pdl_trigger();

    if (ok) {
        const uint32_t row = warp * 32 + lane;  // TMEM lane = tile row
        const uint32_t taddr = tmem + ((warp * 32u) << 16);
        if (p.ksplit == 1) {
            for (uint32_t c0 = 0; c0 < p.bn; c0 += 16) {
                float v[16];
                tmem_ld16(taddr + c0, v);
                tc_epilogue_chunk<EPI>(p, tile, row, c0, v, xch);
            }
        } else {
            // partial of this k-split; splitk_epilogue_kernel folds the splits
            float* ws = p.ws + ((size_t)split * p.tiles + tile) * p.bn * kTcBM;
            for (uint32_t c0 = 0; c0 < p.bn; c0 += 16) {
                float v[16];
                tmem_ld16(taddr + c0, v);
#pragma unroll
                for (int j = 0; j < 16; j++) ws[(size_t)(c0 + j) * kTcBM + row] = v[j];
            }
        }
    } else {
        if (threadIdx.x == 0) {
            atomicOr(p.flags, kFlagWaitTimeout);
            // let the committed MMAs drain before TMEM is released
            mbar_wait_bounded(smem_u32(&done_bar), 0, p.flags);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, p.tmem_cols);
    }
}

// fp32 weights on the tf32 pipe (3xTF32). Stage s holds [W | W lo | X hi | X lo], each a
// K-major 128-byte-swizzled tile of 32 fp32 per row. Warp 0 (lane 0) loads W, X hi and
// X lo by TMA; warps 2-5 split the landed W tile in place into hi and lo (fence to the
// async proxy, then every thread arrives on split_bar[s]); warp 1 (lane 0) issues three
// tf32 MMAs per 8-element k-step and commits the stage back to the producer. Warps 2-5
// then own TMEM lanes 32 * (warp % 4) .. + 31 for the epilogue.
template <int EPI>
__global__ void __launch_bounds__(kTfThreads, 1)
    gemm_tf32x3_kernel(const GemmTcParams p, const __grid_constant__ CUtensorMap ta0,
                       const __grid_constant__ CUtensorMap ta1,
                       const __grid_constant__ CUtensorMap ta2,
                       const __grid_constant__ CUtensorMap tb_hi,
                       const __grid_constant__ CUtensorMap tb_lo) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t full_bar[kTcMaxStages];
    __shared__ __align__(8) uint64_t split_bar[kTcMaxStages];
    __shared__ __align__(8) uint64_t empty_bar[kTcMaxStages];
    __shared__ __align__(8) uint64_t done_bar;
    __shared__ uint32_t tmem_slot;
    __shared__ int sm_ok;
    unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const uint32_t a_bytes = kTcBM * 128;
    const uint32_t b_bytes = p.bn * 128;
    const uint32_t stage_bytes = 2 * a_bytes + 2 * b_bytes;
    float* xch = (float*)(smem + (size_t)p.stages * stage_bytes);  // [2][16][64]
    const uint32_t tile = blockIdx.x, split = blockIdx.y;
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t kb0 = (uint32_t)((uint64_t)split * p.kblocks / p.ksplit);
    const uint32_t kb1 = (uint32_t)((uint64_t)(split + 1) * p.kblocks / p.ksplit);
    const uint32_t nk = kb1 - kb0;
    // each tile walks its k-blocks from its own starting block, so the CTAs of a launch
    // read different activation blocks at any moment instead of all the same L2 lines
    const uint32_t rot = nk ? (tile * p.krot) % nk : 0;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < p.stages; s++) {
            mbar_init(smem_u32(&full_bar[s]), 1);
            mbar_init(smem_u32(&split_bar[s]), 128);
            mbar_init(smem_u32(&empty_bar[s]), 1);
        }
        mbar_init(smem_u32(&done_bar), 1);
        fence_barrier_init();
        sm_ok = 1;
    }
    pdl_wait();
    if (warp == 0) tmem_alloc(smem_u32(&tmem_slot), p.tmem_cols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;

    // roles as in gemm_tc_kernel: lanes 1-31 of the producer and MMA warps park at __syncwarp
    if (warp == 0) {
        if (lane == 0) {
        // TMA producer (counters as in gemm_tc_kernel)
        const CUtensorMap* wmap = &ta0;
        int32_t wy = (int32_t)(tile * kTcBM);
        if (p.interleave) {
            wy = (int32_t)(tile * 64);
        } else if (tile >= p.seg_tiles[0] + p.seg_tiles[1]) {
            wmap = &ta2;
            wy = (int32_t)((tile - p.seg_tiles[0] - p.seg_tiles[1]) * kTcBM);
        } else if (tile >= p.seg_tiles[0]) {
            wmap = &ta1;
            wy = (int32_t)((tile - p.seg_tiles[0]) * kTcBM);
        }
        const uint32_t smem0 = smem_u32(smem);
        uint32_t s = 0, ph = 0, kb = kb0 + rot;
        for (uint32_t i = 0; i < nk; i++) {
            if (i >= p.stages && !mbar_wait_bounded(smem_u32(&empty_bar[s]), ph ^ 1, p.flags)) {
                sm_ok = 0;
                break;
            }
            const int32_t kx = (int32_t)(kb * kTfBK);
            const uint32_t bar = smem_u32(&full_bar[s]);
            const uint32_t a = smem0 + s * stage_bytes;
            const uint32_t b = a + 2 * a_bytes;
            mbar_arrive_expect_tx(bar, a_bytes + 2 * b_bytes);
            tma_load_2d(a, wmap, kx, wy, bar);
            if (p.interleave) tma_load_2d(a + 64 * 128, &ta1, kx, wy, bar);
            tma_load_2d(b, &tb_hi, kx, 0, bar);
            tma_load_2d(b + b_bytes, &tb_lo, kx, 0, bar);
            if (++kb == kb1) kb = kb0;
            if (++s == p.stages) {
                s = 0;
                ph ^= 1;
            }
        }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
        // MMA issuer: small products first, then Whi.Xhi
        const uint32_t idesc = tc_idesc_tf32(kTcBM, p.bn);
        const uint32_t smem0 = smem_u32(smem);
        uint32_t s = 0, ph = 0;
        for (uint32_t i = 0; i < nk; i++) {
            if (!mbar_wait_bounded(smem_u32(&split_bar[s]), ph, p.flags)) {
                sm_ok = 0;
                break;
            }
            tc_fence_after();
            const uint32_t whi = smem0 + s * stage_bytes;
            const uint64_t dwhi = sw128_desc(whi), dwlo = sw128_desc(whi + a_bytes);
            const uint64_t dxhi = sw128_desc(whi + 2 * a_bytes);
            const uint64_t dxlo = sw128_desc(whi + 2 * a_bytes + b_bytes);
#pragma unroll
            for (uint32_t k = 0; k < kTfBK / 8; k++) {
                tc_mma_tf32(tmem, dwlo + 2 * k, dxhi + 2 * k, idesc, (i | k) != 0);
                tc_mma_tf32(tmem, dwhi + 2 * k, dxlo + 2 * k, idesc, 1);
                tc_mma_tf32(tmem, dwhi + 2 * k, dxhi + 2 * k, idesc, 1);
            }
            tc_commit(smem_u32(&empty_bar[s]));
            if (++s == p.stages) {
                s = 0;
                ph ^= 1;
            }
        }
        tc_commit(smem_u32(&done_bar));
        }
        __syncwarp();
    } else if (warp >= 2) {
        // split the landed W tile: hi in place, lo beside it (same swizzled offsets)
        const uint32_t t = threadIdx.x - 64;
        for (uint32_t i = 0; i < nk; i++) {
            const uint32_t s = i % p.stages;
            if (!mbar_wait_bounded(smem_u32(&full_bar[s]), (i / p.stages) & 1, p.flags)) {
                sm_ok = 0;
                break;
            }
            float4* w = (float4*)(smem + (size_t)s * stage_bytes);
            float4* wl = w + a_bytes / 16;
#pragma unroll 4
            for (uint32_t j = t; j < a_bytes / 16; j += 128) {
                const float4 v = w[j];
                const float4 h = make_float4(tf32_hi(v.x), tf32_hi(v.y), tf32_hi(v.z),
                                             tf32_hi(v.w));
                w[j] = h;
                wl[j] = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
            }
            fence_proxy_async_smem();
            mbar_arrive(smem_u32(&split_bar[s]));
        }
    }
    const bool got = mbar_wait_bounded(smem_u32(&done_bar), 0, p.flags);
    tc_fence_after();
    const bool ok = __syncthreads_and(got && sm_ok != 0);
    pdl_trigger();

    if (ok) {
        if (warp >= 2) {
            const uint32_t quarter = warp & 3;
            const uint32_t row = quarter * 32 + lane;  // TMEM lane = tile row
            const uint32_t taddr = tmem + ((quarter * 32u) << 16);
            if (p.ksplit == 1) {
                for (uint32_t c0 = 0; c0 < p.bn; c0 += 16) {
                    float v[16];
                    tmem_ld16(taddr + c0, v);
                    tc_epilogue_chunk<EPI>(p, tile, row, c0, v, xch);
                }
            } else {
                float* ws = p.ws + ((size_t)split * p.tiles + tile) * p.bn * kTcBM;
                for (uint32_t c0 = 0; c0 < p.bn; c0 += 16) {
                    float v[16];
                    tmem_ld16(taddr + c0, v);
#pragma unroll
                    for (int j = 0; j < 16; j++) ws[(size_t)(c0 + j) * kTcBM + row] = v[j];
                }
            }
        }
    } else if (threadIdx.x == 0) {
        atomicOr(p.flags, kFlagWaitTimeout);
        mbar_wait_bounded(smem_u32(&done_bar), 0, p.flags);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, p.tmem_cols);
    }
}

// Exact tf32 split of fp32 activation rows, optionally RMS-normalised first
// (src/kernels.rs:75-101: o = w * (ss * x), ss = 1 / sqrt(mean(x^2) + eps)):
// hi[r, k] = tf32_hi(o), lo[r, k] = o - hi[r, k]. One 256-thread block per row.
template <bool NORM, typename WT>
__global__ void __launch_bounds__(256)
    split_rows_tf32_kernel(const float* __restrict__ x, uint32_t x_stride,
                           const WT* __restrict__ w, float* __restrict__ hi,
                           float* __restrict__ lo, uint32_t dim, float eps) {
    pdl_wait();
    const float* xr = x + (uint64_t)blockIdx.x * x_stride;
    float scale = 1.0f;
    if (NORM) {
        __shared__ float red[8];
        float ss = 0.0f;
        for (uint32_t k = threadIdx.x; k < dim; k += 256) ss = fmaf(xr[k], xr[k], ss);
        ss = warp_sum(ss);
        if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = ss;
        __syncthreads();
        float t = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; i++) t += red[i];
        scale = 1.0f / sqrtf(t / (float)dim + eps);
    }
    float* hr = hi + (uint64_t)blockIdx.x * dim;
    float* lr = lo + (uint64_t)blockIdx.x * dim;
    for (uint32_t k = threadIdx.x; k < dim; k += 256) {
        const float v = NORM ? to_f32(w[k]) * (scale * xr[k]) : xr[k];
        const float h = tf32_hi(v);
        hr[k] = h;
        lr[k] = v - h;
    }
    pdl_trigger();
}

// RMSNorm of fp32 rows into bf16 rows (the GEMM's activation operand): o = w * (ss * x),
// ss = 1 / sqrt(mean(x^2) + eps) (src/kernels.rs:75-101). One 256-thread block per row.
template <typename WT>
__global__ void __launch_bounds__(256)
    rmsnorm_rows_bf16_kernel(const float* __restrict__ x, const WT* __restrict__ w,
                             bf16* __restrict__ out, uint32_t dim, float eps) {
    pdl_wait();
    __shared__ float red[8];
    const float* xr = x + (uint64_t)blockIdx.x * dim;
    bf16* orow = out + (uint64_t)blockIdx.x * dim;
    float ss = 0.0f;
    for (uint32_t k = threadIdx.x; k < dim; k += 256) ss = fmaf(xr[k], xr[k], ss);
    ss = warp_sum(ss);
    if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = ss;
    __syncthreads();
    float t = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) t += red[i];
    const float scale = 1.0f / sqrtf(t / (float)dim + eps);
    for (uint32_t k = threadIdx.x; k < dim; k += 256)
        orow[k] = __float2bfloat16_rn(to_f32(w[k]) * (scale * xr[k]));
    pdl_trigger();
}

// Folds the k-split partials of the tensor-core GEMM (ws[split][tile][col][row]) in split
// order and applies the epilogue. Thread -> (column, 4 consecutive rows) of a tile: float4
// loads of every split are independent, and each thread holds whole row pairs.
// Grid (tiles, ceil(bn / 8)), 256 threads = 8 columns x 32 row quads.
template <int EPI>
__global__ void __launch_bounds__(256) splitk_epilogue_kernel(const GemmTcParams p) {
    // the GEMM lets this kernel launch before its epilogue stored the partials: wait for it
    pdl_wait();
    const uint32_t tile = blockIdx.x;
    const uint32_t col = blockIdx.y * 8 + threadIdx.x / 32;
    const uint32_t quad = threadIdx.x % 32;
    const uint32_t r4 = quad * 4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (col < p.bn) {
        const size_t stride = (size_t)p.tiles * p.bn * kTcBM;
        const float* base = p.ws + ((size_t)tile * p.bn + col) * kTcBM + r4;
        uint32_t sp = 0;
        for (; sp + 4 <= p.ksplit; sp += 4) {
            const float4 a = __ldcg((const float4*)(base + sp * stride));
            const float4 b = __ldcg((const float4*)(base + (sp + 1) * stride));
            const float4 c = __ldcg((const float4*)(base + (sp + 2) * stride));
            const float4 d = __ldcg((const float4*)(base + (sp + 3) * stride));
            acc.x += a.x; acc.y += a.y; acc.z += a.z; acc.w += a.w;
            acc.x += b.x; acc.y += b.y; acc.z += b.z; acc.w += b.w;
            acc.x += c.x; acc.y += c.y; acc.z += c.z; acc.w += c.w;
            acc.x += d.x; acc.y += d.y; acc.z += d.z; acc.w += d.w;
        }
        for (; sp < p.ksplit; sp++) {
            const float4 a = __ldcg((const float4*)(base + sp * stride));
            acc.x += a.x; acc.y += a.y; acc.z += a.z; acc.w += a.w;
        }
    }
    const float v[4] = {acc.x, acc.y, acc.z, acc.w};
    if (EPI == kEpiSwiglu) {
        // rows 0-63 (w1) pair with rows 64-127 (w3): quad k with quad k + 16
        float h3[4];
#pragma unroll
        for (int i = 0; i < 4; i++) h3[i] = __shfl_down_sync(0xffffffffu, v[i], 16);
        if (quad >= 16 || col >= p.nb) return;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t u = tile * 64 + r4 + i;
            const float h = silu_mul(v[i], h3[i]);
            const uint64_t o = (uint64_t)col * p.out_stride + u;
            if (p.out_dtype == AB_F32) ((float*)p.out)[o] = h;
            else ((bf16*)p.out)[o] = __float2bfloat16_rn(h);
        }
        return;
    }
    if (col >= p.nb) return;
#pragma unroll
    for (int i = 0; i < 4; i += 2) {
        const uint32_t r = tile * kTcBM + r4 + i;
        if (r >= p.n_rows) return;
        const float y0 = v[i], y1 = v[i + 1];
        const uint64_t o = (uint64_t)col * p.out_stride + r;
        if (EPI == kEpiResidual) {
            float* out = (float*)p.out;
            out[o] += y0;
            if (r + 1 < p.n_rows) out[o + 1] += y1;
        } else if (EPI == kEpiStore) {
            if (p.out_dtype == AB_F32) {
                const float a0 = p.addend ? p.addend[o] : 0.0f;
                ((float*)p.out)[o] = a0 + y0;
                if (r + 1 < p.n_rows)
                    ((float*)p.out)[o + 1] = (p.addend ? p.addend[o + 1] : 0.0f) + y1;
            } else {
                ((bf16*)p.out)[o] = __float2bfloat16_rn(y0);
                if (r + 1 < p.n_rows) ((bf16*)p.out)[o + 1] = __float2bfloat16_rn(y1);
            }
        } else {  // kEpiQkv
            const uint32_t pos = p.step[col].position;
            if (r < p.qd) {
                float c, s;
                rope_cos_sin(r, p.head, pos, p.theta, &c, &s);
                float* q = p.q + (uint64_t)col * p.qd + r;
                q[0] = y0 * c - y1 * s;
                q[1] = y0 * s + y1 * c;
            } else if (pos >= p.seq) {
                if (r == p.qd) atomicOr(p.flags, kFlagPositionRange);
            } else if (r < p.qd + p.kvd) {
                const uint32_t k = r - p.qd;
                float c, s;
                rope_cos_sin(k, p.head, pos, p.theta, &c, &s);
                const uint64_t ko = (uint64_t)col * p.cache_stride + (uint64_t)pos * p.kvd + k;
                if (p.kv_dtype == AB_F32) {
                    ((float*)p.kcache)[ko] = y0 * c - y1 * s;
                    ((float*)p.kcache)[ko + 1] = y0 * s + y1 * c;
                } else {
                    ((bf16*)p.kcache)[ko] = __float2bfloat16_rn(y0 * c - y1 * s);
                    ((bf16*)p.kcache)[ko + 1] = __float2bfloat16_rn(y0 * s + y1 * c);
                }
            } else {
                const uint32_t k = r - p.qd - p.kvd;
                const uint64_t vo = (uint64_t)col * p.cache_stride + (uint64_t)pos * p.kvd + k;
                if (p.kv_dtype == AB_F32) {
                    ((float*)p.vcache)[vo] = y0;
                    ((float*)p.vcache)[vo + 1] = y1;
                } else {
                    ((bf16*)p.vcache)[vo] = __float2bfloat16_rn(y0);
                    ((bf16*)p.vcache)[vo + 1] = __float2bfloat16_rn(y1);
                }
            }
        }
    }
}

// A residual k-split fold and the RMSNorm of the rows it updates, in one launch: the norm that
// stages the next projection's operand reads the residual stream the fold just wrote, so
// instead of a fold kernel and a norm kernel, one CTA per row b of x (1) folds the partials of
// its row in split order and adds them to x (the arithmetic of
// splitk_epilogue_kernel<kEpiResidual>), keeping the new row in shared memory, then (2) takes
// its RMSNorm exactly as rmsnorm_rows_bf16_kernel / split_rows_tf32_kernel do (256 lanes, the
// same order of sums), writing the bf16 operand or its exact tf32 halves.
// Requirements (checked when recording): dim % 4 == 0, dim <= kFoldNormMaxDim, x rows of
// stride dim, the fold's rows cover [0, dim).
constexpr uint32_t kFoldNormThreads = 1024;
constexpr uint32_t kFoldNormMaxDim = 8192;  // the row staged in shared memory (32 KB)

template <typename WT, bool TF32>
__global__ void __launch_bounds__(kFoldNormThreads)
    splitk_residual_norm_kernel(const float* __restrict__ ws, uint32_t tiles, uint32_t bn,
                                uint32_t ksplit, float* __restrict__ x, uint32_t dim,
                                const WT* __restrict__ w, float eps, bf16* __restrict__ out,
                                float* __restrict__ hi, float* __restrict__ lo) {
    // the GEMM lets this kernel launch before its epilogue stored the partials: wait for it
    pdl_wait();
    __shared__ __align__(16) float xs[kFoldNormMaxDim];
    __shared__ float red[8];
    const uint32_t b = blockIdx.x;
    float* xr = x + (uint64_t)b * dim;
    const size_t stride = (size_t)tiles * bn * kTcBM;
    // (1) thread -> 4 consecutive rows of one tile: a float4 of every split, summed in order
    for (uint32_t k = threadIdx.x * 4; k < dim; k += kFoldNormThreads * 4) {
        const uint32_t tile = k / kTcBM, r = k % kTcBM;
        const float* base = ws + ((size_t)tile * bn + b) * kTcBM + r;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        uint32_t sp = 0;
        for (; sp + 4 <= ksplit; sp += 4) {  // four loads in flight, added in split order
            const float4 a = __ldcg((const float4*)(base + sp * stride));
            const float4 c = __ldcg((const float4*)(base + (sp + 1) * stride));
            const float4 d = __ldcg((const float4*)(base + (sp + 2) * stride));
            const float4 e = __ldcg((const float4*)(base + (sp + 3) * stride));
            acc.x += a.x; acc.y += a.y; acc.z += a.z; acc.w += a.w;
            acc.x += c.x; acc.y += c.y; acc.z += c.z; acc.w += c.w;
            acc.x += d.x; acc.y += d.y; acc.z += d.z; acc.w += d.w;
            acc.x += e.x; acc.y += e.y; acc.z += e.z; acc.w += e.w;
        }
        for (; sp < ksplit; sp++) {
            const float4 a = __ldcg((const float4*)(base + sp * stride));
            acc.x += a.x; acc.y += a.y; acc.z += a.z; acc.w += a.w;
        }
        const float4 xo = *(const float4*)(xr + k);
        const float4 xn = make_float4(xo.x + acc.x, xo.y + acc.y, xo.z + acc.z, xo.w + acc.w);
        *(float4*)(xr + k) = xn;
        *(float4*)(xs + k) = xn;
    }
    __syncthreads();
    // (2) ss over the 256 lanes k = t, t + 256, ... then the eight warps in order
    if (threadIdx.x < 256) {
        float ss = 0.0f;
        for (uint32_t k = threadIdx.x; k < dim; k += 256) ss = fmaf(xs[k], xs[k], ss);
        ss = warp_sum(ss);
        if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = ss;
    }
    __syncthreads();
    float t = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) t += red[i];
    const float scale = 1.0f / sqrtf(t / (float)dim + eps);
    for (uint32_t k = threadIdx.x; k < dim; k += kFoldNormThreads) {
        const float v = to_f32(w[k]) * (scale * xs[k]);
        if (TF32) {
            const float h = tf32_hi(v);
            hi[(uint64_t)b * dim + k] = h;
            lo[(uint64_t)b * dim + k] = v - h;
        } else {
            out[(uint64_t)b * dim + k] = __float2bfloat16_rn(v);
        }
    }
    pdl_trigger();
}

// Fusion of a norm into the residual fold recorded just before it (AMMON_B200_FOLD_NORM=0
// keeps them apart; read at each record, so one process can record either form).
static bool fold_norm_enabled() {
    const char* e = std::getenv("AMMON_B200_FOLD_NORM");
    return !(e && e[0] == '0');
}

// The scheme's last node when it is a residual fold of exactly these rows of x (the rows the
// norm about to be recorded reads), else null.
static Node* fusable_fold(ab_scheme* s, const float* x, uint32_t x_stride, uint32_t rows,
                          uint32_t dim) {
    if (!fold_norm_enabled() || s->nodes.empty()) return nullptr;
    Node& n = s->nodes.back();
    const FoldInfo& f = n.fold;
    if (f.x != x || f.x_stride != dim || x_stride != dim || f.nb != rows || f.n_rows != dim ||
        (uint64_t)f.tiles * kTcBM < dim || dim % 4 || dim > kFoldNormMaxDim || f.ksplit < 2)
        return nullptr;
    return &n;
}

// Replaces the fold node's launch with the fused fold + norm (bf16 operand, or tf32 halves).
template <typename WT>
static void fuse_fold_norm(ab_scheme* s, Node* n, const char* label, const WT* w, float eps,
                           uint32_t dim, bf16* out, float* hi, float* lo) {
    const FoldInfo f = n->fold;
    const bool tf32 = out == nullptr;
    if (tf32)
        n->launch = [=](cudaStream_t st) {
            return launch(st, dim3(f.nb), dim3(kFoldNormThreads), 0, true,
                          splitk_residual_norm_kernel<WT, true>, f.ws, f.tiles, f.bn, f.ksplit,
                          f.x, dim, w, eps, (bf16*)nullptr, hi, lo);
        };
    else
        n->launch = [=](cudaStream_t st) {
            return launch(st, dim3(f.nb), dim3(kFoldNormThreads), 0, true,
                          splitk_residual_norm_kernel<WT, false>, f.ws, f.tiles, f.bn, f.ksplit,
                          f.x, dim, w, eps, out, (float*)nullptr, (float*)nullptr);
        };
    n->label += std::string("+") + label;
    n->fold = FoldInfo{};
    s->dirty = true;
}

GemmTcPlan gemm_tc_plan(uint32_t rows, uint32_t K, uint32_t batch, int sms, bool interleave,
                        bool f32) {
    GemmTcPlan pl = {};
    pl.bn = std::max(16u, (batch + 15) / 16 * 16);
    pl.tiles = interleave ? rows / 64 : (rows + kTcBM - 1) / kTcBM;
    pl.kblocks = K / (f32 ? kTfBK : kTcBK);
    // bf16: [W | X]; fp32: [W | W lo | X hi | X lo], 128 bytes per tile row
    const uint32_t stage_bytes = (kTcBM * 128 + pl.bn * 128) * (f32 ? 2 : 1);
    // two resident CTAs per SM where two stages each fit: one CTA's fill, epilogue and
    // tail overlap the other's main loop, which measured faster than one CTA with a deeper
    // ring at every batch width (128-row passes: 2 x 3 stages; 256: 2 x 2)
    uint32_t per_sm = 2;
    // tuning parameters (the results do not change): CTAs per SM and a stage cap
    if (const char* e = std::getenv("AMMON_B200_GEMM_PER_SM")) {
        const long v = std::atol(e);
        if (v >= 1 && v <= 4) per_sm = (uint32_t)v;
    }
    uint32_t max_stages = kTcMaxStages;
    if (const char* e = std::getenv("AMMON_B200_GEMM_STAGES")) {
        const long v = std::atol(e);
        if (v >= 2 && v <= kTcMaxStages) max_stages = (uint32_t)v;
    }
    // resident CTAs share 227 KB of shared memory (each also holds the 8 KB exchange buffer
    // and 1 KB of alignment slack) and the 512 TMEM columns
    uint32_t cols = 32;
    while (cols < pl.bn) cols <<= 1;
    while (per_sm > 1 && (per_sm * cols > 512 ||
                          per_sm * (2 * stage_bytes + 10u * 1024) > 226u * 1024))
        per_sm--;
    const uint32_t budget = per_sm == 1 ? 200u * 1024 : 220u * 1024 / per_sm - 10u * 1024;
    pl.stages = std::max(2u, std::min(max_stages, budget / stage_bytes));
    const uint32_t target = (uint32_t)std::max(sms, 1) * per_sm;
    uint32_t ks = (target + pl.tiles / 2) / std::max(pl.tiles, 1u);
    // fp32 k-blocks carry three MMAs each: two of them per split still hide the fill
    ks = std::min(ks, std::max(1u, pl.kblocks / (f32 ? 2 : 4)));
    if (const char* e = std::getenv("AMMON_B200_GEMM_MAX_KSPLIT")) {  // tuning parameter
        const long v = std::atol(e);
        if (v >= 1) ks = std::min(ks, (uint32_t)v);
    }
    pl.ksplit = std::max(1u, ks);
    // stagger of the tiles' first k-block (0 walks every tile from its first block; a
    // tuning parameter: the fp32 sums keep their per-tile order, in a rotated sequence)
    pl.krot = f32 ? 0 : 7;  // measured: +1% on bf16 batch-64 decode, -2.5% on 3xTF32 batch 256
    if (const char* e = std::getenv("AMMON_B200_GEMM_ROTATE")) pl.krot = (uint32_t)std::atol(e);
    pl.smem = (size_t)pl.stages * stage_bytes + 2 * 16 * 64 * 4 + 1024;
    pl.tmem_cols = cols;
    pl.ws_floats = pl.ksplit > 1 ? (uint64_t)pl.ksplit * pl.tiles * pl.bn * kTcBM : 0;
    return pl;
}

void gemm_tc_scratch(uint32_t max_tiles, uint32_t max_batch, int sms, uint64_t* ws_floats,
                     uint32_t* tickets) {
    // ksplit <= round(target / tiles) keeps ksplit * tiles <= target + tiles
    const uint32_t bn = std::max(16u, (max_batch + 15) / 16 * 16);
    const uint64_t target = (uint64_t)std::max(sms, 1) * 4;  // up to 4 resident CTAs per SM
    *ws_floats = (target + max_tiles) * (uint64_t)std::min(bn, 256u) * kTcBM;
    *tickets = max_tiles;
}

void alloc_tc_scratch(Runtime* rt, GemmScratch* g, uint32_t max_batch, uint32_t max_k,
                      uint32_t max_tiles) {
    if (max_batch <= kGemvMaxBatch) return;
    rt->activate();
    GemmScratch t;
    try {
        // bf16 activation rows, or the fp32 hi and lo halves of the 3xTF32 path
        t.xn_bytes = (uint64_t)max_batch * max_k * 8;
        cuda_check(cudaMalloc(&t.xn, t.xn_bytes), "cudaMalloc");
        cuda_check(cudaMemset(t.xn, 0, t.xn_bytes), "cudaMemset");
        gemm_tc_scratch(max_tiles, max_batch, rt->sm_count, &t.ws_floats, &t.tickets_n);
        cuda_check(cudaMalloc(&t.ws, t.ws_floats * 4), "cudaMalloc");
        cuda_check(cudaMalloc(&t.tickets, (size_t)t.tickets_n * 4), "cudaMalloc");
        cuda_check(cudaMemset(t.tickets, 0, (size_t)t.tickets_n * 4), "cudaMemset");
    } catch (...) {
        free_tc_scratch(&t);
        throw;
    }
    *g = t;
}

void free_tc_scratch(GemmScratch* g) {
    if (g->xn) cudaFree(g->xn);
    if (g->ws) cudaFree(g->ws);
    if (g->tickets) cudaFree(g->tickets);
    *g = GemmScratch();
}

void attach_tc_scratch(GemvParams* p, const GemmScratch& g) {
    p->xn = g.xn;
    p->xn_bytes = g.xn_bytes;
    p->ws = g.ws;
    p->ws_floats = g.ws_floats;
    p->tickets = g.tickets;
    p->tickets_n = g.tickets_n;
}

bool gemm_tc_fits(uint32_t rows, uint32_t K, uint32_t batch, bool interleave, bool f32) {
    if (batch == 0 || batch > 256 || K == 0 || K % (f32 ? kTfBK : kTcBK)) return false;
    // a single stacked segment may end in a partial tile: TMA fills the missing rows with
    // zeros and the epilogues skip rows >= n_rows
    return interleave ? rows % 64 == 0 : rows > 0;
}

template <int EPI>
static void add_gemm_tc(ab_scheme* s, const char* label, const GemmTcParams& p,
                        const CUtensorMap* maps, size_t smem, bool f32) {
    const CUtensorMap a0 = maps[0], a1 = maps[1], a2 = maps[2], b = maps[3], blo = maps[4];
    dim3 grid(p.tiles, p.ksplit);
    if (f32) {
        auto kern = gemm_tf32x3_kernel<EPI>;
        s->add(label, [=](cudaStream_t st) {
            cudaError_t e = cudaFuncSetAttribute(
                kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
            return launch(st, grid, dim3(kTfThreads), smem, true, kern, p, a0, a1, a2, b, blo);
        });
    } else {
        auto kern = gemm_tc_kernel<EPI>;
        s->add(label, [=](cudaStream_t st) {
            cudaError_t e = cudaFuncSetAttribute(
                kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
            return launch(st, grid, dim3(kTcThreads), smem, true, kern, p, a0, a1, a2, b);
        });
    }
    if (p.ksplit > 1) {
        auto fold = splitk_epilogue_kernel<EPI>;
        dim3 fgrid(p.tiles, (p.bn + 7) / 8);
        FoldInfo info;
        if (EPI == kEpiResidual) {
            info.ws = p.ws;
            info.x = (float*)p.out;
            info.tiles = p.tiles;
            info.bn = p.bn;
            info.ksplit = p.ksplit;
            info.nb = p.nb;
            info.n_rows = p.n_rows;
            info.x_stride = p.out_stride;
        }
        s->add_fold((std::string(label) + "_splitk").c_str(), [=](cudaStream_t st) {
            return launch(st, fgrid, dim3(256), 0, true, fold, p);
        }, info);
    }
}

void record_gemm_tc(ab_scheme* s, const char* label, GemmTcParams p, int32_t wdtype,
                    const void* const* segs, const uint32_t* seg_rows, int nseg, const void* x,
                    const void* x_lo, uint32_t x_stride, int epi) {
    const bool f32 = wdtype == AB_F32;
    if (f32 != (x_lo != nullptr))
        fail(AB_ERR_ARGUMENT, std::string(label) + ": fp32 GEMM needs the split activation");
    const int sms = s->rt ? s->rt->sm_count : 148;
    uint32_t rows = 0;
    for (int i = 0; i < nseg; i++) rows += seg_rows[i];
    if (p.interleave) rows = seg_rows[0];
    const GemmTcPlan pl = gemm_tc_plan(rows, p.K, p.nb, sms, p.interleave != 0, f32);
    p.bn = pl.bn;
    p.tiles = pl.tiles;
    p.kblocks = pl.kblocks;
    p.ksplit = pl.ksplit;
    p.stages = pl.stages;
    p.tmem_cols = pl.tmem_cols;
    p.krot = pl.krot;
    if (pl.ws_floats > p.ws_floats || (pl.ksplit > 1 && p.tickets_n < pl.tiles))
        fail(AB_ERR_ARGUMENT, std::string(label) + ": GEMM workspace too small");
    const int32_t dt = f32 ? AB_F32 : AB_BF16;
    const uint32_t esz = f32 ? 4 : 2;
    const uint32_t bk = f32 ? kTfBK : kTcBK;
    CUtensorMap maps[5];
    const uint32_t box_rows = p.interleave ? 64 : kTcBM;
    for (int i = 0; i < 3; i++) {
        const int j = i < nseg ? i : 0;
        p.seg_tiles[i] = i < nseg && !p.interleave ? (seg_rows[i] + kTcBM - 1) / kTcBM : 0;
        encode_tmap_2d(&maps[i], dt, segs[j], p.K, seg_rows[j], (uint64_t)p.K * esz, bk,
                       box_rows, 128);
    }
    encode_tmap_2d(&maps[3], dt, x, p.K, p.nb, (uint64_t)x_stride * esz, bk, pl.bn, 128);
    maps[4] = maps[3];
    if (f32)
        encode_tmap_2d(&maps[4], dt, x_lo, p.K, p.nb, (uint64_t)x_stride * esz, bk, pl.bn, 128);
    switch (epi) {
        case kEpiStore: return add_gemm_tc<kEpiStore>(s, label, p, maps, pl.smem, f32);
        case kEpiQkv: return add_gemm_tc<kEpiQkv>(s, label, p, maps, pl.smem, f32);
        case kEpiSwiglu: return add_gemm_tc<kEpiSwiglu>(s, label, p, maps, pl.smem, f32);
        case kEpiResidual: return add_gemm_tc<kEpiResidual>(s, label, p, maps, pl.smem, f32);
        default: fail(AB_ERR_ARGUMENT, "unsupported GEMM epilogue");
    }
}

void record_split_rows_tf32(ab_scheme* s, const char* label, const float* x, uint32_t x_stride,
                            const void* norm_w, int32_t w_dtype, float* hi, float* lo,
                            uint32_t rows, uint32_t dim, float eps) {
    if (norm_w) {
        if (Node* n = fusable_fold(s, x, x_stride, rows, dim)) {
            if (w_dtype == AB_F32)
                fuse_fold_norm(s, n, label, (const float*)norm_w, eps, dim, nullptr, hi, lo);
            else
                fuse_fold_norm(s, n, label, (const bf16*)norm_w, eps, dim, nullptr, hi, lo);
            return;
        }
    }
    if (!norm_w) {
        s->add(label, [=](cudaStream_t st) {
            return launch(st, dim3(rows), dim3(256), 0, true,
                          split_rows_tf32_kernel<false, float>, x, x_stride,
                          (const float*)nullptr, hi, lo, dim, eps);
        });
    } else if (w_dtype == AB_F32) {
        const float* wp = (const float*)norm_w;
        s->add(label, [=](cudaStream_t st) {
            return launch(st, dim3(rows), dim3(256), 0, true, split_rows_tf32_kernel<true, float>,
                          x, x_stride, wp, hi, lo, dim, eps);
        });
    } else {
        const bf16* wp = (const bf16*)norm_w;
        s->add(label, [=](cudaStream_t st) {
            return launch(st, dim3(rows), dim3(256), 0, true, split_rows_tf32_kernel<true, bf16>,
                          x, x_stride, wp, hi, lo, dim, eps);
        });
    }
}

void record_rmsnorm_rows_bf16(ab_scheme* s, const char* label, const float* x, const void* w,
                              int32_t w_dtype, void* out, uint32_t rows, uint32_t dim, float eps) {
    bf16* o = (bf16*)out;
    if (Node* n = fusable_fold(s, x, dim, rows, dim)) {
        if (w_dtype == AB_F32)
            fuse_fold_norm(s, n, label, (const float*)w, eps, dim, o, nullptr, nullptr);
        else
            fuse_fold_norm(s, n, label, (const bf16*)w, eps, dim, o, nullptr, nullptr);
        return;
    }
    if (w_dtype == AB_F32) {
        const float* wp = (const float*)w;
        s->add(label, [=](cudaStream_t st) {
            return launch(st, dim3(rows), dim3(256), 0, true, rmsnorm_rows_bf16_kernel<float>, x, wp,
                          o, dim, eps);
        });
    } else {
        const bf16* wp = (const bf16*)w;
        s->add(label, [=](cudaStream_t st) {
            return launch(st, dim3(rows), dim3(256), 0, true, rmsnorm_rows_bf16_kernel<bf16>, x, wp,
                          o, dim, eps);
        });
    }
}

}  // namespace ab
