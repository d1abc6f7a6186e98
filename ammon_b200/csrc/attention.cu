// Fused flash-decoding attention for the block path, replacing the reference's
// attention_partial + attention_combine pair (src/kernels.rs:228-410).
//
// Design (B200):
//  - Grid (splits, kv_heads, batch). One CTA serves every query head of its GQA group
//    from one staged K/V tile, so K/V bytes are read once per kv head rather than once
//    per query head.
//  - The position range [0, pos] is cut into `nsplit` chunks (multiples of the 64-row
//    tile) computed on the device from the step's position, so a graph recorded once
//    serves every position. Splits beyond pos write an empty partial.
//  - Scores, the online softmax (running max m, sum l) and the P.V accumulation happen
//    in one pass over each tile.
//  - The last CTA of a (batch, kv head) to finish (atomic ticket) folds the partials in
//    split order and writes the output, so no second kernel runs; it resets the ticket
//    for the next replay.
#include <algorithm>
#include <mutex>
#include <string>

#include "common.cuh"
#include "internal.h"
#include "ops.h"

namespace ab {

constexpr int kAttnThreads = 128;
constexpr int kAttnTile = 64;

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

struct AttnLayout {
    uint32_t row_words, kstride_words;
    size_t q_off, k_off, v_off, s_off, p_off, st_off, fold_off, w_off, total;
};

// Shared-memory layout; K rows are padded to a stride of 4 (mod 8) words so that lanes
// reading different rows at the same column hit distinct banks.
__host__ __device__ inline AttnLayout attn_layout(uint32_t head, uint32_t esz, uint32_t G,
                                                  uint32_t nsplit) {
    AttnLayout L;
    L.row_words = head * esz / 4;
    L.kstride_words = L.row_words + ((12 - L.row_words % 8) % 8);
    size_t o = 0;
    L.q_off = o;
    o += (size_t)G * head * 4;
    o = (o + 15) & ~(size_t)15;
    L.k_off = o;
    o += (size_t)kAttnTile * L.kstride_words * 4;
    L.v_off = o;
    o += (size_t)kAttnTile * L.row_words * 4;
    L.s_off = o;
    o += (size_t)G * kAttnTile * 4;
    L.p_off = o;
    o += (size_t)kAttnTile * (G < 4 ? 4 : G) * 4;
    L.st_off = o;
    o += 3 * 8 * 4 + 16;
    L.fold_off = o;
    o += (size_t)kAttnThreads * G * 4;
    L.w_off = o;
    o += (size_t)nsplit * G * 4;
    L.total = (o + 15) & ~(size_t)15;
    return L;
}

template <typename KT, typename OT, int G>
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const AttnParams p) {
    extern __shared__ __align__(16) unsigned char smem[];
    constexpr int VE = 16 / sizeof(KT);  // elements per 16-byte vector
    const uint32_t hd = p.head;
    const AttnLayout L = attn_layout(hd, sizeof(KT), G, p.nsplit);
    float* qs = (float*)(smem + L.q_off);       // [G][hd], pre-scaled by 1/sqrt(hd)
    uint32_t* ks = (uint32_t*)(smem + L.k_off);  // [TP][kstride_words]
    uint32_t* vs = (uint32_t*)(smem + L.v_off);  // [TP][row_words]
    float* sc = (float*)(smem + L.s_off);        // [G][TP] scores
    float* pt = (float*)(smem + L.p_off);        // [TP][max(G,4)] probabilities
    float* st = (float*)(smem + L.st_off);       // m[8], l[8], alpha[8], flag
    float* fold = (float*)(smem + L.fold_off);   // [ways][G][hd]
    float* wts = (float*)(smem + L.w_off);       // [nsplit][G] combine weights
    float* sm_m = st;
    float* sm_l = st + 8;
    float* sm_a = st + 16;
    int* sm_last = (int*)(st + 24);
    constexpr int PS = G < 4 ? 4 : G;

    const uint32_t split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const uint32_t tid = threadIdx.x, lane = tid % 32, warp = tid / 32;
    const uint32_t kvd = p.kv_heads * hd;
    const uint32_t nvec = hd / VE;  // 16-byte vectors per K/V row

    pdl_wait();
    pdl_trigger();

    const uint32_t pos = p.step[b].position;
    const bool bad = pos >= p.seq;
    if (bad && split == 0 && kvh == 0 && tid == 0) atomicOr(p.flags, kFlagPositionRange);
    const uint32_t total = bad ? 0u : pos + 1;
    uint32_t chunk = (total + p.nsplit - 1) / p.nsplit;
    chunk = (chunk + kAttnTile - 1) / kAttnTile * kAttnTile;
    const uint32_t start = min(split * chunk, total);
    const uint32_t end = min(start + chunk, total);

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
        // stage K and V rows of the tile (zero rows past the end)
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
        // scores: thread -> (position p, head group hg)
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
        // online softmax per head: warp w takes heads w, w + 4
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
        __syncthreads();
        // P.V: thread -> (dim di, way); ways split the tile's positions
        if (way < ways) {
#pragma unroll
            for (int h = 0; h < G; h++) acc[h] *= sm_a[h];
            for (uint32_t r = way; r < kAttnTile; r += ways) {
                const KT* vr = reinterpret_cast<const KT*>(vs + (size_t)r * L.row_words);
                const float v = to_f32(vr[di]);
                const float* pr = pt + r * PS;
#pragma unroll
                for (int h = 0; h < G; h++) acc[h] = fmaf(pr[h], v, acc[h]);
            }
        }
        __syncthreads();
    }

    // fold the ways in order
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
    if (p.nsplit == 1) {
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

    // write this split's partial, then the last CTA of the group combines
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
        *sm_last = prev == p.nsplit - 1;
    }
    __syncthreads();
    if (!*sm_last) return;
    __threadfence();
    const float* go = p.part_o + grp * p.nsplit * G * hd;
    const float* gml = p.part_ml + grp * p.nsplit * G * 2;
    if (tid < (uint32_t)G) {
        float M = -INFINITY;
        for (uint32_t s = 0; s < p.nsplit; s++) M = fmaxf(M, __ldcg(gml + (s * G + tid) * 2));
        float Lsum = 0.0f;
        for (uint32_t s = 0; s < p.nsplit; s++) {
            const float m = __ldcg(gml + (s * G + tid) * 2);
            const float w = (m == -INFINITY) ? 0.0f : expf(m - M);
            wts[s * G + tid] = w;
            Lsum += w * __ldcg(gml + (s * G + tid) * 2 + 1);
        }
        sm_l[tid] = Lsum;
    }
    __syncthreads();
    for (uint32_t o = tid; o < G * hd; o += kAttnThreads) {
        const uint32_t h = o / hd;
        float v = 0.0f;
        for (uint32_t s = 0; s < p.nsplit; s++) {
            const float w = wts[s * G + h];
            if (w != 0.0f) v += w * __ldcg(go + (size_t)s * G * hd + o);
        }
        const float Lsum = sm_l[h];
        ((OT*)p.out)[orow + o] = from_f32<OT>(Lsum > 0.0f ? v / Lsum : 0.0f);
    }
    if (tid == 0) p.counters[grp] = 0;
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
    const uint64_t target = (uint64_t)std::max(sm_count, 1) * 8;
    const uint64_t groups = std::max<uint64_t>(1, (uint64_t)batch * kv_heads);
    uint64_t ns = (target + groups - 1) / groups;
    ns = std::min<uint64_t>(ns, (seq + kAttnTile - 1) / kAttnTile);
    ns = std::min<uint64_t>(ns, max_splits);
    return (uint32_t)std::max<uint64_t>(ns, 1);
}

void attention_scratch_size(uint32_t batch, uint32_t heads, uint32_t head, uint32_t nsplit,
                            uint64_t* floats, uint64_t* counters) {
    *floats = (uint64_t)batch * heads * nsplit * (head + 2);
    *counters = (uint64_t)batch * heads;
}

template <typename KT, typename OT, int G>
static void add_attn(ab_scheme* s, const char* label, const AttnParams& p) {
    const AttnLayout L = attn_layout(p.head, sizeof(KT), G, p.nsplit);
    const size_t smem = L.total;
    if (smem > 200 * 1024) invalid("attention: shared-memory stage too large");
    auto kern = attn_decode_kernel<KT, OT, G>;
    dim3 grid(p.nsplit, p.kv_heads, p.batch);
    s->add(label, [=](cudaStream_t st) {
        if (smem > 48 * 1024) {
            cudaError_t e =
                cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
        }
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

extern "C" int ab_attention_decode_noalloc(void* stream, ab_tensor q, ab_tensor key_cache,
                                           ab_tensor value_cache, ab_tensor out, ab_tensor step) {
    return guard([&] {
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
        const int cr = q.rank == 3 ? 4 : 3;
        expect_rank("key_cache", key_cache, cr);
        expect_rank("value_cache", value_cache, cr);
        for (int a = 0; a < cr; a++)
            if (value_cache.dims[a] != key_cache.dims[a])
                invalid("parameter `value_cache`: dims must match key_cache " + shape_str(key_cache));
        const int o = cr - 3;
        if (cr == 4 && key_cache.dims[0] < batch)
            expect_dim("key_cache", key_cache, 0, "batch", batch);
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

        int device = 0;
        unsigned char* base = noalloc_scratch(&device);
        int sms = 148;
        cuda_check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device),
                   "query SM count");
        const uint32_t nsplit = attention_choose_splits(batch, kv_heads, seq, sms, 256);
        uint64_t floats = 0, tickets = 0;
        attention_scratch_size(batch, heads, head, nsplit, &floats, &tickets);
        tickets = (uint64_t)batch * kv_heads;
        if (floats > kNoAllocFloats || tickets > kNoAllocTickets)
            fail(AB_ERR_ARGUMENT,
                 "ab_attention_decode_noalloc: this shape needs " + std::to_string(floats * 4) +
                     " bytes of split partials and " + std::to_string(tickets) +
                     " tickets; the static scratch holds " + std::to_string(kNoAllocFloats * 4) +
                     " bytes and " + std::to_string(kNoAllocTickets) + " tickets");

        AttnParams p = {};
        p.q = (const float*)q.data;
        p.kcache = key_cache.data;
        p.vcache = value_cache.data;
        p.kv_dtype = key_cache.dtype;
        p.cache_stride = (uint64_t)seq * kv_heads * head;
        p.out = out.data;
        p.out_dtype = out.dtype;
        p.heads = heads;
        p.kv_heads = kv_heads;
        p.head = head;
        p.seq = seq;
        p.batch = batch;
        p.nsplit = nsplit;
        p.part_o = (float*)base;
        p.part_ml = (float*)base + (uint64_t)batch * heads * nsplit * head;
        p.counters = (uint32_t*)(base + kNoAllocFloats * 4);
        p.flags = (uint32_t*)(base + kNoAllocFloats * 4 + (uint64_t)kNoAllocTickets * 4);
        p.step = (const Step*)step.data;

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
