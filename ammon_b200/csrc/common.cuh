// Device-side helpers shared by the sm_100a kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ab {

struct Step {
    uint32_t token;
    uint32_t position;
};

typedef __nv_bfloat16 bf16;

// ---- element conversion ----------------------------------------------------------------
__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(bf16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) {
    return v;
}
template <>
__device__ __forceinline__ bf16 from_f32<bf16>(float v) {
    return __float2bfloat16_rn(v);
}

// bf16 pair packed in a 32-bit word -> two floats (exact; low half is the lower index).
__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// ---- programmatic dependent launch ----------------------------------------------------
// wait: block until the preceding grid in the stream has completed and its memory is
// visible. launch_dependents: allow the next grid to start launching. Both are no-ops
// when the kernel was launched without the PDL attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- memory ---------------------------------------------------------------------------
// 16-byte streaming load through the non-coherent path without L1 allocation: weights
// are read once per step.
__device__ __forceinline__ uint4 ld_stream(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// Bulk prefetch of [p, p + bytes) into L2 (bytes a multiple of 16, p 16-byte aligned).
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// silu(g) * u in the order of the reference's swiglu kernel (src/kernels.rs:462-476):
// g * (1 / (1 + e^-g)), then times u, with the accurate exponential and an IEEE division.
// Every SwiGLU epilogue (GEMV, single-split GEMM, split-K fold, standalone kernel) calls
// this one expression, so a layer's result does not depend on which of them ran it.
__device__ __forceinline__ float silu_mul(float g, float u) {
    const float s = g * (1.0f / (1.0f + expf(-g)));
    return s * u;
}

// RoPE angle of pair i (even) of a head of size head at position pos
// (src/kernels.rs:195-199): freq = 1 / theta^((i % head) / head).
__device__ __forceinline__ void rope_cos_sin(uint32_t i, uint32_t head, uint32_t pos, float theta,
                                             float* c, float* s) {
    int32_t hd = (int32_t)(i % head);
    float freq = 1.0f / powf(theta, (float)hd / (float)head);
    float val = (float)pos * freq;
    sincosf(val, s, c);
}

}  // namespace ab
