// Runtime, tensors, DecodeStep parcels and record-then-replay schemes.
//
// The reference's Goldy runtime records dispatch nodes into a Scheme and replays them;
// per-step data arrives through a deposit into a retained parcel, so the scheme is not
// re-recorded every token (src/kernels.rs:17-33, tests/kernels.rs:184-222). Here a
// scheme is a list of validated launch closures; the first submit captures them into a
// CUDA graph on the runtime stream and later submits relaunch the instantiated graph.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <sstream>
#include <vector>

#include <cudaTypedefs.h>

#include "common.cuh"
#include "internal.h"
#include "ops.h"

namespace ab {

static thread_local std::string g_last_error;

void set_last_error(const std::string& msg) { g_last_error = msg; }

std::string shape_str(const ab_tensor& t) {
    std::ostringstream o;
    o << "[";
    for (int i = 0; i < t.rank; i++) o << (i ? ", " : "") << t.dims[i];
    o << "] " << dtype_name(t.dtype);
    return o.str();
}

void expect_rank(const char* param, const ab_tensor& t, int rank) {
    if (t.rank != rank)
        invalid(std::string("parameter `") + param + "`: expected rank " + std::to_string(rank) +
                ", got rank " + std::to_string(t.rank) + " " + shape_str(t));
}

void expect_rank_in(const char* param, const ab_tensor& t, int lo, int hi) {
    if (t.rank < lo || t.rank > hi)
        invalid(std::string("parameter `") + param + "`: expected rank " + std::to_string(lo) +
                (hi != lo ? " to " + std::to_string(hi) : std::string()) + ", got rank " +
                std::to_string(t.rank) + " " + shape_str(t));
}

void expect_dtype(const char* param, const ab_tensor& t, int32_t dt) {
    if (t.dtype != dt)
        invalid(std::string("parameter `") + param + "`: expected dtype " + dtype_name(dt) +
                ", got " + dtype_name(t.dtype));
}

void expect_float(const char* param, const ab_tensor& t) {
    if (t.dtype != AB_F32 && t.dtype != AB_BF16)
        invalid(std::string("parameter `") + param + "`: expected dtype f32 or bf16, got " +
                dtype_name(t.dtype));
}

void expect_dim(const char* param, const ab_tensor& t, int axis, const char* sym, uint64_t want) {
    if (axis >= t.rank || t.dims[axis] != want)
        invalid(std::string("parameter `") + param + "`: dim `" + sym + "` (axis " +
                std::to_string(axis) + ") must be " + std::to_string(want) + ", got " +
                shape_str(t));
}

void expect_data(const char* param, const ab_tensor& t) {
    if (t.rank < 1 || t.rank > 4) invalid(std::string("parameter `") + param + "`: bad rank");
    if (t.data == nullptr)
        invalid(std::string("parameter `") + param + "`: null device pointer");
    for (int i = 0; i < t.rank; i++)
        if (t.dims[i] == 0) invalid(std::string("parameter `") + param + "`: zero-sized dim");
}

uint32_t expect_step(const ab_tensor& step, uint32_t need) {
    expect_data("step", step);
    expect_dtype("step", step, AB_U32);
    if (step.rank != 2 || step.dims[1] != 2)
        invalid("parameter `step`: expected a DecodeStep parcel of dims [n, 2], got " +
                shape_str(step));
    if (step.dims[0] < need)
        invalid("parameter `step`: parcel holds " + std::to_string(step.dims[0]) +
                " steps, batch needs " + std::to_string(need));
    return step.dims[0];
}

void Runtime::activate() const { cuda_check(cudaSetDevice(device), "cudaSetDevice"); }

std::string device_flag_message(uint32_t f) {
    std::string m = "device reported:";
    if (f & kFlagTokenRange) m += " token id out of the embedding table's range;";
    if (f & kFlagPositionRange) m += " decode position beyond the cache's seq_len;";
    if (f & kFlagWaitTimeout) m += " a bounded wait timed out;";
    return m;
}

void Runtime::set_wait_limit_ms(uint64_t ms) {
    const uint64_t ns = ms * 1000000ull;
    cuda_check(cudaMemcpy(reinterpret_cast<unsigned char*>(flags) + 8, &ns, 8,
                          cudaMemcpyHostToDevice),
               "write wait limit");
    wait_limit_ms = ms;
}

void Runtime::check_flags() {
    uint32_t f = 0;
    cuda_check(cudaMemcpy(&f, flags, 4, cudaMemcpyDeviceToHost), "read device flags");
    if (f) {
        cuda_check(cudaMemset(flags, 0, 4), "clear device flags");
        fail(AB_ERR_DEVICE, device_flag_message(f));
    }
}

void encode_tmap_2d(CUtensorMap* map, int32_t dtype, const void* base, uint64_t inner,
                    uint64_t rows, uint64_t row_stride_bytes, uint32_t box_inner,
                    uint32_t box_rows, int swizzle_bytes) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess) fn = nullptr;
        return (PFN_cuTensorMapEncodeTiled_v12000)fn;
    }();
    if (!encode) fail(AB_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    if ((uintptr_t)base % 16 || row_stride_bytes % 16)
        fail(AB_ERR_ARGUMENT, "TMA tensor base and row stride must be 16-byte aligned");
    CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_NONE;
    if (swizzle_bytes == 128) swz = CU_TENSOR_MAP_SWIZZLE_128B;
    else if (swizzle_bytes == 64) swz = CU_TENSOR_MAP_SWIZZLE_64B;
    else if (swizzle_bytes == 32) swz = CU_TENSOR_MAP_SWIZZLE_32B;
    cuuint64_t gdim[2] = {inner, rows};
    cuuint64_t gstride[1] = {row_stride_bytes};
    cuuint32_t box[2] = {box_inner, box_rows};
    cuuint32_t estride[2] = {1, 1};
    CUresult r = encode(map, dtype == AB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                              : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                        2, const_cast<void*>(base), gdim, gstride, box, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        fail(AB_ERR_CUDA, "cuTensorMapEncodeTiled failed with code " + std::to_string((int)r));
}

void Scheme::release_graph() {
    if (exec) cudaGraphExecDestroy(exec);
    if (graph) cudaGraphDestroy(graph);
    exec = nullptr;
    graph = nullptr;
}

// ---- seeded synthetic fill (same generator as the test oracle) --------------------------
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static uint64_t mix64_host(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

template <typename T>
__global__ void fill_normal_kernel(T* out, uint64_t n, uint64_t key, float mean, float std) {
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
         i += (uint64_t)gridDim.x * blockDim.x) {
        uint32_t s = 0;
#pragma unroll
        for (int j = 0; j < 3; j++) {
            uint64_t h = mix64(key + 3ull * i + (uint64_t)j);
            s += (uint32_t)(h & 0xffff) + (uint32_t)((h >> 16) & 0xffff) +
                 (uint32_t)((h >> 32) & 0xffff) + (uint32_t)(h >> 48);
        }
        float z = __fmul_rn((float)((int32_t)(2u * s) - 786420), 1.0f / 131072.0f);
        out[i] = from_f32<T>(__fmaf_rn(std, z, mean));
    }
}

template <typename T>
__global__ void fill_normal_region_kernel(T* out, uint64_t rows, uint64_t cols, uint64_t gcols,
                                          uint64_t row0, uint64_t col0, uint64_t key, float mean,
                                          float std) {
    const uint64_t n = rows * cols;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
         i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t g = (row0 + i / cols) * gcols + col0 + i % cols;
        uint32_t s = 0;
#pragma unroll
        for (int j = 0; j < 3; j++) {
            uint64_t h = mix64(key + 3ull * g + (uint64_t)j);
            s += (uint32_t)(h & 0xffff) + (uint32_t)((h >> 16) & 0xffff) +
                 (uint32_t)((h >> 32) & 0xffff) + (uint32_t)(h >> 48);
        }
        float z = __fmul_rn((float)((int32_t)(2u * s) - 786420), 1.0f / 131072.0f);
        out[i] = from_f32<T>(__fmaf_rn(std, z, mean));
    }
}

void fill_normal_region(Runtime* rt, ab_tensor t, uint64_t seed, uint64_t stream, float mean,
                        float std, uint64_t global_cols, uint64_t row0, uint64_t col0) {
    expect_data("t", t);
    expect_float("t", t);
    const uint64_t cols = t.dims[t.rank - 1];
    const uint64_t rows = numel(t) / cols;
    const uint64_t key = mix64_host(seed * 0xD1B54A32D192ED03ull ^ mix64_host(stream));
    rt->activate();
    const unsigned grid =
        (unsigned)std::min<uint64_t>((rows * cols + 255) / 256, (uint64_t)rt->sm_count * 16);
    if (t.dtype == AB_F32)
        fill_normal_region_kernel<float><<<grid, 256, 0, rt->stream>>>(
            (float*)t.data, rows, cols, global_cols, row0, col0, key, mean, std);
    else
        fill_normal_region_kernel<bf16><<<grid, 256, 0, rt->stream>>>(
            (bf16*)t.data, rows, cols, global_cols, row0, col0, key, mean, std);
    cuda_check(cudaGetLastError(), "fill_normal_region launch");
}

// Host ranges page-locked by ab_host_register: (start, bytes), in registration order.
static std::mutex g_host_ranges_mu;
static std::vector<std::pair<uintptr_t, size_t>> g_host_ranges;

bool host_range_registered(const void* p, size_t bytes) {
    const uintptr_t a = (uintptr_t)p;
    std::lock_guard<std::mutex> lock(g_host_ranges_mu);
    for (const auto& r : g_host_ranges)
        if (a >= r.first && a - r.first <= r.second && bytes <= r.second - (a - r.first))
            return true;
    return false;
}

}  // namespace ab

using namespace ab;

extern "C" {

const char* ab_last_error(void) { return g_last_error.c_str(); }

int ab_runtime_create(int32_t device, ab_runtime** out) {
    return guard([&] {
        if (!out) fail(AB_ERR_ARGUMENT, "null output handle");
        *out = nullptr;
        int count = 0;
        cuda_check(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
        if (device < 0 || device >= count)
            fail(AB_ERR_ARGUMENT, "device " + std::to_string(device) + " not present (" +
                                      std::to_string(count) + " visible)");
        auto* rt = new ab_runtime();
        rt->device = device;
        try {
            rt->activate();
            cuda_check(cudaDeviceGetAttribute(&rt->sm_count, cudaDevAttrMultiProcessorCount, device),
                       "query SM count");
            cuda_check(cudaStreamCreateWithFlags(&rt->stream, cudaStreamNonBlocking),
                       "create stream");
            cuda_check(cudaMalloc(&rt->flags, 256), "allocate flag word");
            cuda_check(cudaMemset(rt->flags, 0, 256), "clear flag word");
            uint64_t limit_ms = 2000;
            if (const char* e = std::getenv("AMMON_B200_WAIT_MS")) {
                const long v = std::atol(e);
                if (v > 0) limit_ms = (uint64_t)v;
            }
            rt->set_wait_limit_ms(limit_ms);
        } catch (...) {
            if (rt->stream) cudaStreamDestroy(rt->stream);
            if (rt->flags) cudaFree(rt->flags);
            delete rt;
            throw;
        }
        *out = rt;
    });
}

int ab_runtime_destroy(ab_runtime* rt) {
    return guard([&] {
        if (!rt) return;
        rt->activate();
        cudaStreamSynchronize(rt->stream);
        cudaStreamDestroy(rt->stream);
        cudaFree(rt->flags);
        delete rt;
    });
}

int ab_runtime_synchronize(ab_runtime* rt) {
    return guard([&] {
        if (!rt) fail(AB_ERR_ARGUMENT, "null runtime");
        rt->activate();
        cuda_check(cudaStreamSynchronize(rt->stream), "stream synchronize");
        rt->check_flags();
    });
}

void* ab_runtime_stream(ab_runtime* rt) { return rt ? (void*)rt->stream : nullptr; }

int ab_host_register(void* ptr, uint64_t bytes) {
    return guard([&] {
        if (!ptr || bytes == 0) fail(AB_ERR_ARGUMENT, "null or empty host range");
        cuda_check(cudaHostRegister(ptr, bytes, cudaHostRegisterDefault), "cudaHostRegister");
        std::lock_guard<std::mutex> lock(g_host_ranges_mu);
        g_host_ranges.emplace_back((uintptr_t)ptr, (size_t)bytes);
    });
}

int ab_host_unregister(void* ptr) {
    return guard([&] {
        if (!ptr) fail(AB_ERR_ARGUMENT, "null host pointer");
        {
            // forget the range first: no later step copies into memory about to be unlocked
            std::lock_guard<std::mutex> lock(g_host_ranges_mu);
            for (size_t i = 0; i < g_host_ranges.size(); i++)
                if (g_host_ranges[i].first == (uintptr_t)ptr) {
                    g_host_ranges.erase(g_host_ranges.begin() + (long)i);
                    break;
                }
        }
        cuda_check(cudaHostUnregister(ptr), "cudaHostUnregister");
    });
}

int ab_runtime_set_wait_limit(ab_runtime* rt, uint32_t ms) {
    return guard([&] {
        if (!rt) fail(AB_ERR_ARGUMENT, "null runtime");
        if (ms == 0) fail(AB_ERR_ARGUMENT, "wait limit must be at least 1 ms");
        rt->activate();
        cuda_check(cudaStreamSynchronize(rt->stream), "stream synchronize");
        rt->set_wait_limit_ms(ms);
    });
}

int ab_runtime_wait_limit(ab_runtime* rt, uint32_t* ms) {
    return guard([&] {
        if (!rt || !ms) fail(AB_ERR_ARGUMENT, "null argument");
        *ms = (uint32_t)rt->wait_limit_ms;
    });
}

int ab_runtime_sm_count(ab_runtime* rt, int32_t* out) {
    return guard([&] {
        if (!rt || !out) fail(AB_ERR_ARGUMENT, "null argument");
        *out = rt->sm_count;
    });
}

int ab_tensor_zeros(ab_runtime* rt, int32_t dtype, int32_t rank, const uint32_t* dims,
                    ab_tensor* out) {
    return guard([&] {
        if (!rt || !out || (!dims && rank > 0)) fail(AB_ERR_ARGUMENT, "null argument");
        if (rank < 1 || rank > 4) fail(AB_ERR_ARGUMENT, "rank must be 1..4");
        ab_tensor t = {};
        t.dtype = dtype;
        t.rank = rank;
        for (int i = 0; i < rank; i++) t.dims[i] = dims[i];
        uint64_t bytes = nbytes(t);
        if (bytes == 0) fail(AB_ERR_ARGUMENT, "zero-sized tensor");
        rt->activate();
        cuda_check(cudaMalloc(&t.data, bytes), "cudaMalloc");
        cudaError_t e = cudaMemset(t.data, 0, bytes);
        if (e != cudaSuccess) {
            cudaFree(t.data);
            cuda_check(e, "cudaMemset");
        }
        *out = t;
    });
}

int ab_tensor_free(ab_runtime* rt, ab_tensor* t) {
    return guard([&] {
        if (!rt || !t) fail(AB_ERR_ARGUMENT, "null argument");
        if (t->data) {
            rt->activate();
            cuda_check(cudaStreamSynchronize(rt->stream), "stream synchronize");
            cuda_check(cudaFree(t->data), "cudaFree");
        }
        t->data = nullptr;
    });
}

int ab_tensor_write(ab_runtime* rt, ab_tensor t, const void* host, uint64_t bytes) {
    return guard([&] {
        if (!rt || !host) fail(AB_ERR_ARGUMENT, "null argument");
        expect_data("t", t);
        if (bytes != nbytes(t))
            fail(AB_ERR_ARGUMENT, "write of " + std::to_string(bytes) + " bytes into a tensor of " +
                                      std::to_string(nbytes(t)));
        rt->activate();
        cuda_check(cudaMemcpyAsync(t.data, host, bytes, cudaMemcpyHostToDevice, rt->stream),
                   "host to device copy");
        cuda_check(cudaStreamSynchronize(rt->stream), "stream synchronize");
    });
}

int ab_tensor_read(ab_runtime* rt, ab_tensor t, void* host, uint64_t bytes) {
    return guard([&] {
        if (!rt || !host) fail(AB_ERR_ARGUMENT, "null argument");
        expect_data("t", t);
        if (bytes > nbytes(t))
            fail(AB_ERR_ARGUMENT, "read of " + std::to_string(bytes) + " bytes from a tensor of " +
                                      std::to_string(nbytes(t)));
        rt->activate();
        cuda_check(cudaMemcpyAsync(host, t.data, bytes, cudaMemcpyDeviceToHost, rt->stream),
                   "device to host copy");
        cuda_check(cudaStreamSynchronize(rt->stream), "stream synchronize");
        rt->check_flags();
    });
}

int ab_tensor_fill_normal(ab_runtime* rt, ab_tensor t, uint64_t seed, uint64_t stream, float mean,
                          float std) {
    return guard([&] {
        if (!rt) fail(AB_ERR_ARGUMENT, "null runtime");
        expect_data("t", t);
        expect_float("t", t);
        uint64_t key = mix64_host(seed * 0xD1B54A32D192ED03ull ^ mix64_host(stream));
        uint64_t n = numel(t);
        rt->activate();
        unsigned grid = (unsigned)std::min<uint64_t>((n + 255) / 256, (uint64_t)rt->sm_count * 16);
        if (t.dtype == AB_F32)
            fill_normal_kernel<float><<<grid, 256, 0, rt->stream>>>((float*)t.data, n, key, mean, std);
        else
            fill_normal_kernel<bf16><<<grid, 256, 0, rt->stream>>>((bf16*)t.data, n, key, mean, std);
        cuda_check(cudaGetLastError(), "fill_normal launch");
    });
}

int ab_tensor_narrow(ab_tensor t, uint32_t start, uint32_t len, ab_tensor* out) {
    return guard([&] {
        if (!out) fail(AB_ERR_ARGUMENT, "null output");
        if (t.rank < 1) fail(AB_ERR_VALIDATION, "narrow of a rank-0 tensor");
        if ((uint64_t)start + len > t.dims[0] || len == 0)
            invalid("narrow(0, " + std::to_string(start) + ", " + std::to_string(len) +
                    ") out of range for " + shape_str(t));
        uint64_t inner = numel(t) / t.dims[0];
        ab_tensor r = t;
        r.dims[0] = len;
        r.data = (char*)t.data + (uint64_t)start * inner * dtype_size(t.dtype);
        *out = r;
    });
}

int ab_tensor_reshape(ab_tensor t, int32_t rank, const uint32_t* dims, ab_tensor* out) {
    return guard([&] {
        if (!out || !dims) fail(AB_ERR_ARGUMENT, "null argument");
        if (rank < 1 || rank > 4) fail(AB_ERR_ARGUMENT, "rank must be 1..4");
        ab_tensor r = t;
        r.rank = rank;
        for (int i = 0; i < 4; i++) r.dims[i] = i < rank ? dims[i] : 0;
        if (numel(r) != numel(t))
            invalid("reshape of " + shape_str(t) + " to " + shape_str(r) + " changes numel");
        *out = r;
    });
}

int ab_step_parcel(ab_runtime* rt, uint32_t n, ab_tensor* out) {
    uint32_t dims[2] = {n, 2};
    if (n == 0) {
        set_last_error("a DecodeStep parcel needs at least one step");
        return AB_ERR_ARGUMENT;
    }
    return ab_tensor_zeros(rt, AB_U32, 2, dims, out);
}

int ab_step_deposit(ab_runtime* rt, ab_tensor parcel, const ab_decode_step* steps, uint32_t n) {
    return guard([&] {
        if (!rt || !steps) fail(AB_ERR_ARGUMENT, "null argument");
        expect_step(parcel, n);
        rt->activate();
        // Pageable source: the runtime stages it before returning, so the caller may reuse
        // `steps` immediately; the copy is ordered before later work on the stream.
        cuda_check(cudaMemcpyAsync(parcel.data, steps, sizeof(ab_decode_step) * n,
                                   cudaMemcpyHostToDevice, rt->stream),
                   "deposit DecodeStep");
    });
}

int ab_scheme_create(ab_runtime* rt, ab_scheme** out) {
    return guard([&] {
        if (!out) fail(AB_ERR_ARGUMENT, "null output handle");
        auto* s = new ab_scheme();
        s->rt = rt;  // may be null: validation-only schemes cannot be submitted
        *out = s;
    });
}

int ab_scheme_destroy(ab_scheme* s) {
    return guard([&] {
        if (!s) return;
        if (s->rt) {
            s->rt->activate();
            cudaStreamSynchronize(s->rt->stream);
        }
        s->release_graph();
        for (void* b : s->owned) cudaFree(b);
        delete s;
    });
}

int ab_scheme_submit(ab_scheme* s) {
    return guard([&] {
        if (!s) fail(AB_ERR_ARGUMENT, "null scheme");
        if (!s->rt) fail(AB_ERR_ARGUMENT, "scheme has no runtime");
        Runtime& rt = *s->rt;
        rt.activate();
        s->replays++;
        if (!s->use_graph) {
            for (auto& n : s->nodes) cuda_check(n.launch(rt.stream), n.label.c_str());
            return;
        }
        if (s->dirty || !s->exec) {
            s->release_graph();
            cuda_check(cudaStreamBeginCapture(rt.stream, cudaStreamCaptureModeThreadLocal),
                       "begin capture");
            cudaError_t err = cudaSuccess;
            std::string where;
            for (auto& n : s->nodes) {
                err = n.launch(rt.stream);
                if (err != cudaSuccess) {
                    where = n.label;
                    break;
                }
            }
            cudaGraph_t g = nullptr;
            cudaError_t end = cudaStreamEndCapture(rt.stream, &g);
            if (err != cudaSuccess) {
                if (g) cudaGraphDestroy(g);
                cudaGetLastError();
                fail(AB_ERR_CUDA, "record of `" + where + "`: " + cudaGetErrorString(err));
            }
            cuda_check(end, "end capture");
            s->graph = g;
            cuda_check(cudaGraphInstantiate(&s->exec, g, 0), "instantiate graph");
            s->records++;
            s->dirty = false;
        }
        cuda_check(cudaGraphLaunch(s->exec, rt.stream), "graph launch");
    });
}

int ab_scheme_node_count(const ab_scheme* s, uint32_t* out) {
    return guard([&] {
        if (!s || !out) fail(AB_ERR_ARGUMENT, "null argument");
        *out = (uint32_t)s->nodes.size();
    });
}

int ab_scheme_replay_stats(const ab_scheme* s, uint32_t* records, uint32_t* replays) {
    return guard([&] {
        if (!s) fail(AB_ERR_ARGUMENT, "null scheme");
        if (records) *records = s->records;
        if (replays) *replays = s->replays;
    });
}

int ab_scheme_use_graph(ab_scheme* s, int32_t enable) {
    return guard([&] {
        if (!s) fail(AB_ERR_ARGUMENT, "null scheme");
        s->use_graph = enable != 0;
        s->dirty = true;
    });
}

int ab_scheme_time_nodes(ab_scheme* s, uint32_t iters, float* ms, uint32_t n) {
    return guard([&] {
        if (!s || !ms) fail(AB_ERR_ARGUMENT, "null argument");
        if (!s->rt) fail(AB_ERR_ARGUMENT, "scheme has no runtime");
        if (n < s->nodes.size()) fail(AB_ERR_ARGUMENT, "output holds fewer entries than nodes");
        if (iters == 0) iters = 1;
        Runtime& rt = *s->rt;
        rt.activate();
        cudaEvent_t a, b;
        cuda_check(cudaEventCreate(&a), "event create");
        cuda_check(cudaEventCreate(&b), "event create");
        std::string err;
        for (size_t i = 0; i < s->nodes.size() && err.empty(); i++) {
            cudaError_t e = s->nodes[i].launch(rt.stream);  // warm
            if (e == cudaSuccess) e = cudaEventRecord(a, rt.stream);
            for (uint32_t k = 0; k < iters && e == cudaSuccess; k++) e = s->nodes[i].launch(rt.stream);
            if (e == cudaSuccess) e = cudaEventRecord(b, rt.stream);
            if (e == cudaSuccess) e = cudaEventSynchronize(b);
            float t = 0.0f;
            if (e == cudaSuccess) e = cudaEventElapsedTime(&t, a, b);
            if (e != cudaSuccess) err = s->nodes[i].label + ": " + cudaGetErrorString(e);
            ms[i] = t / (float)iters;
        }
        cudaEventDestroy(a);
        cudaEventDestroy(b);
        if (!err.empty()) fail(AB_ERR_CUDA, "time_nodes: " + err);
        rt.check_flags();
    });
}

int ab_scheme_node_label(const ab_scheme* s, uint32_t i, char* buf, uint32_t cap) {
    return guard([&] {
        if (!s || !buf || cap == 0) fail(AB_ERR_ARGUMENT, "null argument");
        if (i >= s->nodes.size()) fail(AB_ERR_ARGUMENT, "node index out of range");
        const std::string& l = s->nodes[i].label;
        const size_t n = std::min<size_t>(l.size(), cap - 1);
        std::memcpy(buf, l.data(), n);
        buf[n] = 0;
    });
}

}  // extern "C"
