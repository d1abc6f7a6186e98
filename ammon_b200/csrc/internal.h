// Internal host-side structures shared by the translation units of libammon_b200.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdlib>
#include <functional>
#include <stdexcept>
#include <string>
#include <vector>

#include "ammon_b200.h"

namespace ab {

// ---- errors -----------------------------------------------------------------------
// Every C entry point catches ab::Error and turns it into a status + thread-local text.
struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

[[noreturn]] inline void fail(int code, const std::string& msg) { throw Error(code, msg); }
[[noreturn]] inline void invalid(const std::string& msg) { fail(AB_ERR_VALIDATION, msg); }

void set_last_error(const std::string& msg);

inline void cuda_check(cudaError_t e, const char* what) {
    if (e != cudaSuccess)
        fail(AB_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// Runs fn, mapping exceptions to a status code.
template <class F>
int guard(F&& fn) {
    try {
        fn();
        return AB_OK;
    } catch (const Error& e) {
        set_last_error(e.what());
        return e.code;
    } catch (const std::bad_alloc&) {
        set_last_error("host allocation failed");
        return AB_ERR_ARGUMENT;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return AB_ERR_ARGUMENT;
    }
}

// ---- tensors -------------------------------------------------------------------------
inline size_t dtype_size(int32_t dt) {
    switch (dt) {
        case AB_F32: return 4;
        case AB_BF16: return 2;
        case AB_U32: return 4;
        default: fail(AB_ERR_ARGUMENT, "unknown dtype " + std::to_string(dt));
    }
}

inline const char* dtype_name(int32_t dt) {
    switch (dt) {
        case AB_F32: return "f32";
        case AB_BF16: return "bf16";
        case AB_U32: return "u32";
        default: return "?";
    }
}

inline uint64_t numel(const ab_tensor& t) {
    uint64_t n = 1;
    for (int i = 0; i < t.rank; i++) n *= t.dims[i];
    return n;
}

inline uint64_t nbytes(const ab_tensor& t) { return numel(t) * dtype_size(t.dtype); }

std::string shape_str(const ab_tensor& t);

// Contract checks with the reference's message vocabulary ("parameter `x`",
// "expected rank N", symbolic dim names in backticks).
void expect_rank(const char* param, const ab_tensor& t, int rank);
void expect_rank_in(const char* param, const ab_tensor& t, int lo, int hi);
void expect_dtype(const char* param, const ab_tensor& t, int32_t dt);
void expect_float(const char* param, const ab_tensor& t);
void expect_dim(const char* param, const ab_tensor& t, int axis, const char* sym, uint64_t want);
void expect_data(const char* param, const ab_tensor& t);
// Step parcel [n, 2] u32 with n >= need.
uint32_t expect_step(const ab_tensor& step, uint32_t need);

// ---- runtime -----------------------------------------------------------------------
struct Runtime {
    int device = 0;
    int sm_count = 0;
    cudaStream_t stream = nullptr;
    // device flag block (256 bytes): [0] u32 bit flags raised by kernels, [8] u64 limit of
    // every bounded wait in nanoseconds (read by the kernels once a wait has lasted 1 ms)
    uint32_t* flags = nullptr;
    uint64_t wait_limit_ms = 2000;
    void activate() const;      // cudaSetDevice(device)
    void check_flags();         // reads + clears the flag word, throws AB_ERR_DEVICE
    void set_wait_limit_ms(uint64_t ms);  // writes the limit into the flag block
};

enum DeviceFlag : uint32_t {
    kFlagTokenRange = 1u,
    kFlagPositionRange = 2u,
    kFlagWaitTimeout = 4u,
};

// "device reported: ..." text for a non-zero flag word.
std::string device_flag_message(uint32_t flags);

// Whether [p, p + bytes) lies inside one host range page-locked through ab_host_register (and
// not yet unregistered): only such a range takes a device copy without the staging buffer.
bool host_range_registered(const void* p, size_t bytes);

// ---- schemes -------------------------------------------------------------------------
using LaunchFn = std::function<cudaError_t(cudaStream_t)>;

// A recorded residual k-split fold: x[col * x_stride + r] += the sum over splits of
// ws[split][tile][col][128] (rows r < n_rows, columns col < nb). Kept with its node so that an
// RMSNorm of the same rows recorded right after it runs inside the fold (gemm_tc.cu).
struct FoldInfo {
    const float* ws = nullptr;
    float* x = nullptr;  // null: the node is not such a fold
    uint32_t tiles = 0, bn = 0, ksplit = 0, nb = 0, n_rows = 0, x_stride = 0;
};

struct Node {
    std::string label;
    LaunchFn launch;
    FoldInfo fold;
};

struct Scheme {
    Runtime* rt = nullptr;
    std::vector<Node> nodes;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    bool dirty = true;
    bool use_graph = true;
    uint32_t records = 0;
    uint32_t replays = 0;
    // device buffers that recorded nodes use and the scheme frees when it is destroyed
    // (kernel entry points that need scratch of their own, e.g. ab_kernel_attention_decode)
    std::vector<void*> owned;
    void add(const char* label, LaunchFn fn) {
        nodes.push_back(Node{label, std::move(fn), FoldInfo{}});
        dirty = true;
    }
    void add_fold(const char* label, LaunchFn fn, const FoldInfo& fold) {
        nodes.push_back(Node{label, std::move(fn), fold});
        dirty = true;
    }
    void release_graph();
};

// Programmatic dependent launch is on by default (AMMON_B200_PDL=0 turns it off). Measured
// on the 8B-shaped decode graph it gave 1.4% at batch 1 and 2% at batch 64, the same in
// repeated runs. The kernels compute the same results either way (griddepcontrol is a
// no-op without the launch attribute).
inline bool pdl_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("AMMON_B200_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}

// Launch with optional programmatic dependent launch (PDL): the kernel may begin while
// its predecessor drains; kernels call griddepcontrol.wait before reading predecessor
// outputs.
template <typename... KArgs, typename... Args>
cudaError_t launch(cudaStream_t s, dim3 grid, dim3 block, size_t smem, bool pdl,
                   void (*kernel)(KArgs...), Args... args) {
    pdl = pdl && pdl_enabled();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = pdl ? attr : nullptr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

}  // namespace ab

struct ab_runtime : ab::Runtime {};
struct ab_scheme : ab::Scheme {};
