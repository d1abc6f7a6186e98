// NCCL communicator for tensor parallelism over NVLink / NVSwitch.
//
// NCCL is resolved at run time with dlopen: when the process already loaded libnccl.so.2
// (torch.distributed does), that instance is used, so one process never holds two NCCL
// libraries. Collectives are recorded into schemes like kernels and are captured into the
// step's CUDA graph.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "common.cuh"
#include "tma.cuh"

#include "internal.h"
#include "ops.h"

namespace ab {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t,
                               ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
    ncclResult_t (*comm_init_rank_config)(ncclComm_t*, int, ncclUniqueId, int,
                                          ncclConfig_t*) = nullptr;
    ncclResult_t (*get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*comm_finalize)(ncclComm_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
    bool ok = false;
};

static NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) {
            const char* path = std::getenv("AMMON_B200_NCCL");
            h = dlopen(path ? path : "libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        }
        if (!h) return;
        auto sym = [&](const char* n) { return dlsym(h, n); };
        api.get_unique_id = (decltype(api.get_unique_id))sym("ncclGetUniqueId");
        api.comm_init_rank = (decltype(api.comm_init_rank))sym("ncclCommInitRank");
        api.all_reduce = (decltype(api.all_reduce))sym("ncclAllReduce");
        api.all_gather = (decltype(api.all_gather))sym("ncclAllGather");
        api.comm_destroy = (decltype(api.comm_destroy))sym("ncclCommDestroy");
        api.comm_abort = (decltype(api.comm_abort))sym("ncclCommAbort");
        api.comm_init_rank_config =
            (decltype(api.comm_init_rank_config))sym("ncclCommInitRankConfig");
        api.get_async_error = (decltype(api.get_async_error))sym("ncclCommGetAsyncError");
        api.broadcast = (decltype(api.broadcast))sym("ncclBroadcast");
        api.comm_finalize = (decltype(api.comm_finalize))sym("ncclCommFinalize");
        api.error_string = (decltype(api.error_string))sym("ncclGetErrorString");
        api.ok = api.get_unique_id && api.comm_init_rank && api.all_reduce && api.all_gather &&
                 api.comm_destroy && api.comm_abort && api.comm_init_rank_config &&
                 api.get_async_error && api.broadcast && api.comm_finalize && api.error_string;
    });
    if (!api.ok) fail(AB_ERR_NCCL, "libnccl.so.2 could not be loaded (set AMMON_B200_NCCL)");
    return api;
}

static void nccl_check(ncclResult_t r, const char* what) {
    if (r != ncclSuccess)
        fail(AB_ERR_NCCL, std::string(what) + ": " + nccl().error_string(r));
}

// Last NCCL failure inside a recorded launch (launch closures return CUDA codes).
static thread_local std::string g_nccl_error;

}  // namespace ab

struct ab_comm {
    ab::Runtime* rt = nullptr;
    ncclComm_t comm = nullptr;
    int32_t rank = 0, world = 1;
    // NVLink peer exchange (comm_peers_setup): one device block per rank holding
    // [flags: 2 parities x kTpMaxWorld u64][pad][send: 2 parities x max_elems f32],
    // opened by every peer through CUDA IPC.
    bool peers = false;
    size_t max_elems = 0;
    unsigned char* local = nullptr;
    unsigned char* peer_base[ab::kTpMaxWorld] = {};
    uint64_t* epoch = nullptr;   // device: bumped once per recorded step
    uint32_t next_site = 0;      // all-reduce sites numbered in recording order
    // the persistent decode step's exchange block (comm_fused_block), one per rank, opened
    // by every peer through CUDA IPC; released with the communicator
    size_t fused_bytes = 0;
    unsigned char* fused_local = nullptr;
    unsigned char* fused_peer[ab::kTpMaxWorld] = {};
};

namespace ab {

int comm_rank(const ab_comm* c) { return c ? c->rank : 0; }
int comm_world(const ab_comm* c) { return c ? c->world : 1; }

static constexpr size_t kTpFlagBytes = 2 * kTpMaxWorld * sizeof(uint64_t);
static constexpr size_t kTpRecvOff = 256;

static uint64_t* tp_flags(unsigned char* base, uint32_t parity) {
    return (uint64_t*)base + (size_t)parity * kTpMaxWorld;
}
static float* tp_send(const ab_comm* c, unsigned char* base, uint32_t parity) {
    return (float*)(base + kTpRecvOff) + (size_t)parity * c->max_elems;
}

// Blocking NCCL all-gather of host bytes through device staging (setup time only).
static void allgather_host(ab_comm* c, const void* mine, void* all, size_t bytes) {
    unsigned char* d = nullptr;
    cuda_check(cudaMalloc(&d, bytes * (c->world + 1)), "cudaMalloc");
    cudaError_t e = cudaMemcpy(d, mine, bytes, cudaMemcpyHostToDevice);
    ncclResult_t r = ncclSuccess;
    if (e == cudaSuccess) r = nccl().all_gather(d, d + bytes, bytes, ncclUint8, c->comm, c->rt->stream);
    if (e == cudaSuccess && r == ncclSuccess) e = cudaStreamSynchronize(c->rt->stream);
    if (e == cudaSuccess && r == ncclSuccess)
        e = cudaMemcpy(all, d + bytes, bytes * c->world, cudaMemcpyDeviceToHost);
    cudaFree(d);
    nccl_check(r, "ncclAllGather");
    cuda_check(e, "peer exchange");
}

bool comm_peers_setup(ab_comm* c, size_t max_elems) {
    if (c->peers) {
        if (max_elems > c->max_elems)
            fail(AB_ERR_ARGUMENT, "peer buffers were set up for a narrower model on this "
                                  "communicator");
        return true;
    }
    if (c->world < 2 || c->world > (int)kTpMaxWorld) return false;
    const char* force = std::getenv("AMMON_B200_TP_NCCL");
    bool want = !(force && force[0] == '1');
    c->rt->activate();
    c->max_elems = (max_elems + 63) / 64 * 64;
    const size_t bytes = kTpRecvOff + 2 * c->max_elems * sizeof(float);
    static_assert(kTpFlagBytes <= kTpRecvOff, "flag block");
    cudaIpcMemHandle_t mine;
    std::memset(&mine, 0, sizeof(mine));
    int ok = 0;
    if (want && cudaMalloc(&c->local, bytes) == cudaSuccess &&
        cudaMemset(c->local, 0, bytes) == cudaSuccess &&
        cudaMalloc(&c->epoch, sizeof(uint64_t)) == cudaSuccess &&
        cudaMemset(c->epoch, 0, sizeof(uint64_t)) == cudaSuccess &&
        cudaIpcGetMemHandle(&mine, c->local) == cudaSuccess)
        ok = 1;
    cudaGetLastError();
    std::vector<cudaIpcMemHandle_t> all(c->world);
    allgather_host(c, &mine, all.data(), sizeof(mine));
    // every rank opens every peer's block; all must succeed or none use the path
    for (int r = 0; r < c->world && ok; r++) {
        if (r == c->rank) {
            c->peer_base[r] = c->local;
            continue;
        }
        void* ptr = nullptr;
        if (cudaIpcOpenMemHandle(&ptr, all[r], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            ok = 0;
        } else {
            c->peer_base[r] = (unsigned char*)ptr;
        }
    }
    std::vector<int> oks(c->world);
    allgather_host(c, &ok, oks.data(), sizeof(int));
    bool every = true;
    for (int v : oks) every = every && v == 1;
    if (!every) {
        comm_peers_release(c);
        return false;
    }
    c->peers = true;
    return true;
}

void comm_peers_release(ab_comm* c) {
    for (int r = 0; r < (int)kTpMaxWorld; r++) {
        if (c->peer_base[r] && r != c->rank) cudaIpcCloseMemHandle(c->peer_base[r]);
        c->peer_base[r] = nullptr;
    }
    if (c->local) cudaFree(c->local);
    if (c->epoch) cudaFree(c->epoch);
    c->local = nullptr;
    c->epoch = nullptr;
    c->peers = false;
}

bool comm_has_peers(const ab_comm* c) { return c && c->peers; }

static void fused_block_release(ab_comm* c) {
    for (int r = 0; r < (int)kTpMaxWorld; r++) {
        if (c->fused_peer[r] && r != c->rank) cudaIpcCloseMemHandle(c->fused_peer[r]);
        c->fused_peer[r] = nullptr;
    }
    if (c->fused_local) cudaFree(c->fused_local);
    c->fused_local = nullptr;
    c->fused_bytes = 0;
}

bool comm_fused_block(ab_comm* c, size_t bytes, unsigned char** local,
                      unsigned char* peers[kTpMaxWorld]) {
    if (c->fused_local) {
        if (bytes > c->fused_bytes) fail(AB_ERR_ARGUMENT, "fused exchange block set up smaller");
    } else {
        if (c->world < 2 || c->world > (int)kTpMaxWorld) return false;
        c->rt->activate();
        cudaIpcMemHandle_t mine;
        std::memset(&mine, 0, sizeof(mine));
        int ok = 0;
        if (cudaMalloc(&c->fused_local, bytes) == cudaSuccess &&
            cudaMemset(c->fused_local, 0, bytes) == cudaSuccess &&
            cudaIpcGetMemHandle(&mine, c->fused_local) == cudaSuccess)
            ok = 1;
        cudaGetLastError();
        std::vector<cudaIpcMemHandle_t> all(c->world);
        allgather_host(c, &mine, all.data(), sizeof(mine));
        for (int r = 0; r < c->world && ok; r++) {
            if (r == c->rank) {
                c->fused_peer[r] = c->fused_local;
                continue;
            }
            void* ptr = nullptr;
            if (cudaIpcOpenMemHandle(&ptr, all[r], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                cudaGetLastError();
                ok = 0;
            } else {
                c->fused_peer[r] = (unsigned char*)ptr;
            }
        }
        std::vector<int> oks(c->world);
        allgather_host(c, &ok, oks.data(), sizeof(int));
        bool every = true;
        for (int v : oks) every = every && v == 1;
        if (!every) {
            fused_block_release(c);
            return false;
        }
        c->fused_bytes = bytes;
    }
    *local = c->fused_local;
    for (int r = 0; r < (int)kTpMaxWorld; r++) peers[r] = c->fused_peer[r];
    return true;
}
void comm_begin_recording(ab_comm* c) {
    if (c) c->next_site = 0;
}

__global__ void tp_epoch_kernel(uint64_t* epoch) {
    pdl_wait();
    *epoch += 1;
    pdl_trigger();
}

void record_tp_epoch(ab_scheme* s, ab_comm* c) {
    uint64_t* ep = c->epoch;
    s->add("tp_epoch", [=](cudaStream_t st) {
        return launch(st, dim3(1), dim3(1), 0, true, tp_epoch_kernel, ep);
    });
}

TpPush comm_push_target(ab_comm* c) {
    TpPush t = {};
    t.site = c->next_site++;
    t.out = tp_send(c, c->local, t.site & 1);
    return t;
}

// Every rank's send slot of one parity and this rank's flag in every rank's flag block,
// as this rank addresses them (its own, and the peers' through their IPC mappings).
struct TpSources {
    const float* src[kTpMaxWorld];
    uint64_t* flag[kTpMaxWorld];
};

// Announces this rank's partial of the site (stored by the projection kernel before this
// one in stream order, so it already sits in this GPU's memory where the peers read it),
// waits until every rank announced its own, then sums the ranks' partials in rank order
// into x, reading the peers' slots over NVLink (every rank adds the same values in the
// same order, so the replicated x stays bit-identical).
__global__ void __launch_bounds__(256) tp_reduce_kernel(const TpSources srcs,
                                                        const uint64_t* flags,
                                                        const uint64_t* epoch, uint32_t site,
                                                        uint32_t world, float* x, uint32_t n,
                                                        uint32_t* err) {
    pdl_wait();
    __shared__ int ok;
    const uint64_t want = tp_signal_value(*epoch, site);
    if (blockIdx.x == 0 && threadIdx.x < world) {
        __threadfence_system();
        asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(srcs.flag[threadIdx.x]),
                     "l"(want)
                     : "memory");
    }
    if (threadIdx.x == 0) ok = 1;
    __syncthreads();
    if (threadIdx.x < world) {
        const uint64_t* f = flags + threadIdx.x;
        uint64_t v;
        asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(f) : "memory");
        if (v < want) {
            WaitClock clock;
            while (true) {
                asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(f) : "memory");
                if (v >= want) break;
                if (clock.expired(err)) {
                    ok = 0;
                    break;
                }
            }
        }
    }
    __syncthreads();
    if (!ok) {
        if (threadIdx.x == 0) atomicOr(err, kFlagWaitTimeout);
        return;
    }
    if (n % 4 == 0) {
        // four elements per thread, every rank's load in flight before the sum
        for (uint32_t i = (blockIdx.x * blockDim.x + threadIdx.x) * 4; i < n;
             i += gridDim.x * blockDim.x * 4) {
            float4 v[kTpMaxWorld];
#pragma unroll
            for (uint32_t r = 0; r < kTpMaxWorld; r++)
                if (r < world) v[r] = __ldcv(reinterpret_cast<const float4*>(srcs.src[r] + i));
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (uint32_t r = 0; r < kTpMaxWorld; r++) {
                if (r < world) {
                    acc.x += v[r].x;
                    acc.y += v[r].y;
                    acc.z += v[r].z;
                    acc.w += v[r].w;
                }
            }
            *reinterpret_cast<float4*>(x + i) = acc;
        }
    } else {
        for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n;
             i += gridDim.x * blockDim.x) {
            float acc = 0.0f;
            for (uint32_t r = 0; r < world; r++) acc += __ldcv(srcs.src[r] + i);
            x[i] = acc;
        }
    }
    pdl_trigger();
}

void record_tp_reduce(ab_scheme* s, const char* label, ab_comm* c, const TpPush& push,
                      float* x, uint32_t n) {
    if (n > c->max_elems)
        fail(AB_ERR_ARGUMENT, "peer all-reduce of " + std::to_string(n) +
                                  " elements exceeds the send slots set up for " +
                                  std::to_string(c->max_elems));
    const uint32_t parity = push.site & 1;
    TpSources srcs = {};
    for (int r = 0; r < c->world; r++) {
        srcs.src[r] = tp_send(c, c->peer_base[r], parity);
        srcs.flag[r] = tp_flags(c->peer_base[r], parity) + c->rank;
    }
    const uint64_t* flags = tp_flags(c->local, parity);
    const uint64_t* ep = c->epoch;
    const uint32_t site = push.site, world = (uint32_t)c->world;
    uint32_t* err = c->rt->flags;
    // one float4 of every rank per thread: all of a batched step's peer loads in flight at
    // once (up to 64 rows x 4096 = 256 CTAs); a batch-1 row takes 4 CTAs
    const unsigned grid = std::max(1u, std::min(512u, (n + 1023) / 1024));
    s->add(label, [=](cudaStream_t st) {
        return launch(st, dim3(grid), dim3(256), 0, true, tp_reduce_kernel, srcs, flags, ep, site,
                      world, x, n, err);
    });
}

// Records an in-place or out-of-place float sum over the communicator.
void record_allreduce_f32(ab_scheme* s, const char* label, ab_comm* c, const float* send,
                          float* recv, size_t count) {
    NcclApi& api = nccl();
    ncclComm_t comm = c->comm;
    s->add(label, [=, &api](cudaStream_t st) {
        ncclResult_t r = api.all_reduce(send, recv, count, ncclFloat32, ncclSum, comm, st);
        if (r != ncclSuccess) {
            g_nccl_error = api.error_string(r);
            return cudaErrorUnknown;
        }
        return cudaSuccess;
    });
}

// Records an all-gather of `bytes` per rank (recv holds world * bytes).
void record_allgather_bytes(ab_scheme* s, const char* label, ab_comm* c, const void* send,
                            void* recv, size_t bytes) {
    NcclApi& api = nccl();
    ncclComm_t comm = c->comm;
    s->add(label, [=, &api](cudaStream_t st) {
        ncclResult_t r = api.all_gather(send, recv, bytes, ncclUint8, comm, st);
        if (r != ncclSuccess) {
            g_nccl_error = api.error_string(r);
            return cudaErrorUnknown;
        }
        return cudaSuccess;
    });
}

}  // namespace ab

namespace ab {

// Polls a nonblocking communicator until its pending operation ends; false when `deadline`
// (steady clock) passes first. Throws on an NCCL error.
static bool nccl_settle(ncclComm_t comm, std::chrono::steady_clock::time_point deadline,
                        const char* what) {
    while (true) {
        ncclResult_t st = ncclInProgress;
        nccl_check(nccl().get_async_error(comm, &st), what);
        if (st == ncclSuccess) return true;
        if (st != ncclInProgress) nccl_check(st, what);
        if (std::chrono::steady_clock::now() > deadline) return false;
        std::this_thread::sleep_for(std::chrono::milliseconds(1));
    }
}

// Creates the rank's communicator in two stages so that a rank that never joins ends the
// call instead of blocking it forever. Stage 1, the rendezvous: a nonblocking communicator on
// the caller's id, polled until every rank joined or `timeout_ms` passed; on timeout it is
// aborted (ncclCommAbort) and the call fails. Over it rank 0 broadcasts a fresh id, and the
// rendezvous communicator is finalised and destroyed. Stage 2: the blocking communicator on
// the fresh id that the step's collectives use (captured into CUDA graphs, which a nonblocking
// communicator's deferred launches would not allow); every rank is known alive by then.
static ncclComm_t comm_init_bounded(Runtime* rt, const ncclUniqueId& id, int world, int rank,
                                    uint32_t timeout_ms) {
    NcclApi& api = nccl();
    const auto deadline =
        std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclComm_t probe = nullptr;
    ncclResult_t r = api.comm_init_rank_config(&probe, world, id, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) nccl_check(r, "ncclCommInitRankConfig");
    auto give_up = [&](const std::string& why) {
        api.comm_abort(probe);
        fail(AB_ERR_NCCL, why + " (rendezvous communicator aborted)");
    };
    bool ok = false;
    try {
        ok = nccl_settle(probe, deadline, "communicator rendezvous");
    } catch (...) {
        api.comm_abort(probe);
        throw;
    }
    if (!ok)
        give_up("not every one of the " + std::to_string(world) + " ranks joined the "
                "communicator within " + std::to_string(timeout_ms) + " ms");
    ncclUniqueId fresh = {};
    if (rank == 0) {
        r = api.get_unique_id(&fresh);
        if (r != ncclSuccess) give_up(std::string("ncclGetUniqueId: ") + api.error_string(r));
    }
    unsigned char* d = nullptr;
    if (cudaMalloc(&d, sizeof(fresh)) != cudaSuccess) give_up("cudaMalloc of the id buffer");
    cudaError_t e = cudaMemcpy(d, &fresh, sizeof(fresh), cudaMemcpyHostToDevice);
    r = e == cudaSuccess ? api.broadcast(d, d, sizeof(fresh), ncclUint8, 0, probe, rt->stream)
                         : ncclSuccess;
    bool done = e == cudaSuccess && (r == ncclSuccess || r == ncclInProgress) &&
                nccl_settle(probe, deadline, "id broadcast");
    // the broadcast's kernel ends once every rank took part; wait for it, bounded
    while (done) {
        e = cudaStreamQuery(rt->stream);
        if (e == cudaSuccess) break;
        if (e != cudaErrorNotReady || std::chrono::steady_clock::now() > deadline) {
            done = false;
            break;
        }
        std::this_thread::sleep_for(std::chrono::milliseconds(1));
    }
    if (done) done = cudaMemcpy(&fresh, d, sizeof(fresh), cudaMemcpyDeviceToHost) == cudaSuccess;
    if (!done) {
        api.comm_abort(probe);
        cudaStreamSynchronize(rt->stream);
        cudaFree(d);
        fail(AB_ERR_NCCL, "id broadcast over the rendezvous communicator did not complete "
                          "within " + std::to_string(timeout_ms) + " ms (aborted)");
    }
    cudaFree(d);
    r = api.comm_finalize(probe);
    if ((r != ncclSuccess && r != ncclInProgress) || !nccl_settle(probe, deadline, "finalize"))
        give_up("rendezvous communicator did not finalise");
    api.comm_destroy(probe);
    ncclComm_t comm = nullptr;
    nccl_check(api.comm_init_rank(&comm, world, fresh, rank), "ncclCommInitRank");
    return comm;
}

static uint32_t env_comm_timeout_ms() {
    if (const char* e = std::getenv("AMMON_B200_COMM_TIMEOUT_MS")) {
        const long v = std::atol(e);
        if (v > 0) return (uint32_t)v;
    }
    return 300000;
}

}  // namespace ab

using namespace ab;

extern "C" {

int ab_comm_unique_id(uint8_t* id) {
    return guard([&] {
        if (!id) fail(AB_ERR_ARGUMENT, "null id buffer");
        ncclUniqueId u;
        nccl_check(nccl().get_unique_id(&u), "ncclGetUniqueId");
        std::memcpy(id, u.internal, NCCL_UNIQUE_ID_BYTES);
    });
}

int ab_comm_create_timeout(ab_runtime* rt, const uint8_t* id, int32_t rank, int32_t world,
                           uint32_t timeout_ms, ab_comm** out) {
    return guard([&] {
        if (!rt || !id || !out) fail(AB_ERR_ARGUMENT, "null argument");
        if (world < 1 || rank < 0 || rank >= world) fail(AB_ERR_ARGUMENT, "bad rank / world");
        if (timeout_ms == 0) fail(AB_ERR_ARGUMENT, "timeout must be at least 1 ms");
        ncclUniqueId u;
        std::memcpy(u.internal, id, NCCL_UNIQUE_ID_BYTES);
        rt->activate();
        ncclComm_t comm = comm_init_bounded(rt, u, world, rank, timeout_ms);
        auto* c = new ab_comm();
        c->rt = rt;
        c->rank = rank;
        c->world = world;
        c->comm = comm;
        *out = c;
    });
}

int ab_comm_create(ab_runtime* rt, const uint8_t* id, int32_t rank, int32_t world,
                   ab_comm** out) {
    return ab_comm_create_timeout(rt, id, rank, world, env_comm_timeout_ms(), out);
}

// A one-rank run of the all-reduce kernel over `world` slots in this GPU's memory; the
// arrivals of the ranks not in `ready` are never written.
int ab_comm_loopback_reduce(ab_runtime* rt, uint32_t world, uint32_t ready, uint32_t n,
                            float* out) {
    return guard([&] {
        if (!rt || !out) fail(AB_ERR_ARGUMENT, "null argument");
        if (world < 1 || world > kTpMaxWorld) fail(AB_ERR_ARGUMENT, "world must be 1..8");
        if (n == 0 || n > (1u << 24)) fail(AB_ERR_ARGUMENT, "n must be 1..2^24");
        rt->activate();
        // [arrivals: kTpMaxWorld u64][sinks for the peers' copies: kTpMaxWorld u64][epoch u64]
        // [pad to 256][world slots of n floats][n floats of result]
        const size_t bytes = 256 + ((size_t)world + 1) * n * 4;
        unsigned char* d = nullptr;
        cuda_check(cudaMalloc(&d, bytes), "cudaMalloc");
        uint64_t* arrivals = reinterpret_cast<uint64_t*>(d);
        uint64_t* sinks = arrivals + kTpMaxWorld;
        uint64_t* epoch = sinks + kTpMaxWorld;
        float* slots = reinterpret_cast<float*>(d + 256);
        float* x = slots + (size_t)world * n;
        std::vector<uint64_t> head(32, 0);
        const uint64_t ep = 1;
        const uint32_t site = 0;
        for (uint32_t r = 1; r < world; r++)
            if (ready & (1u << r)) head[r] = tp_signal_value(ep, site);
        head[2 * kTpMaxWorld] = ep;
        std::vector<float> h((size_t)world * n);
        for (uint32_t r = 0; r < world; r++)
            for (uint32_t i = 0; i < n; i++) h[(size_t)r * n + i] = (float)(r + 1) + 0.25f * (i % 7);
        TpSources srcs = {};
        for (uint32_t r = 0; r < world; r++) {
            srcs.src[r] = slots + (size_t)r * n;
            srcs.flag[r] = r == 0 ? arrivals : sinks + r;
        }
        // one float4 of every rank per thread: all of a batched step's peer loads in flight at
    // once (up to 64 rows x 4096 = 256 CTAs); a batch-1 row takes 4 CTAs
    const unsigned grid = std::max(1u, std::min(512u, (n + 1023) / 1024));
        cudaError_t e = cudaMemset(d, 0, bytes);
        if (e == cudaSuccess) e = cudaMemcpy(d, head.data(), head.size() * 8, cudaMemcpyHostToDevice);
        if (e == cudaSuccess)
            e = cudaMemcpy(slots, h.data(), h.size() * 4, cudaMemcpyHostToDevice);
        if (e == cudaSuccess)
            e = launch(rt->stream, dim3(grid), dim3(256), 0, false, tp_reduce_kernel, srcs,
                       (const uint64_t*)arrivals, (const uint64_t*)epoch, site, world, x, n,
                       rt->flags);
        if (e == cudaSuccess) e = cudaStreamSynchronize(rt->stream);
        if (e == cudaSuccess) e = cudaMemcpy(out, x, (size_t)n * 4, cudaMemcpyDeviceToHost);
        cudaFree(d);
        cuda_check(e, "loopback all-reduce");
        rt->check_flags();
    });
}

int ab_comm_destroy(ab_comm* c) {
    return guard([&] {
        if (!c) return;
        c->rt->activate();
        cudaStreamSynchronize(c->rt->stream);
        if (c->peers && c->comm) {
            // every rank is done writing into its peers before any block goes away
            int one = 1;
            std::vector<int> all(c->world);
            try {
                allgather_host(c, &one, all.data(), sizeof(int));
            } catch (...) {
            }
        }
        comm_peers_release(c);
        fused_block_release(c);
        if (c->comm) nccl().comm_destroy(c->comm);
        delete c;
    });
}

int ab_comm_abort(ab_comm* c) {
    return guard([&] {
        if (!c) return;
        if (c->comm) nccl().comm_abort(c->comm);
        c->comm = nullptr;
    });
}

int ab_comm_rank(const ab_comm* c, int32_t* rank, int32_t* world) {
    return guard([&] {
        if (!c) fail(AB_ERR_ARGUMENT, "null communicator");
        if (rank) *rank = c->rank;
        if (world) *world = c->world;
    });
}

const char* ab_comm_last_error(void) { return g_nccl_error.c_str(); }

}  // extern "C"
