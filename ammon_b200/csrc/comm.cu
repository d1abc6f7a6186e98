// NCCL communicator for tensor parallelism over NVLink / NVSwitch.
//
// NCCL is resolved at run time with dlopen: when the process already loaded libnccl.so.2
// (torch.distributed does), that instance is used, so one process never holds two NCCL
// libraries. Collectives are recorded into schemes like kernels and are captured into the
// step's CUDA graph.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

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
        api.error_string = (decltype(api.error_string))sym("ncclGetErrorString");
        api.ok = api.get_unique_id && api.comm_init_rank && api.all_reduce && api.all_gather &&
                 api.comm_destroy && api.comm_abort && api.error_string;
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
};

namespace ab {

int comm_rank(const ab_comm* c) { return c ? c->rank : 0; }
int comm_world(const ab_comm* c) { return c ? c->world : 1; }

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

int ab_comm_create(ab_runtime* rt, const uint8_t* id, int32_t rank, int32_t world,
                   ab_comm** out) {
    return guard([&] {
        if (!rt || !id || !out) fail(AB_ERR_ARGUMENT, "null argument");
        if (world < 1 || rank < 0 || rank >= world) fail(AB_ERR_ARGUMENT, "bad rank / world");
        ncclUniqueId u;
        std::memcpy(u.internal, id, NCCL_UNIQUE_ID_BYTES);
        rt->activate();
        auto* c = new ab_comm();
        c->rt = rt;
        c->rank = rank;
        c->world = world;
        ncclResult_t r = nccl().comm_init_rank(&c->comm, world, u, rank);
        if (r != ncclSuccess) {
            delete c;
            nccl_check(r, "ncclCommInitRank");
        }
        *out = c;
    });
}

int ab_comm_destroy(ab_comm* c) {
    return guard([&] {
        if (!c) return;
        c->rt->activate();
        cudaStreamSynchronize(c->rt->stream);
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
