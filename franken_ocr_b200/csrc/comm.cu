// Multi-GPU communicator (focr_comm): NCCL, loaded at run time.
//
// The library does not link NCCL: a host process that already loaded one
// (torch's, or the system's) keeps a single copy, and the CPU-only build and
// tests load the library without NCCL present.  dlopen first asks for an
// already-loaded libnccl.so.2 (RTLD_NOLOAD), then loads it by soname.
//
// A communicator is one NCCL communicator over `world` ranks (one process or
// thread per GPU).  It bootstraps the expert-parallel exchange (all-gather of
// the CUDA IPC handles of every rank's exchange region) and carries the
// vocab-parallel lm-head's all-gather of per-shard top-1 (value, index).
#include <dlfcn.h>
#include <nccl.h>

#include <mutex>

#include "comm.cuh"

namespace focr {

namespace {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    const char *(*error_string)(ncclResult_t) = nullptr;
    bool ok = false;
    std::string why;
};

NcclApi &nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            api.why = std::string("libnccl.so.2 not loadable: ") + dlerror();
            return;
        }
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
        api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_gather &&
                 api.error_string;
        if (!api.ok) api.why = "libnccl.so.2 lacks an expected symbol";
    });
    return api;
}

int nccl_fail(ncclResult_t r, const char *what) {
    return fail(FOCR_E_CUDA, std::string(what) + ": " + nccl().error_string(r));
}

}  // namespace

struct CommImpl {
    ncclComm_t comm = nullptr;
};

int comm_all_gather_bytes(focr_comm *c, const void *send, void *recv, size_t bytes,
                          cudaStream_t st) {
    NcclApi &api = nccl();
    ncclResult_t r = api.all_gather(send, recv, bytes, ncclUint8,
                                    static_cast<CommImpl *>(c->impl)->comm, st);
    if (r != ncclSuccess) return nccl_fail(r, "ncclAllGather");
    return FOCR_OK;
}

}  // namespace focr

using namespace focr;

extern "C" {

int focr_nccl_unique_id(void *id) {
    if (!id) return fail(FOCR_E_ARG, "nccl_unique_id: null pointer");
    NcclApi &api = nccl();
    if (!api.ok) return fail(FOCR_E_UNSUPPORTED, api.why);
    ncclUniqueId u;
    ncclResult_t r = api.get_unique_id(&u);
    if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
    memcpy(id, u.internal, NCCL_UNIQUE_ID_BYTES);
    return FOCR_OK;
}

int focr_comm_create(const void *nccl_id, uint32_t rank, uint32_t world, focr_comm **out) {
    if (!nccl_id || !out) return fail(FOCR_E_ARG, "comm_create: null argument");
    if (world == 0 || world > FOCR_MAX_WORLD || rank >= world)
        return fail(FOCR_E_ARG, "comm_create: need rank < world <= 8");
    NcclApi &api = nccl();
    if (!api.ok) return fail(FOCR_E_UNSUPPORTED, api.why);
    ncclUniqueId u;
    memcpy(u.internal, nccl_id, NCCL_UNIQUE_ID_BYTES);
    CommImpl *impl = new CommImpl();
    ncclResult_t r = api.comm_init_rank(&impl->comm, (int)world, u, (int)rank);
    if (r != ncclSuccess) {
        delete impl;
        return nccl_fail(r, "ncclCommInitRank");
    }
    focr_comm *c = new focr_comm();
    c->rank = rank;
    c->world = world;
    cudaGetDevice(&c->device);
    c->impl = impl;
    *out = c;
    return FOCR_OK;
}

int focr_comm_destroy(focr_comm *c) {
    if (!c) return FOCR_OK;
    CommImpl *impl = static_cast<CommImpl *>(c->impl);
    if (impl && impl->comm) nccl().comm_destroy(impl->comm);
    delete impl;
    delete c;
    return FOCR_OK;
}

}  // extern "C"
