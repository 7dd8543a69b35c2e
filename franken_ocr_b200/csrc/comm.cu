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

__global__ void top1_pack_kernel(const float *__restrict__ val, const int32_t *__restrict__ idx,
                                 int m, uint64_t *__restrict__ out) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r < m)
        out[r] = ((uint64_t)(uint32_t)idx[r] << 32) | (uint64_t)__float_as_uint(val[r]);
}

// argmax_row across shards in rank order: first maximum (v <= best keeps the
// earlier shard, whose vocab range is lower), NaN and empty shards skipped,
// all-NaN -> 0 (sampler.rs:168-186).
__global__ void top1_combine_kernel(const uint64_t *__restrict__ all, int world, int m,
                                    uint32_t *__restrict__ token, float *__restrict__ token_val) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= m) return;
    int32_t b = -1;
    float bv = 0.0f;
    for (int s = 0; s < world; s++) {
        const uint64_t p = all[(size_t)s * m + r];
        const int32_t i = (int32_t)(p >> 32);
        const float v = __uint_as_float((uint32_t)p);
        if (i < 0 || v != v) continue;
        if (b >= 0 && v <= bv) continue;
        b = i;
        bv = v;
    }
    token[r] = b < 0 ? 0u : (uint32_t)b;
    if (token_val) token_val[r] = b < 0 ? __int_as_float(0x7fc00000) : bv;
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

int focr_top1_allgather(focr_comm *c, const float *best_val, const int32_t *best_idx, size_t m,
                        uint32_t *token, float *token_val, void *stream) {
    if (!c) return fail(FOCR_E_ARG, "top1_allgather: null communicator");
    if (m == 0) return FOCR_OK;
    if (!best_val || !best_idx || !token) return fail(FOCR_E_ARG, "top1_allgather: null pointer");
    if (m > (1u << 24)) return fail(FOCR_E_UNSUPPORTED, "top1_allgather: m too large");
    cudaStream_t st = (cudaStream_t)stream;
    if (m > c->top1_rows) {
        cudaFree(c->top1_send);
        cudaFree(c->top1_recv);
        c->top1_send = c->top1_recv = nullptr;
        c->top1_rows = 0;
        cudaError_t e = cudaMalloc(&c->top1_send, m * 8);
        if (e == cudaSuccess) e = cudaMalloc(&c->top1_recv, m * 8 * c->world);
        if (e != cudaSuccess) return fail(FOCR_E_ALLOC, "top1_allgather: cudaMalloc failed");
        c->top1_rows = m;
    }
    const unsigned g = (unsigned)((m + 255) / 256);
    top1_pack_kernel<<<g, 256, 0, st>>>(best_val, best_idx, (int)m, c->top1_send);
    FOCR_CUDA_TRY(cudaGetLastError());
    int rc = comm_all_gather_bytes(c, c->top1_send, c->top1_recv, m * 8, st);
    if (rc) return rc;
    top1_combine_kernel<<<g, 256, 0, st>>>(c->top1_recv, (int)c->world, (int)m, token, token_val);
    FOCR_CUDA_TRY(cudaGetLastError());
    return FOCR_OK;
}

int focr_comm_destroy(focr_comm *c) {
    if (!c) return FOCR_OK;
    cudaFree(c->top1_send);
    cudaFree(c->top1_recv);
    CommImpl *impl = static_cast<CommImpl *>(c->impl);
    if (impl && impl->comm) nccl().comm_destroy(impl->comm);
    delete impl;
    delete c;
    return FOCR_OK;
}

}  // extern "C"
