// Communicator internals shared by the expert-parallel and vocab-parallel paths.
#pragma once

#include "common.cuh"

#define FOCR_MAX_WORLD 8

struct focr_comm {
    uint32_t rank = 0, world = 1;
    int device = 0;
    void *impl = nullptr;          // NCCL communicator (comm.cu)
    // vocab-parallel top-1 exchange buffers (grown on demand)
    uint64_t *top1_send = nullptr, *top1_recv = nullptr;
    size_t top1_rows = 0;
};

namespace focr {

// All-gather `bytes` from every rank into recv[world][bytes] (stream-ordered).
int comm_all_gather_bytes(focr_comm *c, const void *send, void *recv, size_t bytes,
                          cudaStream_t st);

// Bounded spin until *flag >= want (system-scope acquire); false after
// ~`limit_ns` of global time.  Used on flags that other GPUs write over NVLink.
__device__ __forceinline__ bool wait_flag_sys(const unsigned *flag, unsigned want,
                                              unsigned long long limit_ns) {
    unsigned long long t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    for (;;) {
        unsigned v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
        if ((int)(v - want) >= 0) return true;
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        if (t - t0 > limit_ns) return false;
        __nanosleep(32);
    }
}

__device__ __forceinline__ void store_release_sys(unsigned *flag, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flag), "r"(v) : "memory");
}

}  // namespace focr
