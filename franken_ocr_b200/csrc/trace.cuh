// Opt-in device event trace (the GPU counterpart of the reference's
// FOCR_PROFILE_DECODE per-phase counters, native_engine/decoder.rs:986-1024).
//
// When a caller registers a device buffer with focr_trace_set(), the
// tensor-core kernels append one 16-byte event per (CTA, job, phase) with the
// %globaltimer nanosecond clock; with no buffer registered every record site
// is a single predicated-off branch.
#pragma once

#include <stdint.h>

namespace focr {

struct TraceEvent {
    uint32_t tag;    // kernel id << 24 | cta << 12 | job
    uint32_t phase;  // TracePhase
    uint64_t ns;     // %globaltimer
};

enum TracePhase : uint32_t {
    TR_KERNEL_START = 0,   // setup done (barriers, TMEM), before the dependency wait
    TR_DEPS_READY = 1,     // predecessor grid complete
    TR_JOB_LOAD = 2,       // producer issues the job's first stage
    TR_JOB_MMA = 3,        // MMA warp sees the job's first full stage
    TR_JOB_MMA_DONE = 4,   // MMA warp committed the job's accumulator
    TR_JOB_EPI = 5,        // epilogue sees the accumulator
    TR_JOB_EPI_DONE = 6,   // epilogue released the accumulator
    TR_KERNEL_END = 7,
    TR_MARK = 8,           // numbered checkpoint of a single-pass kernel (job = checkpoint)
};

struct TraceBuf {
    TraceEvent *ev;
    unsigned long long *count;
    unsigned long long cap;
};

// Host copy of the registered buffer; launchers copy it into each kernel's
// parameters (no relocatable device code needed).
TraceBuf host_trace();

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void trace_event(const TraceBuf &tb, uint32_t kernel, uint32_t job,
                                            uint32_t phase) {
    if (!tb.ev) return;
    const unsigned long long i = atomicAdd(tb.count, 1ull);
    if (i >= tb.cap) return;
    TraceEvent e;
    e.tag = (kernel << 24) | ((blockIdx.x & 0xFFFu) << 12) | (job & 0xFFFu);
    e.phase = phase;
    e.ns = globaltimer_ns();
    tb.ev[i] = e;
}

// Record into a fixed slot (no counter): for kernels whose events have a
// known place, e.g. (CTA, checkpoint); `count` is left to the caller.
__device__ __forceinline__ void trace_event_slot(const TraceBuf &tb, unsigned long long slot,
                                                 uint32_t kernel, uint32_t job, uint32_t phase) {
    if (!tb.ev || slot >= tb.cap) return;
    TraceEvent e;
    e.tag = (kernel << 24) | ((blockIdx.x & 0xFFFu) << 12) | (job & 0xFFFu);
    e.phase = phase;
    e.ns = globaltimer_ns();
    tb.ev[slot] = e;
}

}  // namespace focr
