// focr_trace_set: register (or clear) the device event-trace buffer.
#include <mutex>

#include "common.cuh"
#include "trace.cuh"

namespace focr {

static std::mutex g_trace_mu;
static TraceBuf g_trace_host = {nullptr, nullptr, 0};

TraceBuf host_trace() {
    std::lock_guard<std::mutex> lock(g_trace_mu);
    return g_trace_host;
}

}  // namespace focr

extern "C" int focr_trace_set(void *events, unsigned long long *count, size_t capacity) {
    std::lock_guard<std::mutex> lock(focr::g_trace_mu);
    if (!events || !count || !capacity) {
        focr::g_trace_host = {nullptr, nullptr, 0};
        return FOCR_OK;
    }
    focr::g_trace_host = {static_cast<focr::TraceEvent *>(events), count, capacity};
    return FOCR_OK;
}
