// trace.h -- NVTX ranges around the C ABI's entry points, for timelines in
// Nsight Systems and for ncu's NVTX filters. Off unless the environment has
// HESA_CUDA_NVTX=1 (read once per process); then each traced entry point
// pushes a range named after itself on the calling host thread and pops it
// on return. The ranges cover host-side validation and enqueueing: the
// kernels run later on their stream (and a captured CUDA graph replays
// without them). NVTX v3 is header-only; with no tool attached the calls do
// nothing.
#pragma once

#include <nvtx3/nvToolsExt.h>

#include <cstdlib>

namespace hesa_cuda {

inline bool trace_enabled() {
    static const bool on = [] {
        const char* v = std::getenv("HESA_CUDA_NVTX");
        return v != nullptr && v[0] == '1' && v[1] == '\0';
    }();
    return on;
}

struct TraceScope {
    bool on;
    explicit TraceScope(const char* name) : on(trace_enabled()) {
        if (on) nvtxRangePushA(name);
    }
    ~TraceScope() {
        if (on) nvtxRangePop();
    }
    TraceScope(const TraceScope&) = delete;
    TraceScope& operator=(const TraceScope&) = delete;
};

}  // namespace hesa_cuda

#define HESA_TRACE(name) ::hesa_cuda::TraceScope hesa_trace_scope_(name)
