#pragma once
// trace.h -- NVTX ranges around the host-side calls of the backend.
//
// The reference traces with `tracing` macros at model load and decode
// (src/engine/mod.rs:626-683,1163) and has no timers beyond the bench's
// Instant.  Here every public model call and every device step opens an NVTX
// range (header-only NVTX v3: without a profiler attached the calls return at
// once), so an Nsight timeline shows which API call and which step size each
// kernel belongs to.
#include <nvtx3/nvToolsExt.h>

#include <cstdio>

namespace nx {

struct TraceRange {
    explicit TraceRange(const char *name) { nvtxRangePushA(name); }
    // "<name> <n>": e.g. the token count of a step
    TraceRange(const char *name, long long n) {
        char buf[64];
        snprintf(buf, sizeof(buf), "%s %lld", name, n);
        nvtxRangePushA(buf);
    }
    ~TraceRange() { nvtxRangePop(); }
    TraceRange(const TraceRange &) = delete;
    TraceRange &operator=(const TraceRange &) = delete;
};

}  // namespace nx
