// gpb2_nvtx.h -- NVTX ranges of the library (no-ops unless a profiler is attached): one range per
// C entry point, named after it (the operation), and one per depth batch ("forward level b",
// "reverse level b") in the host-driven batch loops -- the per-batch sweep modes and the
// level-sharded schedule.  The persistent sweeps walk every batch inside one launch and carry
// only the operation's range.
#pragma once

#include <nvtx3/nvToolsExt.h>

#include <cstdio>

namespace gpb2 {

struct NvtxRange {
    explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
    NvtxRange(const char* what, long long level) {
        char b[64];
        std::snprintf(b, sizeof b, "%s level %lld", what, level);
        nvtxRangePushA(b);
    }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange&) = delete;
    NvtxRange& operator=(const NvtxRange&) = delete;
};

}  // namespace gpb2
