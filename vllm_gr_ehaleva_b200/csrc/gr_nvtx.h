// gr_nvtx.h — one NVTX range per C-ABI call, named after the entry point, so
// that a profiler's timeline groups each call's kernels under it.  NVTX is
// header-only; without a profiler attached a range costs a few nanoseconds.
#pragma once
#include <nvtx3/nvToolsExt.h>

namespace gr {
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};
}  // namespace gr
