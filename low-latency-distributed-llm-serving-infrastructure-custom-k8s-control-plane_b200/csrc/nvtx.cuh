// NVTX ranges for a timeline profile: one range per C-ABI call that enqueues kernels, named for
// the entry point, so a trace shows which call launched which kernels.  NVTX v3 is header-only;
// with no tool attached a push/pop costs a check of a null function pointer.
#pragma once

#include <nvtx3/nvToolsExt.h>

namespace b200 {

struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

}  // namespace b200
