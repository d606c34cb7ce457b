// NVTX ranges around the C-ABI entry points, so that Nsight Systems shows each call on the host
// timeline and `ncu --nvtx --nvtx-include "bolt3_prefill_fwd/"` profiles only the kernels one entry
// point launches. The header-only NVTX3 API of the CUDA toolkit is used: with no tool attached a
// push or pop is one test of a null function pointer; with one attached, the first call loads it.
// The ranges go to NVTX's default domain, the one torch.cuda.nvtx writes, so the Python module's
// ranges and these nest in one stack per thread.
#pragma once

#include <nvtx3/nvToolsExt.h>

namespace b3 {

class TraceRange {
 public:
  explicit TraceRange(const char* name) { nvtxRangePushA(name); }
  ~TraceRange() { nvtxRangePop(); }
  TraceRange(const TraceRange&) = delete;
  TraceRange& operator=(const TraceRange&) = delete;
};

}  // namespace b3
