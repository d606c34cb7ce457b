// Prefill phases B + C for callers that cannot allocate device memory.
//
// bolt3_prefill_fwd needs a snapshot workspace between its consolidation scan and its attention.
// Some hosts cannot provide one from their hot path: a serving engine that reserved all of HBM for
// its own pool at start-up and hands out only fixed tensors, a non-Python host calling the C-ABI
// that has no device allocator of its own, or a latency-critical loop where cudaMalloc's implicit
// device-wide synchronisation is not acceptable. This entry point takes the workspace from a
// fixed-size array that the library itself reserves on every GPU it is loaded on.
#include <mutex>

#include "../../include/bolt3.h"
#include "common.cuh"

namespace {

// One array per GPU that loads the library, held until the process exits.
__device__ __align__(256) unsigned char g_noalloc_scratch[BOLT3_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Device address of g_noalloc_scratch on the current device. In host code the array's name only
// stands in for the symbol, so the address is looked up (once per device, with that device current)
// and cached.
int scratch_on_current_device(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return BOLT3_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return BOLT3_ERR_CUDA;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return BOLT3_OK;
}

}  // namespace

extern "C" int bolt3_prefill_fwd_noalloc(const bolt3_prefill_args* a, void* stream) {
  if (!a) return BOLT3_ERR_ARG;
  if (a->B <= 0 || a->T <= 0 || a->HKV <= 0 || a->H % a->HKV || (a->HD != 64 && a->HD != 128))
    return BOLT3_ERR_SHAPE;
  const size_t need = bolt3_prefill_workspace_size(a->B * a->HKV, a->T, a->HD);
  if (need > (size_t)BOLT3_NOALLOC_SCRATCH_BYTES) return BOLT3_ERR_CAPACITY;
  void* scratch = nullptr;
  const int rc = scratch_on_current_device(&scratch);
  if (rc != BOLT3_OK) return rc;
  // Every snapshot slot the attention reads is written earlier in the same call, so whatever a
  // previous call left in the array needs no clearing.
  bolt3_prefill_args b = *a;
  b.workspace = scratch;
  b.workspace_bytes = (size_t)BOLT3_NOALLOC_SCRATCH_BYTES;
  return bolt3_prefill_fwd(&b, stream);
}
