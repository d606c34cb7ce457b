// Prefill phases B + C for callers that cannot allocate device memory.
//
// bolt3_prefill_fwd needs a snapshot workspace between its consolidation scan and its attention.
// Some hosts cannot provide one from their hot path: a serving engine that reserved all of HBM for
// its own pool at start-up and hands out only fixed tensors, a non-Python host calling the C-ABI
// that has no device allocator of its own, or a latency-critical loop where cudaMalloc's implicit
// device-wide synchronisation is not acceptable. This entry point takes the workspace from a
// fixed-size array that the library itself reserves on every GPU it is used on.
#include <mutex>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "../../include/bolt3.h"
#include "common.cuh"
#include "trace.h"

namespace {

// One array per GPU (per CUDA context) that uses the library, held until the process exits.
__device__ __align__(256) unsigned char g_noalloc_scratch[BOLT3_NOALLOC_SCRATCH_BYTES];

// In host code the array's name only stands in for the symbol: its device address depends on the
// context the library's module is loaded into. The address is looked up with cudaGetSymbolAddress
// while that context is current, once per context, and cached under the driver's unique context
// id (cuCtxGetId), so a host that drives its own contexts, or recreates one after
// cudaDeviceReset, never receives an address from another context.
constexpr int kCacheSlots = 64;
struct CacheEntry {
  unsigned long long ctx_id;
  void* ptr;
};
CacheEntry g_cache[kCacheSlots] = {};
int g_cache_next = 0;
std::mutex g_cache_mu;

struct CtxFns {
  PFN_cuCtxGetCurrent_v4000 current = nullptr;
  PFN_cuCtxGetId_v12000 id = nullptr;
};

const CtxFns& ctx_fns() {
  static CtxFns f;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      f.current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      f.id = reinterpret_cast<PFN_cuCtxGetId_v12000>(p);
  });
  return f;
}

int lookup_symbol(void** out) {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return BOLT3_ERR_CUDA;
  *out = p;
  return BOLT3_OK;
}

// Device address of g_noalloc_scratch in the calling thread's current context.
int scratch_in_current_context(void** out) {
  const CtxFns& f = ctx_fns();
  if (!f.current || !f.id) return lookup_symbol(out);  // no context ids: look it up on every call
  CUcontext ctx = nullptr;
  if (f.current(&ctx) != CUDA_SUCCESS) return BOLT3_ERR_CUDA;
  if (ctx == nullptr) {
    // no context is current yet: the runtime binds the current device's primary context here
    const int rc = lookup_symbol(out);
    if (rc != BOLT3_OK) return rc;
    if (f.current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return BOLT3_ERR_CUDA;
  }
  unsigned long long id = 0;
  if (f.id(ctx, &id) != CUDA_SUCCESS) return BOLT3_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_cache_mu);
  for (int i = 0; i < kCacheSlots; ++i)
    if (g_cache[i].ptr != nullptr && g_cache[i].ctx_id == id) {
      *out = g_cache[i].ptr;
      return BOLT3_OK;
    }
  void* p = nullptr;
  const int rc = lookup_symbol(&p);
  if (rc != BOLT3_OK) return rc;
  g_cache[g_cache_next] = CacheEntry{id, p};
  g_cache_next = (g_cache_next + 1) % kCacheSlots;
  *out = p;
  return BOLT3_OK;
}

}  // namespace

extern "C" int bolt3_prefill_fwd_noalloc(const bolt3_prefill_args* a, void* stream) {
  const b3::TraceRange trace_range("bolt3_prefill_fwd_noalloc");
  if (!a) return BOLT3_ERR_ARG;
  if (a->B <= 0 || a->T <= 0 || a->HKV <= 0 || a->H % a->HKV || (a->HD != 64 && a->HD != 128))
    return BOLT3_ERR_SHAPE;
  const size_t need = bolt3_prefill_workspace_size(a->B * a->HKV, a->T, a->HD);
  if (need > (size_t)BOLT3_NOALLOC_SCRATCH_BYTES) return BOLT3_ERR_CAPACITY;
  void* scratch = nullptr;
  const int rc = scratch_in_current_context(&scratch);
  if (rc != BOLT3_OK) return rc;
  // Every snapshot slot the attention reads is written earlier in the same call, so whatever a
  // previous call left in the array needs no clearing.
  bolt3_prefill_args b = *a;
  b.workspace = scratch;
  b.workspace_bytes = (size_t)BOLT3_NOALLOC_SCRATCH_BYTES;
  return bolt3_prefill_fwd(&b, stream);
}
