// SwiGLU's elementwise step of the hybrid model's MLP: y = silu(g) * u from one [rows][2I] bf16 GEMM
// output whose first I columns are the gate projection and the last I the up projection.
//
// Replaces `F.silu(gate_proj(x)) * up_proj(x)` (vsa_lm/surgery.py:202-211) after the two projections
// are one GEMM, with torch's bf16 roundings: silu in fp32 (x / (1 + exp(-x))) rounded to bf16, then the
// product rounded to bf16. HBM-bound elementwise work, 16-byte accesses.
#include "../../include/bolt3.h"
#include "common.cuh"
#include "trace.h"

#include <algorithm>

namespace {

using namespace b3;

__global__ void __launch_bounds__(256) silu_mul_kernel(const bolt3_silu_mul_args a) {
  const int64_t per_row = a.I / 8;                    // 16-byte pieces of an output row
  const int64_t n = a.rows * per_row;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / per_row, c = i % per_row;
    const bf16* row = reinterpret_cast<const bf16*>(a.gu) + r * 2 * a.I;
    const uint4 g = reinterpret_cast<const uint4*>(row)[c];
    const uint4 u = reinterpret_cast<const uint4*>(row + a.I)[c];
    const uint32_t gw[4] = {g.x, g.y, g.z, g.w}, uw[4] = {u.x, u.y, u.z, u.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 gf = unpack_bf16(gw[e]), uf = unpack_bf16(uw[e]);
      uint32_t sp;
      const float2 s = rbf2(gf.x / (1.0f + expf(-gf.x)), gf.y / (1.0f + expf(-gf.y)), sp);
      o[e] = pack_bf16(__fmul_rn(s.x, uf.x), __fmul_rn(s.y, uf.y));
    }
    reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(a.y) + r * a.I)[c] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace

extern "C" int bolt3_silu_mul(const bolt3_silu_mul_args* a, void* stream) {
  const b3::TraceRange trace_range("bolt3_silu_mul");
  if (!a || !a->gu || !a->y) return BOLT3_ERR_ARG;
  if (a->rows < 0 || a->I <= 0 || a->I % 8) return BOLT3_ERR_SHAPE;
  if (a->rows == 0) return BOLT3_OK;
  if ((uintptr_t)a->gu % 16 || (uintptr_t)a->y % 16) return BOLT3_ERR_ALIGN;
  const int64_t n = a->rows * (a->I / 8);
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, (int64_t)sms * 8);
  silu_mul_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(*a);
  return cudaGetLastError() == cudaSuccess ? BOLT3_OK : BOLT3_ERR_CUDA;
}
