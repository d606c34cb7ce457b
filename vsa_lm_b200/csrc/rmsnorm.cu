// RMSNorm of bf16 rows in one pass: y = bf16(x * rsqrt(mean(x^2) + eps) * w), fp32 inside.
//
// Replaces LlamaRMSNorm.forward (vsa_lm/surgery.py:43-53: the input cast to fp32, the normalisation,
// the weight product in fp32 and the cast back) for the hybrid model's block norms, final norm and the
// anchors' per-head q/k norms, which torch runs as four kernels each (two casts, the norm, a cast
// back); at decode sizes those launches, not bytes, are the cost. One warp per row: each lane reads
// 16-byte pieces of the row, the sum of squares is reduced across the warp, and the lane writes its
// pieces back normalised and scaled by the weight (bf16 or fp32, read as fp32). Few wide rows take a
// block each instead (rmsnorm_row_kernel).
#include "../../include/bolt3.h"
#include "common.cuh"
#include "trace.h"

namespace {

using namespace b3;

constexpr int kWarps = 8;

// x + r for eight bf16 pairs: each element added in fp32 and rounded to bf16 once (torch's bf16 add)
B3_DEV uint4 add_round(const uint4 x, const uint4 r) {
  const uint32_t xw[4] = {x.x, x.y, x.z, x.w}, rw[4] = {r.x, r.y, r.z, r.w};
  uint32_t o[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 a = unpack_bf16(xw[e]), b = unpack_bf16(rw[e]);
    o[e] = pack_bf16(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

template <int MAXV, bool WF32>
__global__ void __launch_bounds__(32 * kWarps) rmsnorm_kernel(const bolt3_rmsnorm_args a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarps + warp;
  if (row >= a.rows) return;
  const int nv = a.D / 8;                              // 16-byte pieces of a row
  const uint4* xr = reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(a.x) + row * a.x_stride);
  uint4 u[MAXV];
  float ss = 0.f;
  const uint4* rr = a.r ? reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(a.r) + row * a.D) : nullptr;
  uint4* sr = a.r ? reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(a.sum) + row * a.D) : nullptr;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c = lane + 32 * i;
    u[i] = c < nv ? xr[c] : make_uint4(0, 0, 0, 0);
    if (rr != nullptr && c < nv) {
      u[i] = add_round(u[i], rr[c]);
      sr[c] = u[i];
    }
    const uint32_t w4[4] = {u[i].x, u[i].y, u[i].z, u[i].w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = unpack_bf16(w4[e]);
      ss = fmaf(f.x, f.x, ss);
      ss = fmaf(f.y, f.y, ss);
    }
  }
  ss = warp_sum(ss);
  const float rs = rsqrtf(ss / (float)a.D + a.eps);
  uint4* yr = reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(a.y) + row * a.D);
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c = lane + 32 * i;
    if (c >= nv) break;
    float w[8];
    if constexpr (WF32) {
      const float4* wp = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.w) + c * 8);
      const float4 w0 = wp[0], w1 = wp[1];
      w[0] = w0.x; w[1] = w0.y; w[2] = w0.z; w[3] = w0.w; w[4] = w1.x; w[5] = w1.y; w[6] = w1.z; w[7] = w1.w;
    } else {
      const uint4 wu = reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(a.w))[c];
      const uint32_t ww[4] = {wu.x, wu.y, wu.z, wu.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack_bf16(ww[e]);
        w[2 * e] = f.x;
        w[2 * e + 1] = f.y;
      }
    }
    const uint32_t x4[4] = {u[i].x, u[i].y, u[i].z, u[i].w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = unpack_bf16(x4[e]);
      o[e] = pack_bf16(__fmul_rn(__fmul_rn(f.x, rs), w[2 * e]), __fmul_rn(__fmul_rn(f.y, rs), w[2 * e + 1]));
    }
    yr[c] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Few wide rows (a decode step's 64 hidden-state rows of 2560): one 256-thread block per row, so that
// the rows' loads spread over as many SMs as there are rows; each thread takes up to MAXC 16-byte
// pieces, and the sum of squares is reduced across the block.
template <int MAXC, bool WF32>
__global__ void __launch_bounds__(256) rmsnorm_row_kernel(const bolt3_rmsnorm_args a) {
  __shared__ float red[8];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t row = blockIdx.x;
  const int nv = a.D / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(a.x) + row * a.x_stride);
  uint4 u[MAXC];
  float ss = 0.f;
  const uint4* rr = a.r ? reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(a.r) + row * a.D) : nullptr;
  uint4* sr = a.r ? reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(a.sum) + row * a.D) : nullptr;
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = tid + 256 * i;
    u[i] = c < nv ? xr[c] : make_uint4(0, 0, 0, 0);
    if (rr != nullptr && c < nv) {
      u[i] = add_round(u[i], rr[c]);
      sr[c] = u[i];
    }
    const uint32_t w4[4] = {u[i].x, u[i].y, u[i].z, u[i].w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = unpack_bf16(w4[e]);
      ss = fmaf(f.x, f.x, ss);
      ss = fmaf(f.y, f.y, ss);
    }
  }
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) tot += red[w];
  const float rs = rsqrtf(tot / (float)a.D + a.eps);
  uint4* yr = reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(a.y) + row * a.D);
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = tid + 256 * i;
    if (c >= nv) break;
    float w[8];
    if constexpr (WF32) {
      const float4* wp = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.w) + c * 8);
      const float4 w0 = wp[0], w1 = wp[1];
      w[0] = w0.x; w[1] = w0.y; w[2] = w0.z; w[3] = w0.w; w[4] = w1.x; w[5] = w1.y; w[6] = w1.z; w[7] = w1.w;
    } else {
      const uint4 wu = reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(a.w))[c];
      const uint32_t ww[4] = {wu.x, wu.y, wu.z, wu.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack_bf16(ww[e]);
        w[2 * e] = f.x;
        w[2 * e + 1] = f.y;
      }
    }
    const uint32_t x4[4] = {u[i].x, u[i].y, u[i].z, u[i].w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = unpack_bf16(x4[e]);
      o[e] = pack_bf16(__fmul_rn(__fmul_rn(f.x, rs), w[2 * e]), __fmul_rn(__fmul_rn(f.y, rs), w[2 * e + 1]));
    }
    yr[c] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

template <int MAXV>
void launch_v(const bolt3_rmsnorm_args* a, cudaStream_t s) {
  const unsigned grid = (unsigned)((a->rows + kWarps - 1) / kWarps);
  if (a->w_fp32) rmsnorm_kernel<MAXV, true><<<grid, 32 * kWarps, 0, s>>>(*a);
  else rmsnorm_kernel<MAXV, false><<<grid, 32 * kWarps, 0, s>>>(*a);
}

}  // namespace

extern "C" int bolt3_rmsnorm(const bolt3_rmsnorm_args* a, void* stream) {
  const b3::TraceRange trace_range("bolt3_rmsnorm");
  if (!a || !a->x || !a->w || !a->y) return BOLT3_ERR_ARG;
  if (a->rows < 0 || a->D <= 0 || a->D % 8 || a->D > 32 * 8 * 16 || a->x_stride < a->D) return BOLT3_ERR_SHAPE;
  if (a->rows == 0) return BOLT3_OK;
  if ((uintptr_t)a->x % 16 || (uintptr_t)a->y % 16 || (uintptr_t)a->w % 16 || a->x_stride % 8) return BOLT3_ERR_ALIGN;
  if ((a->r == nullptr) != (a->sum == nullptr)) return BOLT3_ERR_ARG;
  if (a->r && ((uintptr_t)a->r % 16 || (uintptr_t)a->sum % 16)) return BOLT3_ERR_ALIGN;
  if (a->rows / kWarps >= 0x7fffffff) return BOLT3_ERR_SHAPE;
  cudaStream_t s = (cudaStream_t)stream;
  const int nv = a->D / 8;
  // rows of 1024 values and more, too few to fill the GPU with a warp each: a block per row
  if (nv >= 128 && a->rows <= 4096) {
    const unsigned grid = (unsigned)a->rows;
    if (nv <= 256) {
      if (a->w_fp32) rmsnorm_row_kernel<1, true><<<grid, 256, 0, s>>>(*a);
      else rmsnorm_row_kernel<1, false><<<grid, 256, 0, s>>>(*a);
    } else {
      if (a->w_fp32) rmsnorm_row_kernel<2, true><<<grid, 256, 0, s>>>(*a);
      else rmsnorm_row_kernel<2, false><<<grid, 256, 0, s>>>(*a);
    }
    return cudaGetLastError() == cudaSuccess ? BOLT3_OK : BOLT3_ERR_CUDA;
  }
  if (nv <= 32) launch_v<1>(a, s);
  else if (nv <= 64) launch_v<2>(a, s);
  else if (nv <= 128) launch_v<4>(a, s);
  else if (nv <= 256) launch_v<8>(a, s);
  else launch_v<16>(a, s);
  return cudaGetLastError() == cudaSuccess ? BOLT3_OK : BOLT3_ERR_CUDA;
}
