// Shared device helpers for the Bolt-3 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

typedef __nv_bfloat16 bf16;

#define B3_DEV __device__ __forceinline__

namespace b3 {

B3_DEV float neg_inf() { return __int_as_float(0xff800000); }

// ---- bf16 rounding helpers (round-to-nearest-even, as torch's float->bfloat16 cast)
B3_DEV float rbf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
B3_DEV float bf2f(bf16 x) { return __bfloat162float(x); }
B3_DEV uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
B3_DEV float2 unpack_bf16(uint32_t u) {
  return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}
// Two roundings for the price of one conversion instruction: `packed` gets the bf16 pair, the
// return value the same two values as floats.
B3_DEV float2 rbf2(float lo, float hi, uint32_t& packed) {
  packed = pack_bf16(lo, hi);
  return unpack_bf16(packed);
}

// ---- packed bf16 pair arithmetic, each result rounded to nearest even on its own (no contraction of
// a multiply into a following add)
B3_DEV uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;\n" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
B3_DEV uint32_t add_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;\n" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
B3_DEV uint32_t neg_bf16x2(uint32_t a) { return a ^ 0x80008000u; }

// ---- warp reductions
B3_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
B3_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// reduce over the 4 lanes of an mma quad (lanes 4g..4g+3)
B3_DEV float quad_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  return v;
}
B3_DEV float quad_max(float v) {
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
  return v;
}

// ---- swizzled [128][COLS] bf16 tiles in shared memory, in the 128-byte-swizzle layout the tensor
// cores read: COLS / 64 blocks of [128 rows][64 columns]; within a 128-byte row the 16-byte chunk
// index is XOR-ed with (row & 7), so ldmatrix reads of 8 consecutive rows hit distinct banks.
template <int COLS>
B3_DEV int swz(int r, int c) {
  static_assert(COLS % 64 == 0, "swizzled tiles are made of 64-column blocks");
  return (c >> 6) * (128 * 64) + r * 64 + (((((c >> 3) & 7) ^ (r & 7))) << 3) + (c & 7);
}

// ---- legacy warp-level tensor-core MMA (m16n8k16, bf16 in, fp32 accumulate)
B3_DEV void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

B3_DEV void ldsm_x4(uint32_t (&r)[4], const void* p) {
  uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}
B3_DEV void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}

// ---- cp.async (16-byte, L2-cached) with zero fill when `valid` is false
B3_DEV void cp_async16(void* smem, const void* gmem, bool valid) {
  uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(n));
}
B3_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
B3_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// ---- order-preserving float <-> uint32 key
B3_DEV uint32_t fkey(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// ---- programmatic dependent launch. A kernel launched with programmatic stream serialisation
// may start while the kernel before it on the stream is still running; it must call
// grid_dep_wait() before it reads anything that kernel writes (or writes anything it reads).
// grid_dep_wait() returns once every earlier grid of the stream has completed and its writes are
// visible; in a kernel launched without the attribute it returns at once. grid_dep_launch() lets
// the next such kernel begin launching once every block of this grid has called it or exited.
B3_DEV void grid_dep_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
B3_DEV void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

// <<<grid, block, smem, s>>> with programmatic stream serialisation: the kernel's blocks may be
// scheduled before the previous kernel on `s` has finished (it calls grid_dep_wait() first)
template <typename... P, typename... A>
inline cudaError_t launch_overlapped(void (*kern)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                     A&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<A>(args)...);
}

}  // namespace b3
