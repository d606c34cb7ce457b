// One-token decode step of a softmax anchor layer (the hybrid model's full-attention layers):
// append the new key/value to the layer's KV cache, then causal GQA attention of the G query heads
// of each KV head over every cached key.
//
// Replaces the anchor branch of Bolt3Decoder.step for one new token (vsa_lm/config/bolt3.py:426-445:
// StaticKV.append, then scaled_dot_product_attention over the cache with enable_gqa). The softmax
// is exact (a running maximum and sum over key blocks, fp32 throughout); the output is rounded to
// bf16 once.
//
// HBM-bound: each (sequence, KV head) streams its n cached keys and values once. One CTA of 256
// threads per (sequence, KV head) walks the cache in blocks of 256 keys: a thread per key for the
// G scores (its whole key row requested at once), the block's probabilities to shared memory, then
// the P.V product with each thread owning eight value columns of all G heads for a sixteenth of the
// block's keys (HD = 128), every value row read as 16-byte pieces that a warp's lanes share out.
//
// The cache length comes from the launch (n) or, for a step replayed from a CUDA graph, from the
// device (n + *pos_dev - pos_ref), like the Bolt-3 kernels' device step position.
#include "../../include/bolt3.h"
#include "common.cuh"

namespace {

using namespace b3;

constexpr int kThreads = 256;
constexpr int kBlockKeys = 256;  // one key per thread per block
constexpr int kMaxG = 8;

template <int HD, int G>
struct AnchorSmem {
  static constexpr int CG = HD / 8;             // 8-column groups of a value row
  static constexpr int NKG = kThreads / CG;     // key groups of the P.V product
  static constexpr size_t floats = G * HD + G * kBlockKeys + 8 * G + NKG * G * HD;
};

template <int HD, int G>
__global__ void __launch_bounds__(kThreads) anchor_decode_kernel(const bolt3_anchor_args a) {
  using L_ = AnchorSmem<HD, G>;
  constexpr int CG = L_::CG, NKG = L_::NKG;
  constexpr float kLog2e = 1.4426950408889634f;
  extern __shared__ __align__(16) float smem[];
  float* qs = smem;                         // [G][HD] query rows (fp32)
  float* ps = qs + G * HD;                  // [G][kBlockKeys] probabilities of the block
  float* red = ps + G * kBlockKeys;         // [8 warps][G] reductions
  float* op = red + 8 * G;                  // [NKG][G][HD] partial outputs

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x;                 // (sequence, KV head)
  const int b = c / a.HKV, kvh = c % a.HKV;
  int64_t n = a.n;
  if (a.pos_dev != nullptr) {
    const int64_t d = *a.pos_dev - a.pos_ref;
    if (d < 0 || d >= a.pos_span) {
      if (tid == 0 && a.status) atomicOr(a.status, 8);
      return;
    }
    n += d;
  }
  const int64_t L = n + 1;                  // keys after the append
  bf16* kc = reinterpret_cast<bf16*>(a.k_cache) + (int64_t)c * a.cap * HD;
  bf16* vc = reinterpret_cast<bf16*>(a.v_cache) + (int64_t)c * a.cap * HD;

  // append the new key and value at position n
  if (tid < HD / 8) {
    const uint4* kn = reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(a.k_new) + (int64_t)c * HD);
    const uint4* vn = reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(a.v_new) + (int64_t)c * HD);
    reinterpret_cast<uint4*>(kc + n * HD)[tid] = kn[tid];
    reinterpret_cast<uint4*>(vc + n * HD)[tid] = vn[tid];
  }
  // the query rows of the G heads that read this KV head
  const bf16* q = reinterpret_cast<const bf16*>(a.q) + ((int64_t)b * a.H + (int64_t)kvh * G) * HD;
  for (int i = tid; i < G * HD; i += kThreads) qs[i] = bf2f(q[i]);
  __syncthreads();  // the appended row and the query rows are visible to the whole block

  float m_run[G], l_run[G], acc[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m_run[g] = neg_inf();
    l_run[g] = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[g][e] = 0.f;
  }
  const int cg = tid % CG, kg = tid / CG;
  for (int64_t k0 = 0; k0 < L; k0 += kBlockKeys) {
    // -- scores: thread tid takes key k0 + tid; its whole key row is requested at once
    const int64_t j = k0 + tid;
    float s[G];
#pragma unroll
    for (int g = 0; g < G; ++g) s[g] = 0.f;
    if (j < L) {
      uint4 kr[HD / 8];
#pragma unroll
      for (int ch = 0; ch < HD / 8; ++ch) kr[ch] = reinterpret_cast<const uint4*>(kc + j * HD)[ch];
#pragma unroll
      for (int ch = 0; ch < HD / 8; ++ch) {
        const uint32_t w[4] = {kr[ch].x, kr[ch].y, kr[ch].z, kr[ch].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 kf = unpack_bf16(w[e]);
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const float2 qf = *reinterpret_cast<const float2*>(&qs[g * HD + ch * 8 + 2 * e]);
            s[g] = fmaf(qf.x, kf.x, s[g]);
            s[g] = fmaf(qf.y, kf.y, s[g]);
          }
        }
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      s[g] = j < L ? __fmul_rn(s[g], a.scale) : neg_inf();
      const float m = warp_max(s[g]);
      if (lane == 0) red[warp * G + g] = m;
    }
    __syncthreads();
    float alpha[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float bm = neg_inf();
#pragma unroll
      for (int w = 0; w < 8; ++w) bm = fmaxf(bm, red[w * G + g]);
      const float m_new = fmaxf(m_run[g], bm);   // finite: every block holds at least one key
      alpha[g] = exp2f((m_run[g] - m_new) * kLog2e);
      const float p = j < L ? exp2f((s[g] - m_new) * kLog2e) : 0.f;
      ps[g * kBlockKeys + tid] = p;
      m_run[g] = m_new;
      s[g] = p;
    }
    __syncthreads();  // red is reused for the sums; ps is complete
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float sm = warp_sum(s[g]);
      if (lane == 0) red[warp * G + g] = sm;
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float bs = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) bs += red[w * G + g];
      l_run[g] = fmaf(l_run[g], alpha[g], bs);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[g][e] *= alpha[g];
    }
    // -- P.V: thread (8-column group cg, key group kg) over keys kg, kg + NKG, ... of the block, a
    // 16-byte load of the value row per key (a warp reads whole rows)
    const int nb = L - k0 < kBlockKeys ? (int)(L - k0) : kBlockKeys;
    constexpr int KPT = kBlockKeys / NKG;       // keys per thread per block
    uint4 vr[KPT];
#pragma unroll
    for (int i = 0; i < KPT; ++i) {
      const int kk = kg + i * NKG;
      vr[i] = kk < nb ? reinterpret_cast<const uint4*>(vc + (k0 + kk) * HD)[cg] : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int i = 0; i < KPT; ++i) {
      const int kk = kg + i * NKG;
      const uint32_t w[4] = {vr[i].x, vr[i].y, vr[i].z, vr[i].w};
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float p = kk < nb ? ps[g * kBlockKeys + kk] : 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 vf = unpack_bf16(w[e]);
          acc[g][2 * e] = fmaf(p, vf.x, acc[g][2 * e]);
          acc[g][2 * e + 1] = fmaf(p, vf.y, acc[g][2 * e + 1]);
        }
      }
    }
    __syncthreads();  // ps and red are rewritten by the next block
  }
  // -- the key groups' partial outputs summed, normalised and rounded once
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float4* dst = reinterpret_cast<float4*>(&op[(kg * G + g) * HD + cg * 8]);
    dst[0] = make_float4(acc[g][0], acc[g][1], acc[g][2], acc[g][3]);
    dst[1] = make_float4(acc[g][4], acc[g][5], acc[g][6], acc[g][7]);
  }
  __syncthreads();
  bf16* y = reinterpret_cast<bf16*>(a.y) + ((int64_t)b * a.H + (int64_t)kvh * G) * HD;
  for (int i = tid; i < G * HD; i += kThreads) {
    const int g = i / HD, e = i % HD;
    float o = 0.f;
    for (int k = 0; k < NKG; ++k) o += op[(k * G + g) * HD + e];
    float lg = 0.f;
#pragma unroll
    for (int gg = 0; gg < G; ++gg)
      if (gg == g) lg = l_run[gg];
    y[i] = __float2bfloat16_rn(o / lg);
  }
}

template <int HD, int G>
int launch_g(const bolt3_anchor_args* a, cudaStream_t s) {
  const size_t smem = sizeof(float) * AnchorSmem<HD, G>::floats;
  auto kern = anchor_decode_kernel<HD, G>;
  if (smem > 48 * 1024 && cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return BOLT3_ERR_CUDA;
  kern<<<(unsigned)(a->B * a->HKV), kThreads, smem, s>>>(*a);
  return cudaGetLastError() == cudaSuccess ? BOLT3_OK : BOLT3_ERR_CUDA;
}

template <int HD>
int launch_hd(const bolt3_anchor_args* a, cudaStream_t s) {
  switch (a->H / a->HKV) {
    case 1: return launch_g<HD, 1>(a, s);
    case 2: return launch_g<HD, 2>(a, s);
    case 4: return launch_g<HD, 4>(a, s);
    case 8: return launch_g<HD, 8>(a, s);
    default: return BOLT3_ERR_SHAPE;
  }
}

}  // namespace

extern "C" int bolt3_anchor_decode(const bolt3_anchor_args* a, void* stream) {
  if (!a || !a->q || !a->k_new || !a->v_new || !a->k_cache || !a->v_cache || !a->y) return BOLT3_ERR_ARG;
  if (a->B <= 0 || a->HKV <= 0 || a->H <= 0 || a->H % a->HKV || a->H / a->HKV > kMaxG) return BOLT3_ERR_SHAPE;
  if ((int64_t)a->B * a->HKV > 0x7fffffff) return BOLT3_ERR_SHAPE;
  if (a->pos_dev != nullptr && a->pos_span < 1) return BOLT3_ERR_ARG;
  const int64_t dmax = a->pos_dev != nullptr ? a->pos_span - 1 : 0;
  if (a->n < 0 || a->n + dmax + 1 > a->cap) return BOLT3_ERR_CAPACITY;
  const uintptr_t al = (uintptr_t)a->q | (uintptr_t)a->k_new | (uintptr_t)a->v_new | (uintptr_t)a->k_cache |
                       (uintptr_t)a->v_cache;
  if (al & 15) return BOLT3_ERR_ALIGN;
  cudaStream_t s = (cudaStream_t)stream;
  if (a->HD == 128) return launch_hd<128>(a, s);
  if (a->HD == 64) return launch_hd<64>(a, s);
  return BOLT3_ERR_SHAPE;
}
