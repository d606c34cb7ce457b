// One-token decode step of a softmax anchor layer (the hybrid model's full-attention layers):
// append the new key/value to the layer's KV cache, then causal GQA attention of the G query heads
// of each KV head over every cached key.
//
// Replaces the anchor branch of Bolt3Decoder.step for one new token (vsa_lm/config/bolt3.py:426-445:
// StaticKV.append, then scaled_dot_product_attention over the cache with enable_gqa). Scores, the
// running maxima and sums and the output accumulate in fp32; the output is rounded to bf16 once.
//
// HBM-bound: each (sequence, KV head) streams its n cached keys and values once. One CTA of three
// warps per (sequence, KV head) walks the cache in blocks of 48 keys, double-buffered in shared memory
// by cp.async (16-byte pieces, chunk index XOR-swizzled by row so that ldmatrix reads are free of bank
// conflicts); 48 KB of stages per CTA lets four CTAs share an SM, so the 512 CTAs of configs[3] run
// in one wave with up to 192 KB per SM in flight. Each warp takes 16 keys of every block: the scores
// S = Q.K^T and the product P.V are mma.sync m16n8k16 tiles (the G query rows padded to 16), P is
// rounded to bf16 for the product as the flash attention of the reference's SDPA does, and every
// warp keeps a running maximum, sum and output of its own keys; the three are merged once at the end.
//
// The cache length comes from the launch (n) or, for a step replayed from a CUDA graph, from the
// device (n + *pos_dev - pos_ref), like the Bolt-3 kernels' device step position.
#include "../../include/bolt3.h"
#include "common.cuh"
#include "trace.h"

namespace {

using namespace b3;

constexpr int kWarps = 3;
constexpr int kThreads = 32 * kWarps;
constexpr int kKeysPerWarp = 16;
constexpr int kBlockKeys = kWarps * kKeysPerWarp;   // 48
constexpr int kMaxG = 8;

template <int HD>
struct AnchorSmem {
  static constexpr int kStage = kBlockKeys * HD * 2;      // bytes of one K (or V) block
  // two stages of K and V (the final merge reuses them for the warps' partial outputs), then the RoPE
  // cos / sin table
  static constexpr size_t stages = 2 * 2 * (size_t)kStage;
  static constexpr size_t bytes = stages + HD / 2 * 4;
  static_assert((size_t)kWarps * kMaxG * HD * 4 + 2 * kWarps * kMaxG * 4 <= stages, "merge area fits the stages");
};

// byte offset of 16-byte chunk c of row r in a [rows][HD] bf16 block, chunk index XOR-swizzled by row
template <int HD>
B3_DEV uint32_t sw_off(int r, int c) { return (uint32_t)(r * HD * 2 + ((c ^ (r & 7)) << 4)); }

template <int HD, int G>
__global__ void __launch_bounds__(kThreads) anchor_decode_kernel(const bolt3_anchor_args a) {
  constexpr int CPR = HD / 8;                    // 16-byte chunks per row
  constexpr int KS = HD / 16;                    // k16 steps of a dot product
  constexpr int NT = HD / 8;                     // n8 tiles of an output row
  constexpr uint32_t kStage = AnchorSmem<HD>::kStage;
  constexpr float kLog2e = 1.4426950408889634f;
  extern __shared__ __align__(128) unsigned char smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int grp = lane >> 2, tig = lane & 3;
  const int c = blockIdx.x;                      // (sequence, KV head)
  const int b = c / a.HKV, kvh = c % a.HKV;
  int64_t n = a.n, d = 0;
  if (a.pos_dev != nullptr) {
    d = *a.pos_dev - a.pos_ref;
    if (d < 0 || d >= a.pos_span) {
      if (tid == 0 && a.status) atomicOr(a.status, 8);
      return;
    }
    n += d;
  }
  const int64_t L = n + 1;                       // keys after the append
  bf16* kc = reinterpret_cast<bf16*>(a.k_cache) + (int64_t)c * a.cap * HD;
  bf16* vc = reinterpret_cast<bf16*>(a.v_cache) + (int64_t)c * a.cap * HD;
  const bool rope = a.inv_freq != nullptr;

  // bf16 cos / sin of the HD/2 frequencies at the token's position, as pairs of adjacent
  // frequencies (the operands of the packed rotations below), after the stages
  uint32_t* trig = reinterpret_cast<uint32_t*>(smem + AnchorSmem<HD>::stages);   // [HD/4] cos, [HD/4] sin
  if (rope) {
    if (tid < HD / 4) {
      const float pos = (float)(a.pos0 + d);
      float s0, c0, s1, c1;
      sincosf(__fmul_rn(pos, a.inv_freq[2 * tid]), &s0, &c0);
      sincosf(__fmul_rn(pos, a.inv_freq[2 * tid + 1]), &s1, &c1);
      trig[tid] = pack_bf16(c0, c1);
      trig[HD / 4 + tid] = pack_bf16(s0, s1);
    }
    __syncthreads();
  }
  // rotate-half RoPE of the packed bf16 pairs x1 (dims f, f+1 of the first half) and x2 (their partners
  // HD/2 later) with the pair's cos / sin words: x1' = x1 c - x2 s, x2' = x2 c + x1 s, every product and
  // sum rounded to bf16 (the same single roundings as LlamaRoPE's bf16 tensor arithmetic)
  auto rot = [&](uint32_t& x1, uint32_t& x2, int fpair) {
    const uint32_t cw = trig[fpair], sw = trig[HD / 4 + fpair];
    const uint32_t n1 = add_bf16x2(mul_bf16x2(x1, cw), neg_bf16x2(mul_bf16x2(x2, sw)));
    const uint32_t n2 = add_bf16x2(mul_bf16x2(x2, cw), mul_bf16x2(x1, sw));
    x1 = n1;
    x2 = n2;
  };

  // append the new key (rotated) and value at position n
  if (tid < CPR / 2) {
    const uint4* kn = reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(a.k_new) + (int64_t)c * HD);
    const uint4* vn = reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(a.v_new) + (int64_t)c * HD);
    uint4 k1 = kn[tid], k2 = kn[tid + CPR / 2];     // dims 8 tid .. 8 tid + 7 and their partners
    if (rope) {
      rot(k1.x, k2.x, 4 * tid + 0);
      rot(k1.y, k2.y, 4 * tid + 1);
      rot(k1.z, k2.z, 4 * tid + 2);
      rot(k1.w, k2.w, 4 * tid + 3);
    }
    reinterpret_cast<uint4*>(kc + n * HD)[tid] = k1;
    reinterpret_cast<uint4*>(kc + n * HD)[tid + CPR / 2] = k2;
    reinterpret_cast<uint4*>(vc + n * HD)[tid] = vn[tid];
    reinterpret_cast<uint4*>(vc + n * HD)[tid + CPR / 2] = vn[tid + CPR / 2];
  }
  __threadfence_block();
  __syncthreads();  // the appended row is visible to the block's copies below

  const int64_t n_blk = (L + kBlockKeys - 1) / kBlockKeys;
  auto issue = [&](int64_t blk) {
    unsigned char* ks = smem + (blk & 1) * 2 * kStage;
    unsigned char* vs = ks + kStage;
    for (int i = tid; i < kBlockKeys * CPR; i += kThreads) {
      const int r = i / CPR, ch = i % CPR;
      const int64_t key = blk * kBlockKeys + r;
      const bool ok = key < L;
      const int64_t src = (ok ? key : 0) * HD + ch * 8;
      cp_async16(ks + sw_off<HD>(r, ch), kc + src, ok);
      cp_async16(vs + sw_off<HD>(r, ch), vc + src, ok);
    }
    cp_async_commit();
  };
  issue(0);
  if (n_blk > 1) issue(1);

  // the query rows as A fragments (rows 0..G-1 real, the rest zero): a0 / a2 of every k16 step
  uint32_t qa[KS][2];
  {
    const bf16* q = reinterpret_cast<const bf16*>(a.q) + ((int64_t)b * a.H + (int64_t)kvh * G) * HD;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      if (grp < G) {
        qa[ks][0] = *reinterpret_cast<const uint32_t*>(q + grp * HD + ks * 16 + tig * 2);
        qa[ks][1] = *reinterpret_cast<const uint32_t*>(q + grp * HD + ks * 16 + 8 + tig * 2);
      } else {
        qa[ks][0] = qa[ks][1] = 0u;
      }
    }
    // RoPE: the partner of a fragment's dims (ks, offset) is (ks + KS/2, same offset), held by the
    // same thread; frequency pair (16 ks + 2 tig) / 2 for a0, 8 more for a2
    if (rope) {
#pragma unroll
      for (int ks = 0; ks < KS / 2; ++ks) {
        rot(qa[ks][0], qa[ks + KS / 2][0], 8 * ks + tig);
        rot(qa[ks][1], qa[ks + KS / 2][1], 8 * ks + 4 + tig);
      }
    }
  }

  const float sl2 = a.scale * kLog2e;             // scores in the log2 domain
  float m_run = neg_inf(), l_run = 0.f;           // row grp of this warp's keys
  float o[NT][4];
#pragma unroll
  for (int t = 0; t < NT; ++t) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.f;

  for (int64_t blk = 0; blk < n_blk; ++blk) {
    if (blk + 1 < n_blk) cp_async_wait<1>();
    else cp_async_wait<0>();
    __syncthreads();  // block blk has landed for every thread
    const unsigned char* ks_ = smem + (blk & 1) * 2 * kStage;
    const unsigned char* vs_ = ks_ + kStage;
    const int r0 = warp * kKeysPerWarp;           // this warp's 16 keys of the block
    // -- S = Q K^T: two n8 tiles (keys r0..r0+7, r0+8..r0+15)
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kst = 0; kst < KS; ++kst) {
      uint32_t bfr[4];
      const int m = lane >> 3;                    // matrix: (key half, dim half)
      const int row = r0 + ((m >> 1) << 3) + (lane & 7);
      const int ch = kst * 2 + (m & 1);
      ldsm_x4(bfr, ks_ + sw_off<HD>(row, ch));
      const uint32_t afr[4] = {qa[kst][0], 0u, qa[kst][1], 0u};
      mma16816(sc[0], afr, bfr[0], bfr[1]);
      mma16816(sc[1], afr, bfr[2], bfr[3]);
    }
    // -- running softmax of row grp over this warp's keys (the padding rows grp + 8 are not used)
    const int64_t kbase = blk * kBlockKeys + r0;
    float p[2][2];
    float bm = neg_inf();
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int64_t key = kbase + t * 8 + tig * 2 + e;
        p[t][e] = key < L ? __fmul_rn(sc[t][e], sl2) : neg_inf();
        bm = fmaxf(bm, p[t][e]);
      }
    bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 1));
    bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 2));
    const float m_new = fmaxf(m_run, bm);
    const float mref = m_new == neg_inf() ? 0.f : m_new;   // a warp whose keys are all past L so far
    const float alpha = exp2f(m_run - mref);
    float rs = 0.f;
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        p[t][e] = exp2f(p[t][e] - mref);
        rs += p[t][e];
      }
    rs += __shfl_xor_sync(0xffffffffu, rs, 1);
    rs += __shfl_xor_sync(0xffffffffu, rs, 2);
    l_run = fmaf(l_run, alpha, rs);
    m_run = m_new;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      o[t][0] *= alpha;
      o[t][1] *= alpha;
    }
    // -- O += P V: P (bf16) as the A fragment of a k16 step over the warp's 16 keys
    const uint32_t pa[4] = {pack_bf16(p[0][0], p[0][1]), 0u, pack_bf16(p[1][0], p[1][1]), 0u};
#pragma unroll
    for (int t2 = 0; t2 < NT / 2; ++t2) {
      uint32_t bfr[4];
      const int m = lane >> 3;                    // matrix: (key half, dim tile)
      const int row = r0 + ((m & 1) << 3) + (lane & 7);
      const int ch = t2 * 2 + (m >> 1);
      ldsm_x4_t(bfr, vs_ + sw_off<HD>(row, ch));
      mma16816(o[2 * t2], pa, bfr[0], bfr[1]);
      mma16816(o[2 * t2 + 1], pa, bfr[2], bfr[3]);
    }
    __syncthreads();  // every warp is done with stage blk & 1 before it is refilled
    if (blk + 2 < n_blk) issue(blk + 2);
  }

  // -- merge the warps' running states: m = max m_w, O = sum O_w 2^(m_w - m), l likewise
  float* op = reinterpret_cast<float*>(smem);                 // [kWarps][kMaxG][HD]
  float* ml = op + kWarps * kMaxG * HD;                       // [kWarps][kMaxG] maxima, then sums
  if (grp < G) {
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      op[(warp * kMaxG + grp) * HD + t * 8 + tig * 2] = o[t][0];
      op[(warp * kMaxG + grp) * HD + t * 8 + tig * 2 + 1] = o[t][1];
    }
    if (tig == 0) {
      ml[warp * kMaxG + grp] = m_run;
      ml[kWarps * kMaxG + warp * kMaxG + grp] = l_run;
    }
  }
  __syncthreads();
  bf16* y = reinterpret_cast<bf16*>(a.y) + ((int64_t)b * a.H + (int64_t)kvh * G) * HD;
  for (int i = tid; i < G * HD; i += kThreads) {
    const int g = i / HD, e = i % HD;
    float m = neg_inf();
#pragma unroll
    for (int w = 0; w < kWarps; ++w) m = fmaxf(m, ml[w * kMaxG + g]);
    float acc = 0.f, l = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float mw = ml[w * kMaxG + g];
      const float f = mw == neg_inf() ? 0.f : exp2f(mw - m);
      acc = fmaf(op[(w * kMaxG + g) * HD + e], f, acc);
      l = fmaf(ml[kWarps * kMaxG + w * kMaxG + g], f, l);
    }
    y[i] = __float2bfloat16_rn(acc / l);
  }
}

template <int HD, int G>
int launch_g(const bolt3_anchor_args* a, cudaStream_t s) {
  const size_t smem = AnchorSmem<HD>::bytes;
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
  const b3::TraceRange trace_range("bolt3_anchor_decode");
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
