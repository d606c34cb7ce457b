// Phase A epilogue: from the fused projection output to head-major q/k/v with RoPE and gates.
//
// Mirrors Bolt3Attn.head_qkv (vsa_lm/config/bolt3.py:59-66: per-head LlamaRMSNorm when qk_norm,
// surgery.py:43-53), LlamaRoPE (surgery.py:80-93) in the storage dtype (cos/sin cast to bf16, every
// product and the sum rounded to bf16), beta = sigmoid(beta_proj x) and eta = tanh(eta_proj x)
// (bolt3.py:198-199) computed from the bf16 logits and rounded to bf16.
//
// HBM-bound elementwise work: one CTA per token, one warp per head row; a lane owns the element
// pairs (i, i + HD/2) that rotate-half RoPE couples, so no cross-lane exchange is needed.
#include "../../include/bolt3.h"
#include "common.cuh"

namespace {

using namespace b3;

template <int HD>
__global__ void __launch_bounds__(256) prep_kernel(bolt3_prep_args a) {
  constexpr int E = HD / 64;  // elements per lane in each half
  const int tok = blockIdx.x;           // b * T + t
  const int b = tok / a.T, t = tok % a.T;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bf16* row = reinterpret_cast<const bf16*>(a.proj) + (int64_t)tok * a.ld;
  const float pos = (float)(a.pos0 + t);

  // cos/sin of this lane's frequencies (shared by every head of the token)
  float cs[E], sn[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const float ang = __fmul_rn(pos, a.inv_freq[lane * E + e]);
    float s, c;
    sincosf(ang, &s, &c);
    cs[e] = rbf(c);
    sn[e] = rbf(s);
  }

  const int n_rows = a.H + 2 * a.HKV;
  for (int r = warp; r < n_rows; r += 8) {
    const bf16* src;
    int kind, head;  // 0 = q, 1 = k, 2 = v
    if (r < a.H) { kind = 0; head = r; src = row + (int64_t)head * HD; }
    else if (r < a.H + a.HKV) { kind = 1; head = r - a.H; src = row + (int64_t)(a.H + head) * HD; }
    else { kind = 2; head = r - a.H - a.HKV; src = row + (int64_t)(a.H + a.HKV + head) * HD; }
    float x0[E], x1[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
      x0[e] = bf2f(src[lane * E + e]);
      x1[e] = bf2f(src[HD / 2 + lane * E + e]);
    }
    const int nh = kind == 0 ? a.H : a.HKV;
    const int64_t hs = kind == 0 ? a.q_head_stride : a.k_head_stride;
    const int64_t to = kind == 0 ? a.q_t_off : a.k_t_off;
    const int64_t off = (((int64_t)b * nh + head) * hs + to + t) * HD;
    if (kind == 2) {
      bf16* dst = reinterpret_cast<bf16*>(a.v) + off;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        dst[lane * E + e] = __float2bfloat16_rn(x0[e]);
        dst[HD / 2 + lane * E + e] = __float2bfloat16_rn(x1[e]);
      }
      continue;
    }
    const float* nw = kind == 0 ? a.q_norm_w : a.k_norm_w;
    float l2 = 0.f;  // |q_raw| of the stored (bf16) row, for the M_res read-out
    if (nw != nullptr) {
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) ss += x0[e] * x0[e] + x1[e] * x1[e];
      ss = warp_sum(ss);
      const float r_ = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, (float)HD), a.eps));
#pragma unroll
      for (int e = 0; e < E; ++e) {
        x0[e] = rbf(__fmul_rn(__fmul_rn(x0[e], r_), nw[lane * E + e]));
        x1[e] = rbf(__fmul_rn(__fmul_rn(x1[e], r_), nw[HD / 2 + lane * E + e]));
      }
    }
    if (kind == 0 && a.q_l2 != nullptr) {
#pragma unroll
      for (int e = 0; e < E; ++e) l2 = fmaf(rbf(x0[e]), rbf(x0[e]), fmaf(rbf(x1[e]), rbf(x1[e]), l2));
      l2 = warp_sum(l2);
      if (lane == 0) a.q_l2[((int64_t)b * a.H + head) * a.eta_head_stride + a.eta_t_off + t] = sqrtf(l2);
    }
    bf16* draw = reinterpret_cast<bf16*>(kind == 0 ? a.q_raw : a.k_raw) + off;
    bf16* drope = reinterpret_cast<bf16*>(kind == 0 ? a.q_rope : a.k_rope) + off;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      draw[lane * E + e] = __float2bfloat16_rn(x0[e]);
      draw[HD / 2 + lane * E + e] = __float2bfloat16_rn(x1[e]);
      // rotate_half: first half pairs with -x1, second half with x0
      const float r0 = rbf(__fadd_rn(rbf(__fmul_rn(x0[e], cs[e])), rbf(__fmul_rn(-x1[e], sn[e]))));
      const float r1 = rbf(__fadd_rn(rbf(__fmul_rn(x1[e], cs[e])), rbf(__fmul_rn(x0[e], sn[e]))));
      drope[lane * E + e] = __float2bfloat16_rn(r0);
      drope[HD / 2 + lane * E + e] = __float2bfloat16_rn(r1);
    }
  }

  // gates: HKV beta logits then H eta logits
  const bf16* gl = row + (int64_t)(a.H + 2 * a.HKV) * HD;
  for (int i = threadIdx.x; i < a.HKV + a.H; i += blockDim.x) {
    const float z = bf2f(gl[i]);
    if (i < a.HKV) {
      const float s = rbf(1.0f / (1.0f + expf(-z)));
      a.beta[((int64_t)b * a.HKV + i) * a.beta_head_stride + a.beta_t_off + t] = s;
    } else {
      const int h = i - a.HKV;
      a.eta[((int64_t)b * a.H + h) * a.eta_head_stride + a.eta_t_off + t] = rbf(tanhf(z));
    }
  }
}

}  // namespace

extern "C" int bolt3_prep(const bolt3_prep_args* a, void* stream) {
  if (!a || !a->proj || !a->inv_freq || !a->q_raw || !a->q_rope || !a->k_raw || !a->k_rope || !a->v ||
      !a->beta || !a->eta)
    return BOLT3_ERR_ARG;
  if (a->B <= 0 || a->T <= 0 || a->H <= 0 || a->HKV <= 0 || a->H % a->HKV) return BOLT3_ERR_SHAPE;
  if (a->ld < (int64_t)(a->H + 2 * a->HKV) * a->HD + a->HKV + a->H) return BOLT3_ERR_CAPACITY;
  if (a->q_head_stride < a->q_t_off + a->T || a->k_head_stride < a->k_t_off + a->T ||
      a->beta_head_stride < a->beta_t_off + a->T || a->eta_head_stride < a->eta_t_off + a->T)
    return BOLT3_ERR_CAPACITY;
  const int64_t n_tok = (int64_t)a->B * a->T;
  if (n_tok > 0x7fffffff) return BOLT3_ERR_SHAPE;
  cudaStream_t s = (cudaStream_t)stream;
  if (a->HD == 128) prep_kernel<128><<<(unsigned)n_tok, 256, 0, s>>>(*a);
  else if (a->HD == 64) prep_kernel<64><<<(unsigned)n_tok, 256, 0, s>>>(*a);
  else return BOLT3_ERR_SHAPE;
  return cudaGetLastError() == cudaSuccess ? BOLT3_OK : BOLT3_ERR_CUDA;
}
