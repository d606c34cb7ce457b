// Decode-step attention: the same three-field softmax + M_res read-out as attend.cu, for steps that
// bring only a few query rows per chain (G heads x t <= 16 tokens; a one-token step has G = 4 rows).
//
// Such a step is bound by streaming the chain's state from HBM (attractor keys and values, the
// local window, fp32 M_res: about 236 KB per chain at HD = 128) while its arithmetic is tiny. One
// warp owns one chain, with no block-wide barrier, so a CTA of WPC warps holds WPC independent
// chains and every SM interleaves many of them:
//   scores  a lane per key (32 keys per round), the key row read with sixteen 16-byte loads in
//           flight, dot products against the query rows in shared memory (fp32 of the bf16 values,
//           so the products are exact);
//   softmax warp reductions per row, p = bf16(exp(s - max) / sum) as the reference rounds it;
//   P@V     a lane per HD/32 output columns, each value row read by the whole warp at once, 16
//           rows per batch with the next batch in flight;
//   M_res   a lane per HD/32 columns e sums q_raw[d] * M[d][e] over d directly in fp32.
// Reference: vsa_lm/config/bolt3.py:365-402 (decoder attention) with the forward's chunk body
// :219-256 for the shared math. Keys: [4 sinks][S attractors: RoPE'd, + kappa*log(max(mass, 1)),
// -inf if inactive][previous chunk][current chunk, causal: key j visible to new token i iff
// j <= len_before + i].
#include "../../include/bolt3.h"
#include "common.cuh"

#include <type_traits>

namespace b3dec {

using namespace b3;

constexpr int S = 128;
constexpr int kMaxKeys = 4 + S + 256;
constexpr int kLP = (kMaxKeys + 3) & ~3;  // score row stride

// warps (= chains) per CTA for NRM query rows: shared memory per warp is 2 * NRM * HD + NRM * kLP floats
template <int NRM>
__host__ __device__ constexpr int warps_per_cta() { return NRM <= 4 ? 8 : (NRM <= 8 ? 4 : 2); }

template <int HD, int NRM>
__global__ void __launch_bounds__(32 * warps_per_cta<NRM>()) attend_decode_kernel(const bolt3_attend_args a) {
  constexpr int WPC = warps_per_cta<NRM>();
  constexpr int CPL = HD / 32;  // output columns per lane
  extern __shared__ __align__(16) float dsm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x * WPC + warp;
  if (c >= a.n_chains) return;  // whole warps only: nothing below synchronises across warps
  float* qf = dsm + (size_t)warp * (2 * NRM * HD + NRM * kLP);  // [NRM][HD] q_rope
  float* qr = qf + NRM * HD;                                    // [NRM][HD] q_raw
  float* sc = qr + NRM * HD;                                    // [NRM][kLP] scores, then probabilities

  const int kvh = c % a.hkv, b = c / a.hkv;
  const int G = a.G, T = (int)a.Tq, NR = G * T, H = a.hkv * G;
  const bool has_sinks = a.has_sinks != 0, has_bank = a.has_bank != 0;
  const int n_sk = has_sinks ? 4 : 0, n_at = has_bank ? S : 0;
  const int L0 = a.seg0_len, L1 = a.seg1_len;
  const int L = n_sk + n_at + L0 + L1;

  const int64_t bofs = (int64_t)c * a.bank_cap;
  const bf16* sk = has_sinks ? reinterpret_cast<const bf16*>(a.sink_k) + (int64_t)c * a.sink_chain_tokens * HD : nullptr;
  const bf16* sv = has_sinks ? reinterpret_cast<const bf16*>(a.sink_v) + (int64_t)c * a.sink_chain_tokens * HD : nullptr;
  const bf16* bk = has_bank ? reinterpret_cast<const bf16*>(a.bank_ak_rope) + bofs * S * HD : nullptr;
  const bf16* bv = has_bank ? reinterpret_cast<const bf16*>(a.bank_av) + bofs * S * HD : nullptr;
  const bf16* k0 = reinterpret_cast<const bf16*>(a.seg0_k) + (int64_t)c * a.seg0_chain_tokens * HD;
  const bf16* v0 = reinterpret_cast<const bf16*>(a.seg0_v) + (int64_t)c * a.seg0_chain_tokens * HD;
  const bf16* k1 = reinterpret_cast<const bf16*>(a.seg1_k) + (int64_t)c * a.seg1_chain_tokens * HD;
  const bf16* v1 = reinterpret_cast<const bf16*>(a.seg1_v) + (int64_t)c * a.seg1_chain_tokens * HD;
  // key k of the concatenated list: its key row, value row, segment and index within the segment
  auto key_rows = [&](int k, const bf16*& kp, const bf16*& vp, int& seg, int& j) {
    if (k < n_sk) { seg = 0; j = k; kp = sk + (int64_t)j * HD; vp = sv + (int64_t)j * HD; return; }
    k -= n_sk;
    if (k < n_at) { seg = 1; j = k; kp = bk + (int64_t)j * HD; vp = bv + (int64_t)j * HD; return; }
    k -= n_at;
    if (k < L0) { seg = 2; j = k; kp = k0 + (int64_t)j * HD; vp = v0 + (int64_t)j * HD; return; }
    seg = 3; j = k - L0; kp = k1 + (int64_t)j * HD; vp = v1 + (int64_t)j * HD;
  };

  // ---- the first key row of this lane is requested before the query rows are staged
  uint4 kv[HD / 8];
  int seg_n = 0, j_n = 0;
  if (lane < L) {
    const bf16 *kp, *vp;
    key_rows(lane, kp, vp, seg_n, j_n);
#pragma unroll
    for (int ch = 0; ch < HD / 8; ++ch) kv[ch] = __ldg(reinterpret_cast<const uint4*>(kp) + ch);
  }
  const bf16* q_rope = reinterpret_cast<const bf16*>(a.q_rope);
  const bf16* q_raw = reinterpret_cast<const bf16*>(a.q_raw);
  auto qrow = [&](int r) { return ((int64_t)c * G + r / T) * a.Tq + r % T; };  // row of (head g, token i)
  for (int i = lane; i < NR * HD / 8; i += 32) {
    const int r = i / (HD / 8), ch = i % (HD / 8);
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(q_rope + qrow(r) * HD) + ch);
    const uint4 w = __ldg(reinterpret_cast<const uint4*>(q_raw + qrow(r) * HD) + ch);
    const uint32_t uu[4] = {u.x, u.y, u.z, u.w}, ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = unpack_bf16(uu[q]), h2 = unpack_bf16(ww[q]);
      qf[r * HD + ch * 8 + 2 * q] = f.x;
      qf[r * HD + ch * 8 + 2 * q + 1] = f.y;
      qr[r * HD + ch * 8 + 2 * q] = h2.x;
      qr[r * HD + ch * 8 + 2 * q + 1] = h2.y;
    }
  }
  __syncwarp();

  // ---- scores: a lane per key
  constexpr float scale = HD == 128 ? 0.08838834764831845f : 0.125f;  // fp32(HD ** -0.5)
  for (int k = lane; k < L; k += 32) {
    int seg = seg_n, j = j_n;
    if (k != lane) {
      const bf16 *kp, *vp;
      key_rows(k, kp, vp, seg, j);
#pragma unroll
      for (int ch = 0; ch < HD / 8; ++ch) kv[ch] = __ldg(reinterpret_cast<const uint4*>(kp) + ch);
    }
    float acc[NRM];
#pragma unroll
    for (int r = 0; r < NRM; ++r) acc[r] = 0.f;
#pragma unroll
    for (int ch = 0; ch < HD / 8; ++ch) {
      const uint32_t w[4] = {kv[ch].x, kv[ch].y, kv[ch].z, kv[ch].w};
      float kf[8];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float2 f = unpack_bf16(w[u]);
        kf[2 * u] = f.x;
        kf[2 * u + 1] = f.y;
      }
#pragma unroll
      for (int r = 0; r < NRM; ++r) {
        if (r >= NR) break;
        const float4 qa = *reinterpret_cast<const float4*>(qf + r * HD + ch * 8);
        const float4 qb = *reinterpret_cast<const float4*>(qf + r * HD + ch * 8 + 4);
        float s2 = acc[r];
        s2 = fmaf(qa.x, kf[0], s2); s2 = fmaf(qa.y, kf[1], s2); s2 = fmaf(qa.z, kf[2], s2); s2 = fmaf(qa.w, kf[3], s2);
        s2 = fmaf(qb.x, kf[4], s2); s2 = fmaf(qb.y, kf[5], s2); s2 = fmaf(qb.z, kf[6], s2); s2 = fmaf(qb.w, kf[7], s2);
        acc[r] = s2;
      }
    }
    float bias = 0.f;
    if (seg == 1)
      bias = a.bank_act[bofs * S + j] ? __fmul_rn(a.kappa[kvh], logf(fmaxf(a.bank_mass[bofs * S + j], 1.0f)))
                                      : neg_inf();
#pragma unroll
    for (int r = 0; r < NRM; ++r) {
      if (r >= NR) break;
      const int i = r % T;  // the row's new token
      float s2 = __fmul_rn(acc[r], scale);
      if (seg == 1) s2 = __fadd_rn(s2, bias);
      if (seg == 3 && j > a.len_before + i) s2 = neg_inf();
      sc[r * kLP + k] = s2;
    }
  }
  __syncwarp();

  // ---- softmax per row: p = bf16(exp(s - max) * (1 / sum))
  for (int r = 0; r < NR; ++r) {
    float* row = sc + r * kLP;
    float mx = neg_inf();
    for (int k = lane; k < L; k += 32) mx = fmaxf(mx, row[k]);
    mx = warp_max(mx);
    float sum = 0.f;
    for (int k = lane; k < L; k += 32) sum += expf(row[k] - mx);
    sum = warp_sum(sum);
    const float inv = 1.0f / sum;
    for (int k = lane; k < L; k += 32) row[k] = rbf(__fmul_rn(expf(row[k] - mx), inv));
  }
  __syncwarp();

  // ---- P@V: lane -> columns lane*CPL .. +CPL-1. Value rows in batches of VB, the next batch in
  // flight while this one is accumulated.
  using VT = typename std::conditional<CPL == 4, uint2, uint32_t>::type;  // CPL bf16
  constexpr int VB = 16;
  float o[NRM][CPL];
#pragma unroll
  for (int r = 0; r < NRM; ++r)
#pragma unroll
    for (int e = 0; e < CPL; ++e) o[r][e] = 0.f;
  auto fetch_v = [&](int kb, VT (&vq)[VB]) {
#pragma unroll
    for (int u = 0; u < VB; ++u) {
      const int k = kb + u;
      if (k < L) {
        const bf16 *kp, *vp;
        int seg, j;
        key_rows(k, kp, vp, seg, j);
        vq[u] = __ldg(reinterpret_cast<const VT*>(vp) + lane);
      }
    }
  };
  auto accum_v = [&](int kb, const VT (&vq)[VB]) {
#pragma unroll
    for (int u = 0; u < VB; ++u) {
      const int k = kb + u;
      if (k >= L) break;
      float vf[CPL];
      if constexpr (CPL == 4) {
        const float2 f0 = unpack_bf16(vq[u].x), f1 = unpack_bf16(vq[u].y);
        vf[0] = f0.x; vf[1] = f0.y; vf[2] = f1.x; vf[3] = f1.y;
      } else {
        const float2 f0 = unpack_bf16(vq[u]);
        vf[0] = f0.x; vf[1] = f0.y;
      }
#pragma unroll
      for (int r = 0; r < NRM; ++r) {
        if (r >= NR) break;
        const float p = sc[r * kLP + k];
#pragma unroll
        for (int e = 0; e < CPL; ++e) o[r][e] = fmaf(p, vf[e], o[r][e]);
      }
    }
  };
  {
    VT va[VB], vb[VB];
    fetch_v(0, va);
    for (int kb = 0; kb < L; kb += 2 * VB) {
      if (kb + VB < L) fetch_v(kb + VB, vb);
      accum_v(kb, va);
      if (kb + VB >= L) break;
      if (kb + 2 * VB < L) fetch_v(kb + 2 * VB, va);
      accum_v(kb + VB, vb);
    }
  }

  // ---- M_res read-out: R[r][e] = sum_d q_raw[r][d] * M[d][e] in fp32, lane -> its CPL columns e
  float ym[NRM][CPL];
  float rs[NRM];
  if (has_bank) {
    const float* M = reinterpret_cast<const float*>(a.bank_m) + (int64_t)c * a.bank_cap * HD * HD;
    using MT = typename std::conditional<CPL == 4, float4, float2>::type;
#pragma unroll
    for (int r = 0; r < NRM; ++r)
#pragma unroll
      for (int e = 0; e < CPL; ++e) ym[r][e] = 0.f;
    // rows d in batches of 8, the next batch in flight while this one is accumulated
    MT mn[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) mn[u] = __ldg(reinterpret_cast<const MT*>(M + (int64_t)u * HD) + lane);
    for (int d0 = 0; d0 < HD; d0 += 8) {
      MT mv[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) mv[u] = mn[u];
      if (d0 + 8 < HD) {
#pragma unroll
        for (int u = 0; u < 8; ++u) mn[u] = __ldg(reinterpret_cast<const MT*>(M + (int64_t)(d0 + 8 + u) * HD) + lane);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        float mf[CPL];
        if constexpr (CPL == 4) {
          mf[0] = mv[u].x; mf[1] = mv[u].y; mf[2] = mv[u].z; mf[3] = mv[u].w;
        } else {
          mf[0] = mv[u].x; mf[1] = mv[u].y;
        }
#pragma unroll
        for (int r = 0; r < NRM; ++r) {
          if (r >= NR) break;
          const float qv = qr[r * HD + d0 + u];
#pragma unroll
          for (int e = 0; e < CPL; ++e) ym[r][e] = fmaf(qv, mf[e], ym[r][e]);
        }
      }
    }
    // ym = R / |q_raw| * coef; rs = 1 / sqrt(mean(ym^2) + eps)
    const float coef = a.coef[kvh];
#pragma unroll
    for (int r = 0; r < NRM; ++r) {
      if (r >= NR) break;
      float qn;
      if (a.q_l2 != nullptr) {
        qn = a.q_l2[qrow(r)];
      } else {
        float s2 = 0.f;
        for (int d = lane; d < HD; d += 32) s2 = fmaf(qr[r * HD + d], qr[r * HD + d], s2);
        qn = sqrtf(warp_sum(s2));
      }
      const float iq = 1.0f / fmaxf(qn, 1e-12f);
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < CPL; ++e) {
        ym[r][e] = __fmul_rn(__fmul_rn(ym[r][e], iq), coef);
        ss = fmaf(ym[r][e], ym[r][e], ss);
      }
      ss = warp_sum(ss);
      rs[r] = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, (float)HD), a.eps));
    }
  }

  // ---- output: y = bf16(bf16(O) + bf16(eta * (ym * rs) * w))
  bf16* y = reinterpret_cast<bf16*>(a.y);
#pragma unroll
  for (int r = 0; r < NRM; ++r) {
    if (r >= NR) break;
    const float eta = has_bank ? a.eta[qrow(r)] : 0.f;
    uint32_t packed[CPL / 2];
#pragma unroll
    for (int e = 0; e < CPL; e += 2) {
      const float2 ob = rbf2(o[r][e], o[r][e + 1], packed[e / 2]);
      if (has_bank) {
        float t[2];
#pragma unroll
        for (int u = 0; u < 2; ++u)
          t[u] = __fmul_rn(eta, __fmul_rn(__fmul_rn(ym[r][e + u], rs[r]), a.res_w[lane * CPL + e + u]));
        uint32_t tmp;
        const float2 tr = rbf2(t[0], t[1], tmp);
        packed[e / 2] = pack_bf16(__fadd_rn(ob.x, tr.x), __fadd_rn(ob.y, tr.y));
      }
    }
    const int g = r / T, i = r % T;
    bf16* yrow = y + (((int64_t)b * a.y_tokens + i) * H + kvh * G + g) * HD + lane * CPL;
    if constexpr (CPL == 4) *reinterpret_cast<uint2*>(yrow) = make_uint2(packed[0], packed[1]);
    else *reinterpret_cast<uint32_t*>(yrow) = packed[0];
  }
}

template <int HD, int NRM>
int launch(const bolt3_attend_args* a, cudaStream_t s) {
  constexpr int WPC = warps_per_cta<NRM>();
  const size_t smem = sizeof(float) * (size_t)WPC * (2 * NRM * HD + NRM * kLP);
  auto kern = attend_decode_kernel<HD, NRM>;
  if (smem > 48 * 1024 && cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return BOLT3_ERR_CUDA;
  kern<<<(a->n_chains + WPC - 1) / WPC, 32 * WPC, smem, s>>>(*a);
  return cudaGetLastError() == cudaSuccess ? BOLT3_OK : BOLT3_ERR_CUDA;
}

}  // namespace b3dec

// Launch for bolt3_attend (prefill = 0, G * Tq <= 16); returns a bolt3 status.
int b3_attend_decode_launch(const bolt3_attend_args* a, cudaStream_t s) {
  const int NR = a->G * (int)a->Tq;
  if (NR > 16 || a->seg0_len + a->seg1_len > 256) return BOLT3_ERR_SHAPE;
  if (a->HD == 128) return NR <= 4 ? b3dec::launch<128, 4>(a, s) : (NR <= 8 ? b3dec::launch<128, 8>(a, s) : b3dec::launch<128, 16>(a, s));
  if (a->HD == 64) return NR <= 4 ? b3dec::launch<64, 4>(a, s) : (NR <= 8 ? b3dec::launch<64, 8>(a, s) : b3dec::launch<64, 16>(a, s));
  return BOLT3_ERR_SHAPE;
}
