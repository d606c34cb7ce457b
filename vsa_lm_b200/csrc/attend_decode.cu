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
#include "tc5.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <type_traits>

// 3-D tensor map of bf16 rows (attend.cu)
bool b3_encode_bf16_rows(CUtensorMap* m, const void* base, int hd, int64_t rows, int64_t slice_stride,
                         int64_t slices, int box_rows);

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
  // device step position: segment 1 holds d more keys, all visible d positions later
  int dpos = 0;
  if (a.pos_dev != nullptr) {
    const int64_t d = *a.pos_dev - a.pos_ref;
    if (d < 0 || d >= a.pos_span) {
      if (lane == 0 && a.status) atomicOr(a.status, 8);
      return;
    }
    dpos = (int)d;
  }
  const int L0 = a.seg0_len, L1 = a.seg1_len + dpos, len_before = a.len_before + dpos;
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
      if (seg == 3 && j > len_before + i) s2 = neg_inf();
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


// ---------------------------------------------------------------------------------------------
// Tensor-core streaming kernel for HD = 128 and at most four query rows per chain (the one-token step
// with G <= 4).
//
// The step reads every chain's state once, so it is bound by how much of it is in flight. Persistent
// CTAs (two per SM) walk strided lists of chains with three roles: a producer warp whose
// lane 0 copies the operands with the TMA engine into a ring of NST 32 KB stages, an MMA warp whose
// lane 0 issues every tensor-core product, and eight consumer warps for the softmax, the M_res
// read-out and the output. The roles meet only at mbarriers, so no role waits on another's data
// unless it needs that data. The MMA warp is the ring's one reader: as an R piece lands, the whole
// warp copies the chain's operands out of it into per-chain buffers (the Q tile and the sink values'
// tile, the attractor score bias, q_raw transposed, the rows' norms) and hands them to the consumers
// through a per-chain mbarrier, so the stage turns over without waiting for them. The ring pieces:
//   R  piece   the chain's small operands: q_rope rows as a 16-row K-major tile (rows past the
//              chain's own read as zero), the 4 sink keys and values as 16-row tiles, q_raw, and the
//              bank's mass and act;
//   K  pieces  one per segment (attractors, previous chunk, current chunk): 128 rows by 3-D tensor
//              maps into 128-byte swizzled tiles; rows past the segment read as zero;
//   V  pieces  the value rows of each segment, the same way.
// Every ring operand is read once, so its copies carry an evict-first L2 policy. The ring carries the
// chains software-pipelined, R and K of chain i+1 ahead of V of chain i: chain i+1's scores are
// computed while chain i's softmax runs, and chain i's values are multiplied as soon as they land
// after it. The fp32 M_res (64 KB) does not travel in the ring: a bulk prefetch pulls it into L2 when
// the consumers start the chain, and they read it from there with plain loads after the softmax.
// Scores are one tcgen05.mma per segment and 16-key step, S^T[key][row] = K . Q^T into tensor
// memory (double-buffered across chains; columns 16 s .. 16 s + 15 of a buffer, a lane per key). The
// softmax reads them back (exact: a sweep for the max, one for the sum) and writes the bf16
// probabilities as the K-major B tile of O^T[e][row] = V^T . P^T, issued per value segment with V as
// the MN-major A operand. The M_res read-out stays on the CUDA cores in fp32 (paired FMAs). Stages
// are released by a tcgen05.commit once the tensor cores (and, for R, the consumers) are done.
namespace stream {

constexpr int HD = 128;
constexpr int NST = 2;             // ring stages (two CTAs share an SM: four stages per SM)
constexpr int kStage = 32768;      // bytes per stage: 128 rows x 256 bytes
constexpr int NRM = 4;             // query rows per chain, padded
constexpr int NCW = 8;             // consumer warps (warps 0-7); warp 8 produces, warp 9 issues the MMAs
constexpr int NCT = NCW * 32;      // consumer threads
constexpr int kThreads = NCT + 64;
constexpr int kCtasPerSm = 2;      // two independent CTAs per SM interleave their chains' dependent phases
constexpr uint32_t kIters = 1u << 24;
// byte offsets inside the R piece: 16-row tiles (two 64-column halves each) of q_rope, sink keys,
// sink values; then q_raw, mass, act
constexpr int kRQ = 0, kRSK = 4096, kRSV = 8192, kRQRaw = 12288, kRMass = 13312, kRAct = 13824;
constexpr uint32_t kColO = 128;    // TMEM: scores buffer b in columns [64 b, 64 b + 64); O^T at 128
constexpr uint32_t kTmemCols = 256;
constexpr float kLog2e = 1.4426950408889634f;

// 2^x on the special-function unit (relative error ~2^-22; results below 2^-126 flush to zero)
B3_DEV float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

struct __align__(64) Maps {
  CUtensorMap q;                   // q_rope rows: {HD, NR, chains}, box {64, 16, 1}
  CUtensorMap k[4], v[4];          // sinks (box {64, 16, 1}); attractors, previous, current chunk (box {64, 128, 1})
};

struct __align__(1024) Smem {
  unsigned char ring[NST][kStage];
  unsigned char svt[2][4096];      // per chain buffer: the sink values' 16-row tile (MN-major A of P@V)
  unsigned char qbuf[2][4096];     // per chain buffer: the Q tile (K-major B of the score MMAs)
  unsigned char ptile[4][2][2048]; // probabilities of each segment: 16 rows x (2 x 64 keys), K-major SW128
  bf16 qd[3][HD][NRM];             // per chain buffer (local chain % 3): q_raw[row][d]
  float ypart[4][NRM][HD];         // M_res read-out partial sums of each quarter of d
  float bias[2][S];                // per chain buffer: the attractors' score bias
  float red[NCW][NRM], red2[NCW][NRM];
  float qn[3][NRM];                // per chain buffer (local chain % 3): |q_raw| of each row
  uint64_t full[NST], empty[NST];
  uint64_t bar_s[2], bar_o;        // MMA warp -> consumers: scores of a chain buffer; O^T of a chain
  uint64_t p_ready;                // consumers -> MMA warp: probabilities written
  uint64_t r_ready[2];             // MMA warp -> consumers: a chain's bias, q_raw and norms are written
  uint64_t fin;                    // the MMA warp's last commit
  uint32_t tbase;
  int err;
};

B3_DEV void cons_sync() { asm volatile("bar.sync 1, %0;\n" ::"n"(NCT) : "memory"); }
// OR of `v` over the consumer threads (also a barrier among them)
B3_DEV bool cons_any(bool v) {
  uint32_t r;
  asm volatile(
      "{\n.reg .pred p, q;\nsetp.ne.u32 p, %1, 0;\nbar.red.or.pred q, 1, %2, p;\nselp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(NCT)
      : "memory");
  return r != 0;
}

__global__ void __launch_bounds__(kThreads, kCtasPerSm) attend_stream_kernel(const bolt3_attend_args a,
                                                                    const __grid_constant__ Maps tm) {
  extern __shared__ unsigned char smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (a.wait_probe) {  // failure-path test hook: an expired bounded wait, reported as bit 2
    if (tid == 0 && !tc5::probe_wait(&sm.bar_o, a.wait_probe) && a.status) atomicOr(a.status, 2);
    return;
  }
  const int G = a.G, T = (int)a.Tq, NR = G * T, H = a.hkv * G;
  const bool has_bank = a.has_bank != 0, has_sinks = a.has_sinks != 0;
  // device step position (written before the step's first kernel ran): segment 1 holds d more keys,
  // all visible d positions later; out of range, the CTA reports it and does nothing
  int dpos = 0;
  if (a.pos_dev != nullptr) {
    const int64_t d = *a.pos_dev - a.pos_ref;
    if (d < 0 || d >= a.pos_span) {
      if (tid == 0 && a.status) atomicOr(a.status, 8);
      return;
    }
    dpos = (int)d;
  }
  const int len_before = a.len_before + dpos;
  const int len[4] = {has_sinks ? 4 : 0, has_bank ? S : 0, a.seg0_len, a.seg1_len + dpos};
  // the segments that travel as ring pieces (the sinks travel in the R piece)
  int n_kv = 0, kv_list[3];
#pragma unroll
  for (int s = 1; s < 4; ++s)
    if (len[s] > 0) kv_list[n_kv++] = s;
  // chains of this CTA: blockIdx.x + li * gridDim.x, li < n_local
  const int n_local = a.n_chains > (int)blockIdx.x ? (a.n_chains - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  // a wait that gives up records the error; once one has, the MMA warp skips its later waits (the
  // work after them is void) so that the CTA ends quickly
  auto wait_or_flag = [&](uint64_t* bar, uint32_t parity) {
    if (*reinterpret_cast<volatile int*>(&sm.err) == 0 && !tc5::mbar_wait(bar, parity, kIters)) sm.err = 1;
  };

  if (tid == 0) {
    for (int s = 0; s < NST; ++s) {
      tc5::mbar_init(&sm.full[s], 1);
      tc5::mbar_init(&sm.empty[s], 1);
    }
    tc5::mbar_init(&sm.bar_s[0], 1);
    tc5::mbar_init(&sm.bar_s[1], 1);
    tc5::mbar_init(&sm.bar_o, 1);
    tc5::mbar_init(&sm.r_ready[0], 1);
    tc5::mbar_init(&sm.r_ready[1], 1);
    tc5::mbar_init(&sm.p_ready, 1);
    tc5::mbar_init(&sm.fin, 1);
    tc5::mbar_fence_init();
    sm.err = 0;
  }
  if (warp == 0) {
    tc5::tmem_alloc(&sm.tbase, kTmemCols);
    tc5::tmem_relinquish();
  }
  tc5::fence_before_sync();
  __syncthreads();
  tc5::fence_after_sync();
  const uint32_t tb = sm.tbase;
  // launched overlapped with the step's prep kernel: the set-up above touched only this CTA's own
  // shared and tensor memory; q, q_raw, the gates and the new window rows are read from here on
  b3::grid_dep_wait();

  if (warp == NCW) {
    // ---- producer: per step li = -1 .. n_local - 1, R and K of chain li + 1, then V of chain li
    if (lane == 0) {
      uint32_t it = 0;
      bool stop = false;
      // every ring operand is read once: its L2 lines go first, ahead of the prefetched M_res
      const uint64_t pol = tc5::policy_evict_first();
      // one ring piece; false once an error was recorded
      auto put = [&](auto&& issue) -> bool {
        const int s = (int)(it % NST);
        if (it >= (uint32_t)NST && !tc5::mbar_wait(&sm.empty[s], ((it / NST) & 1u) ^ 1u, kIters)) sm.err = 1;
        if (*reinterpret_cast<volatile int*>(&sm.err)) return false;
        issue(sm.ring[s], &sm.full[s]);
        ++it;
        return true;
      };
      for (int li = -1; li < n_local && !stop; ++li) {
        if (li + 1 < n_local) {
          const int c = (int)blockIdx.x + (li + 1) * (int)gridDim.x;
          const int64_t bofs = (int64_t)c * a.bank_cap;
          stop = !put([&](unsigned char* buf, uint64_t* bar) {
            const uint32_t qb = (uint32_t)NR * HD * 2;
            tc5::mbar_expect_tx(bar, 2 * 2048 + (has_sinks ? 4 * 2048 : 0) + qb + (has_bank ? S * 4 + S : 0));
            for (int h = 0; h < 2; ++h) tc5::tma_load_3d(buf + kRQ + h * 2048, &tm.q, h * 64, 0, c, bar, pol);
            if (has_sinks)
              for (int h = 0; h < 2; ++h) {
                tc5::tma_load_3d(buf + kRSK + h * 2048, &tm.k[0], h * 64, 0, c, bar, pol);
                tc5::tma_load_3d(buf + kRSV + h * 2048, &tm.v[0], h * 64, 0, c, bar, pol);
              }
            tc5::bulk_load(buf + kRQRaw, reinterpret_cast<const bf16*>(a.q_raw) + (int64_t)c * NR * HD, qb, bar, pol);
            if (has_bank) {
              tc5::bulk_load(buf + kRMass, a.bank_mass + bofs * S, S * 4, bar, pol);
              tc5::bulk_load(buf + kRAct, a.bank_act + bofs * S, S, bar, pol);
            }
          });
          for (int i = 0; i < n_kv && !stop; ++i) {
            const int sg = kv_list[i];
            stop = !put([&](unsigned char* buf, uint64_t* bar) {
              tc5::mbar_expect_tx(bar, 2 * 16384);
              for (int h = 0; h < 2; ++h)
                tc5::tma_load_3d(buf + h * 16384, &tm.k[sg], h * 64, 0, sg == 1 ? (int)bofs : c, bar, pol);
            });
          }
        }
        if (li >= 0 && !stop) {
          const int c = (int)blockIdx.x + li * (int)gridDim.x;
          const int64_t bofs = (int64_t)c * a.bank_cap;
          for (int i = 0; i < n_kv && !stop; ++i) {
            const int sg = kv_list[i];
            stop = !put([&](unsigned char* buf, uint64_t* bar) {
              tc5::mbar_expect_tx(bar, 2 * 16384);
              for (int h = 0; h < 2; ++h)
                tc5::tma_load_3d(buf + h * 16384, &tm.v[sg], h * 64, 0, sg == 1 ? (int)bofs : c, bar, pol);
            });
          }
        }
      }
      // after an early stop, copies may still be in flight: wait (bounded) for the last phase armed
      // on every stage before the CTA's shared memory is released
      for (uint32_t j = it > (uint32_t)NST ? it - NST : 0; j < it; ++j)
        tc5::mbar_wait(&sm.full[j % NST], (j / NST) & 1u, kIters);
    }
  } else if (warp == NCW + 1) {
    // ---- MMA warp: per step, the R piece and the score MMAs of chain li + 1, then the P@V MMAs of
    // chain li. The whole warp copies the R piece's operands out as soon as it lands, so that its
    // stage turns over without waiting for the consumers; lane 0 issues the MMAs and commits.
    constexpr uint32_t kIdS = tc5::idesc_bf16(128, 16, false, false);
    constexpr uint32_t kIdO = tc5::idesc_bf16(128, 16, true, false);
    uint32_t it = 0;
    auto stage_wait = [&]() -> int {
      const int s = (int)(it % NST);
      wait_or_flag(&sm.full[s], (it / NST) & 1u);
      tc5::fence_after_sync();
      return s;
    };
    for (int li = -1; li < n_local; ++li) {
      if (li + 1 < n_local) {
        const int cn = li + 1, bn = cn & 1, qi = cn % 3;
        const int c = (int)blockIdx.x + cn * (int)gridDim.x;
        const int sr = stage_wait();
        ++it;
        // buffers of chain cn: qbuf and bias were last read by chain cn - 2's scores and softmax
        // (complete: this warp has seen chain li - 1's probabilities); svt by its P@V, which may
        // still run; qd and qn are three-deep (chain cn - 3's read-out and epilogue are done)
        if (li >= 1 && has_sinks) wait_or_flag(&sm.bar_o, (uint32_t)(li - 1) & 1u);
        tc5::fence_after_sync();
        const unsigned char* buf = sm.ring[sr];
        for (int j = lane; j < 4096 / 16; j += 32) {
          reinterpret_cast<uint4*>(sm.qbuf[bn])[j] = reinterpret_cast<const uint4*>(buf + kRQ)[j];
          if (has_sinks) reinterpret_cast<uint4*>(sm.svt[bn])[j] = reinterpret_cast<const uint4*>(buf + kRSV)[j];
        }
        if (has_bank) {
          const float kappa = __ldg(a.kappa + c % a.hkv);
          const float* mass = reinterpret_cast<const float*>(buf + kRMass);
          for (int j = lane; j < S; j += 32)
            sm.bias[bn][j] = buf[kRAct + j] ? __fmul_rn(kappa, logf(fmaxf(mass[j], 1.0f))) : neg_inf();
          // q_raw transposed to qd[d][row] (rows past NR zero): lane takes d = 4 lane .. 4 lane + 3
          const uint32_t* qr = reinterpret_cast<const uint32_t*>(buf + kRQRaw);
          uint2 w[NRM];
#pragma unroll
          for (int r = 0; r < NRM; ++r) w[r] = r < NR ? make_uint2(qr[r * (HD / 2) + 2 * lane], qr[r * (HD / 2) + 2 * lane + 1])
                                                      : make_uint2(0u, 0u);
          uint2* qo = reinterpret_cast<uint2*>(&sm.qd[qi][4 * lane][0]);
          qo[0] = make_uint2(__byte_perm(w[0].x, w[1].x, 0x5410), __byte_perm(w[2].x, w[3].x, 0x5410));
          qo[1] = make_uint2(__byte_perm(w[0].x, w[1].x, 0x7632), __byte_perm(w[2].x, w[3].x, 0x7632));
          qo[2] = make_uint2(__byte_perm(w[0].y, w[1].y, 0x5410), __byte_perm(w[2].y, w[3].y, 0x5410));
          qo[3] = make_uint2(__byte_perm(w[0].y, w[1].y, 0x7632), __byte_perm(w[2].y, w[3].y, 0x7632));
          if (a.q_l2 == nullptr) {
            // |q_raw| per row: lane sums d = lane, lane + 32, ... in order, then the warp
            const bf16* qb = reinterpret_cast<const bf16*>(buf + kRQRaw);
            for (int r = 0; r < NR; ++r) {
              float s2 = 0.f;
              for (int d = lane; d < HD; d += 32) {
                const float q = __bfloat162float(qb[r * HD + d]);
                s2 = fmaf(q, q, s2);
              }
              s2 = warp_sum(s2);
              if (lane == 0) sm.qn[qi][r] = sqrtf(s2);
            }
          }
        }
        // the copies are read by the tensor cores (Q, sink values) and by the consumers
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          tc5::mbar_arrive(&sm.r_ready[bn]);
          // S^T = K . Q^T per segment; the sinks' keys are read from the R piece itself
          const uint32_t ra = tc5::smem_u32(sm.ring[sr]);
          const uint32_t qa = tc5::smem_u32(sm.qbuf[bn]);
          if (has_sinks) {
#pragma unroll
            for (int ks = 0; ks < HD / 16; ++ks)
              tc5::mma_ss(tb + 64 * bn, tc5::sdesc(ra + kRSK + (ks >> 2) * 2048 + (ks & 3) * 32, 16, 1024),
                          tc5::sdesc(qa + (ks >> 2) * 2048 + (ks & 3) * 32, 16, 1024), kIdS, ks > 0);
          }
          tc5::commit(&sm.empty[sr]);
        }
        // S^T = K . Q^T of the ring segments
        const uint32_t qa = tc5::smem_u32(sm.qbuf[bn]);
        for (int i = 0; i < n_kv; ++i) {
          const int s = stage_wait();
          ++it;
          if (lane == 0) {
            const uint32_t ka = tc5::smem_u32(sm.ring[s]);
            const uint32_t dcol = tb + 64 * bn + 16 * kv_list[i];
#pragma unroll
            for (int ks = 0; ks < HD / 16; ++ks)
              tc5::mma_ss(dcol, tc5::sdesc(ka + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024),
                          tc5::sdesc(qa + (ks >> 2) * 2048 + (ks & 3) * 32, 16, 1024), kIdS, ks > 0);
            tc5::commit(&sm.empty[s]);
          }
        }
        if (lane == 0) tc5::commit(&sm.bar_s[bn]);
        __syncwarp();
      }
      if (li >= 0) {
        // O^T = V^T . P^T once the consumers have written chain li's probabilities
        const int bi = li & 1;
        wait_or_flag(&sm.p_ready, (uint32_t)li & 1u);
        tc5::fence_after_sync();
        bool first = true;
        if (has_sinks && lane == 0) {  // one 16-key step: sink rows 4..15 of the tile are zero, their P columns too
          tc5::mma_ss(tb + kColO, tc5::sdesc(tc5::smem_u32(sm.svt[bi]), 2048, 1024),
                      tc5::sdesc(tc5::smem_u32(sm.ptile[0][0]), 16, 1024), kIdO, false);
        }
        if (has_sinks) first = false;
        for (int i = 0; i < n_kv; ++i) {
          const int s = stage_wait();
          ++it;
          const int sg = kv_list[i];
          const int nks = (len[sg] + 15) / 16;
          if (lane == 0) {
            const uint32_t va = tc5::smem_u32(sm.ring[s]);
            const uint32_t pa = tc5::smem_u32(sm.ptile[sg][0]);
            for (int ks = 0; ks < nks; ++ks)
              tc5::mma_ss(tb + kColO, tc5::sdesc(va + ks * 2048, 16384, 1024),
                          tc5::sdesc(pa + (ks >> 2) * 2048 + (ks & 3) * 32, 16, 1024), kIdO, !first || ks > 0);
            tc5::commit(&sm.empty[s]);
          }
          if (nks > 0) first = false;
        }
        if (lane == 0) tc5::commit(&sm.bar_o);
        __syncwarp();
      }
    }
    // every product issued has completed before the tensor memory is released (also after an error)
    if (lane == 0) {
      tc5::commit(&sm.fin);
      tc5::mbar_wait(&sm.fin, 0, kIters);
    }
    __syncwarp();
  } else {
    // ---- consumers (threads 0..255)
    const int t = tid;
    constexpr float scale = 0.08838834764831845f;  // fp32(128 ** -0.5)
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
    const int rg = warp >> 2;               // query rows 2 rg, 2 rg + 1 in the softmax and the epilogue
    const int kq = 32 * (warp & 3) + lane;  // this thread's TMEM lane: a key of a segment, or a column e
    for (int li = 0; li < n_local; ++li) {
      const int c = (int)blockIdx.x + li * (int)gridDim.x;
      const int kvh = c % a.hkv, b = c / a.hkv;
      const int bi = li & 1;
      // the chain's fp32 M_res is read straight from L2 after the softmax: pull it in now (earlier,
      // and the operands streaming through L2 meanwhile evict much of it before it is read)
      if (has_bank && t == 0)
        tc5::prefetch_l2(reinterpret_cast<const float*>(a.bank_m) + (int64_t)c * a.bank_cap * HD * HD, HD * HD * 4);
      // the epilogue's per-row scalars, requested now and used at the end
      float eta_r[2], ql2_r[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int r = 2 * rg + j;
        eta_r[j] = has_bank && r < NR ? __ldg(a.eta + (int64_t)c * NR + r) : 0.f;
        ql2_r[j] = has_bank && r < NR && a.q_l2 != nullptr ? __ldg(a.q_l2 + (int64_t)c * NR + r) : 0.f;
      }
      const float coef = has_bank ? __ldg(a.coef + kvh) : 0.f;
      const float res_w = has_bank ? __ldg(a.res_w + kq) : 0.f;

      // -- softmax of chain li: thread (key kq of each segment, rows 2 rg, 2 rg + 1)
      if (!tc5::mbar_wait(&sm.r_ready[bi], (uint32_t)(li >> 1) & 1u, kIters)) sm.err = 1;
      if (!tc5::mbar_wait(&sm.bar_s[bi], (uint32_t)(li >> 1) & 1u, kIters)) sm.err = 1;
      tc5::fence_after_sync();
      uint32_t v[4][4];
#pragma unroll
      for (int sg = 0; sg < 4; ++sg)
        if (len[sg] > 0) tc5::ld4(tb + lane_off + 64 * bi + 16 * sg, v[sg]);
      tc5::ld_wait();
      float sv[4][2];
      float mx[2] = {neg_inf(), neg_inf()};
#pragma unroll
      for (int sg = 0; sg < 4; ++sg) {
        sv[sg][0] = sv[sg][1] = neg_inf();
        if (kq >= len[sg]) continue;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int r = 2 * rg + u;
          if (r >= NR) continue;
          float s2 = __fmul_rn(__uint_as_float(v[sg][r]), scale);
          if (sg == 1) s2 = __fadd_rn(s2, sm.bias[bi][kq]);
          if (sg == 3 && kq > len_before + r % T) s2 = neg_inf();
          sv[sg][u] = s2;
          mx[u] = fmaxf(mx[u], s2);
        }
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const float m = warp_max(mx[u]);
        if (lane == 0) sm.red[warp][2 * rg + u] = m;
      }
      cons_sync();
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int r = 2 * rg + u;
        mx[u] = fmaxf(fmaxf(sm.red[4 * rg][r], sm.red[4 * rg + 1][r]), fmaxf(sm.red[4 * rg + 2][r], sm.red[4 * rg + 3][r]));
        float sum = 0.f;
#pragma unroll
        for (int sg = 0; sg < 4; ++sg) {
          // exp(s - max), kept for the probabilities
          sv[sg][u] = kq < len[sg] && r < NR ? ex2(__fmul_rn(sv[sg][u] - mx[u], kLog2e)) : 0.f;
          sum += sv[sg][u];
        }
        const float w = warp_sum(sum);
        if (lane == 0) sm.red2[warp][r] = w;
      }
      cons_sync();
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int r = 2 * rg + u;
        const float tot = sm.red2[4 * rg][r] + sm.red2[4 * rg + 1][r] + sm.red2[4 * rg + 2][r] + sm.red2[4 * rg + 3][r];
        const float inv = 1.0f / tot;
#pragma unroll
        for (int sg = 0; sg < 4; ++sg) {
          if (len[sg] == 0) continue;
          const float pv = r < NR ? rbf(__fmul_rn(sv[sg][u], inv)) : 0.f;
          *reinterpret_cast<bf16*>(sm.ptile[sg][kq >> 6] + tc5::sw128_off(r, kq & 63)) = __float2bfloat16_rn(pv);
        }
      }
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
      tc5::fence_before_sync();
      cons_sync();
      if (t == 0) tc5::mbar_arrive(&sm.p_ready);

      // -- M_res read-out: R[r][e] = sum_d q_raw[r][d] * M[d][e] in fp32; thread (column pair, quarter
      // of the rows d), all four rows, two columns per paired FMA
      float2 ym2[NRM];
#pragma unroll
      for (int r = 0; r < NRM; ++r) ym2[r] = make_float2(0.f, 0.f);
      const int cpm = t & 63, dq = t >> 6;
      if (has_bank) {
        // M read from L2 (prefetched at the start of the chain), eight rows of M in flight
        const int d0 = dq * (HD / 4);
        const float2* mg = reinterpret_cast<const float2*>(reinterpret_cast<const float*>(a.bank_m) +
                                                           (int64_t)c * a.bank_cap * HD * HD + (int64_t)d0 * HD) + cpm;
        float2 mb[2][8];
#pragma unroll
        for (int u = 0; u < 8; ++u) mb[0][u] = __ldg(mg + u * (HD / 2));
#pragma unroll
        for (int blk = 0; blk < HD / 4 / 8; ++blk) {
          const int cur = blk & 1;
          if (blk + 1 < HD / 4 / 8) {
#pragma unroll
            for (int u = 0; u < 8; ++u) mb[cur ^ 1][u] = __ldg(mg + ((blk + 1) * 8 + u) * (HD / 2));
          }
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const float2 m2 = mb[cur][u];
            const uint2 qq = *reinterpret_cast<const uint2*>(&sm.qd[li % 3][d0 + blk * 8 + u][0]);
            const float2 q01 = unpack_bf16(qq.x), q23 = unpack_bf16(qq.y);
            const float4 q = make_float4(q01.x, q01.y, q23.x, q23.y);
            ym2[0] = __ffma2_rn(make_float2(q.x, q.x), m2, ym2[0]);
            ym2[1] = __ffma2_rn(make_float2(q.y, q.y), m2, ym2[1]);
            ym2[2] = __ffma2_rn(make_float2(q.z, q.z), m2, ym2[2]);
            ym2[3] = __ffma2_rn(make_float2(q.w, q.w), m2, ym2[3]);
          }
        }
      }
#pragma unroll
      for (int r = 0; r < NRM; ++r) *reinterpret_cast<float2*>(&sm.ypart[dq][r][2 * cpm]) = ym2[r];
      cons_sync();

      // -- epilogue: thread (column e = its TMEM lane, rows 2 rg, 2 rg + 1)
      const int e = kq;
      if (!tc5::mbar_wait(&sm.bar_o, (uint32_t)li & 1u, kIters)) sm.err = 1;
      tc5::fence_after_sync();
      uint32_t ov[4];
      tc5::ld4(tb + lane_off + kColO, ov);
      tc5::ld_wait();
      float ym[2], rs_r[2] = {0.f, 0.f};
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int r = 2 * rg + u;
        ym[u] = ((sm.ypart[0][r][e] + sm.ypart[1][r][e]) + sm.ypart[2][r][e]) + sm.ypart[3][r][e];
      }
      if (has_bank) {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int r = 2 * rg + u;
          const float qn = a.q_l2 != nullptr ? ql2_r[u] : (r < NR ? sm.qn[li % 3][r] : 1.f);
          const float iq = 1.0f / fmaxf(qn, 1e-12f);
          ym[u] = __fmul_rn(__fmul_rn(ym[u], iq), coef);
          const float ss = warp_sum(__fmul_rn(ym[u], ym[u]));
          if (lane == 0) sm.red[warp][r] = ss;
        }
        cons_sync();
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int r = 2 * rg + u;
          const float ss = ((sm.red[4 * rg][r] + sm.red[4 * rg + 1][r]) + sm.red[4 * rg + 2][r]) + sm.red[4 * rg + 3][r];
          rs_r[u] = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, (float)HD), a.eps));
        }
      }
      bf16* y = reinterpret_cast<bf16*>(a.y);
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int r = 2 * rg + u;
        if (r >= NR) break;
        float yv = rbf(__uint_as_float(ov[r]));
        if (has_bank) yv = __fadd_rn(yv, rbf(__fmul_rn(eta_r[u], __fmul_rn(__fmul_rn(ym[u], rs_r[u]), res_w))));
        const int g = r / T, i = r % T;
        y[(((int64_t)b * a.y_tokens + i) * H + kvh * G + g) * HD + e] = __float2bfloat16_rn(yv);
      }
      // the next chain overwrites the probability tile, the partial sums and the exchange rows
      tc5::fence_before_sync();
      if (cons_any(*reinterpret_cast<volatile int*>(&sm.err) != 0)) break;
      tc5::fence_after_sync();
    }
    if (t == 0 && sm.err && a.status) atomicOr(a.status, 2);
  }
  tc5::fence_before_sync();
  __syncthreads();
  tc5::fence_after_sync();
  if (warp == 0) tc5::tmem_dealloc(tb, kTmemCols);
}

// encodes the maps and launches kCtasPerSm CTAs per SM (at most one per chain); < 0: a map could not be
// encoded (the caller then uses the warp-per-chain kernel)
int launch(const bolt3_attend_args* a, cudaStream_t s) {
  Maps m;
  memset(&m, 0, sizeof(m));
  const int64_t nc = a->n_chains, NR = (int64_t)a->G * a->Tq;
  if (!b3_encode_bf16_rows(&m.q, a->q_rope, HD, NR, NR, nc, 16)) return -1;
  const void* kb[4] = {a->sink_k, a->bank_ak_rope, a->seg0_k, a->seg1_k};
  const void* vb[4] = {a->sink_v, a->bank_av, a->seg0_v, a->seg1_v};
  // segment 1's map covers the longest window a device step position allows (rows past the current
  // length are read and masked)
  const int64_t dmax = a->pos_dev != nullptr ? a->pos_span - 1 : 0;
  const int64_t rows[4] = {4, S, a->seg0_len, a->seg1_len + dmax};
  const int64_t stride[4] = {a->sink_chain_tokens, S, a->seg0_chain_tokens, a->seg1_chain_tokens};
  const int64_t slices[4] = {nc, nc * a->bank_cap, nc, nc};
  const bool on[4] = {a->has_sinks != 0, a->has_bank != 0, a->seg0_len > 0, a->seg1_len > 0};
  for (int i = 0; i < 4; ++i) {
    const int box = i == 0 ? 16 : 128;
    if (on[i] && (!b3_encode_bf16_rows(&m.k[i], kb[i], HD, rows[i], stride[i], slices[i], box) ||
                  !b3_encode_bf16_rows(&m.v[i], vb[i], HD, rows[i], stride[i], slices[i], box)))
      return -1;
  }
  const size_t smem = sizeof(Smem) + 1024;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return BOLT3_ERR_CUDA;
  // the shared-memory opt-in is per device: set it the first time each device launches
  constexpr int kMaxDev = 64;
  static std::atomic<bool> attr_set[kMaxDev];
  if (dev >= kMaxDev) return BOLT3_ERR_CUDA;
  if (!attr_set[dev].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(attend_stream_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess ||
        cudaFuncSetAttribute(attend_stream_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
      return BOLT3_ERR_CUDA;
    attr_set[dev].store(true, std::memory_order_release);
  }
  const int grid = (int)std::min<int64_t>(nc, (int64_t)sms * kCtasPerSm);
  // overlapped with the kernel before it (the step's prep): the CTAs allocate tensor memory and
  // initialise their barriers while prep finishes
  const cudaError_t e = b3::launch_overlapped(attend_stream_kernel, dim3(grid), dim3(kThreads), smem, s, *a, m);
  return e == cudaSuccess && cudaGetLastError() == cudaSuccess ? BOLT3_OK : BOLT3_ERR_CUDA;
}

}  // namespace stream

}  // namespace b3dec

// Launch for bolt3_attend (prefill = 0, G * Tq <= 16); returns a bolt3 status.
int b3_attend_decode_launch(const bolt3_attend_args* a, cudaStream_t s) {
  const int NR = a->G * (int)a->Tq;
  if (a->pos_dev != nullptr && a->pos_span < 1) return BOLT3_ERR_ARG;
  const int64_t dmax = a->pos_dev != nullptr ? a->pos_span - 1 : 0;
  if (NR > 16 || a->seg0_len + a->seg1_len + dmax > 256 || a->seg1_len + dmax > a->seg1_chain_tokens)
    return BOLT3_ERR_SHAPE;
  // HD = 128 with up to four query rows: the tensor-core streaming kernel, when its bulk copies'
  // alignment holds (the tensor maps are checked as they are encoded; a map that cannot be encoded
  // selects the warp-per-chain kernel below)
  const uintptr_t al = (uintptr_t)a->bank_mass | (uintptr_t)a->bank_act;
  if (NR <= 4 && (al & 15) == 0 && a->HD == 128) {
    const int rc = b3dec::stream::launch(a, s);
    if (rc >= 0) return rc;
  }
  if (a->HD == 128) return NR <= 4 ? b3dec::launch<128, 4>(a, s) : (NR <= 8 ? b3dec::launch<128, 8>(a, s) : b3dec::launch<128, 16>(a, s));
  if (a->HD == 64) return NR <= 4 ? b3dec::launch<64, 4>(a, s) : (NR <= 8 ? b3dec::launch<64, 8>(a, s) : b3dec::launch<64, 16>(a, s));
  return BOLT3_ERR_SHAPE;
}
