// Phase C: three-field softmax attention with the fused M_res read-out, on tcgen05 + TMEM.
//
// One CTA owns a 128-row query tile: prefill = 128 tokens of one query head; decode = the (head g,
// token) pairs of one KV head. Its scores against all keys stay resident in tensor memory, so the
// softmax is exact in one sweep of MMAs:
//   TMEM columns [0,128) attractors, [128,256) previous chunk, [256,384) current chunk (fp32 S);
//   [384, 384+HD) the P@V accumulator O. P (bf16, two per column) is written back over S in
//   columns [0,192) and is the A operand of the P@V MMAs; the M_res read-out accumulates into
//   columns [192, 192+HD) once the softmax has consumed them.
// Keys: [4 sinks] [S attractors: RoPE'd at their mean position, + kappa*log(mass), -inf if inactive]
// [previous chunk] [current chunk, causal] (vsa_lm/config/bolt3.py:219-249). The 4 sink scores are
// computed on the CUDA cores; everything else is tcgen05.mma with bf16 operands in 128-byte swizzled
// shared memory and fp32 accumulation. Probabilities are normalised before their bf16 cast exactly
// as the reference does (F.softmax(...).to(dtype), bolt3.py:249). The epilogue reads M_res out
// (bolt3.py:251-256): y = bf16( bf16(P@V) + bf16( eta * RMSNorm_w( q_raw @ (M_hi + M_lo) / |q_raw|
// * (1-gamma)/sqrt(HD) ) ) ), with M split into two bf16 terms.
//
// Both warpgroups handle every query row (TMEM lane = row), each on half of the columns, and swap
// row max / sum / RMS partials through shared memory. Warpgroup 1 also stages the M_res operand,
// the sink scores, and V / q_raw behind the consumed K tiles. Thread 0 issues the MMAs.
#include "../../include/bolt3.h"
#include "common.cuh"
#include "tc5.cuh"

#include <algorithm>
#include <type_traits>

namespace {

using namespace b3;

constexpr int S = 128;
constexpr int CC = 128;
constexpr int NT = 256;
constexpr uint32_t kWaitIters = 1u << 24;
constexpr uint32_t kColO = 384, kColR = 192;

template <int HD>
struct __align__(1024) Smem {
  unsigned char q[HD / 64][16384];        // q_rope tile, then the q_raw tile (K-major SW128)
  unsigned char kv[3][HD / 64][16384];    // K tiles of attractors / prev / cur, then their V tiles
  unsigned char m[2][HD / 64][HD * 128];  // M_res hi / lo (MN-major B): rows = input dim d, N blocks of e
  bf16 sink_k[4][HD];
  bf16 sink_v[4][HD];
  float sink_vf[4][HD];     // sink values in fp32 for the epilogue
  float sink_s[128][4];     // scaled sink scores per query row
  float res_w[HD];
  float red_max[2][128];    // per-row partial results exchanged between the two warpgroups
  float red_sum[2][128];
  float bias[S];
  uint64_t bar_s, bar_o;
  uint32_t tbase;
  int err;
};

// Contiguous 16-byte-chunk copy of a tile that is already a SW128 operand image (the snapshots
// written by the consolidation scan).
template <int HD>
B3_DEV void copy_image(unsigned char (*dst)[16384], const bf16* src, int t, int nthreads) {
  const unsigned char* s = reinterpret_cast<const unsigned char*>(src);
  for (int i = t; i < 128 * HD * 2 / 16; i += nthreads) cp_async16(&dst[0][0] + i * 16, s + i * 16, true);
}

// 16-byte-chunk cp.async of 128 rows of an [*][HD] bf16 array into a SW128 tile; rows at or beyond
// `valid` are zero-filled. Threads t, t + nthreads, ... take part.
template <int HD>
B3_DEV void load_tile(unsigned char (*dst)[16384], const bf16* src, int valid, int t, int nthreads) {
  constexpr int CPR = HD / 8;
  for (int i = t; i < 128 * CPR; i += nthreads) {
    const int r = i / CPR, ch = i % CPR;
    const bool ok = r < valid;
    unsigned char* d = dst[ch >> 3] + r * 128 + (((ch & 7) ^ (r & 7)) << 4);
    cp_async16(d, ok ? src + (int64_t)r * HD + ch * 8 : src, ok);
  }
}

template <int HD>
__global__ void __launch_bounds__(NT, 1) attend_tc_kernel(const bolt3_attend_args a) {
  extern __shared__ unsigned char smem_raw[];
  Smem<HD>& sm = *reinterpret_cast<Smem<HD>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5;
  const int G = a.G;
  const int g_fast = blockIdx.x;  // head group within the KV head: the G CTAs of one chain-chunk run
  const int blk = (int)a.blk_begin + blockIdx.y;  // together and share K/V through L2
  const int c = blockIdx.z;
  const int kvh = c % a.hkv, b = c / a.hkv;
  const int H = a.hkv * G;

  // ---- geometry
  const int ntok = (int)min((int64_t)128, a.Tq - (int64_t)blk * 128);
  const int gn = a.prefill ? 1 : max(1, min(G, 128 / ntok));
  const int g0 = g_fast * gn;
  const int n_rows = min(gn, G - g0) * ntok;
  int L0, L1, len_before;
  const bf16 *k0, *v0, *k1, *v1, *sk = nullptr, *sv = nullptr;
  bool has_sinks, has_bank;
  int64_t bank_idx = 0;
  if (a.prefill) {
    const int64_t base = (int64_t)c * a.seg0_chain_tokens;
    L0 = blk >= 1 ? CC : 0;
    L1 = ntok;
    len_before = 0;
    k0 = reinterpret_cast<const bf16*>(a.seg0_k) + (base + (int64_t)max(blk - 1, 0) * CC) * HD;
    v0 = reinterpret_cast<const bf16*>(a.seg0_v) + (base + (int64_t)max(blk - 1, 0) * CC) * HD;
    k1 = reinterpret_cast<const bf16*>(a.seg1_k) + (base + (int64_t)blk * CC) * HD;
    v1 = reinterpret_cast<const bf16*>(a.seg1_v) + (base + (int64_t)blk * CC) * HD;
    has_sinks = has_bank = blk >= 2;
    sk = reinterpret_cast<const bf16*>(a.seg0_k) + base * HD;
    sv = reinterpret_cast<const bf16*>(a.seg0_v) + base * HD;
    bank_idx = blk - 2;
  } else {
    L0 = a.seg0_len;
    L1 = a.seg1_len;
    len_before = a.len_before;
    k0 = reinterpret_cast<const bf16*>(a.seg0_k) + (int64_t)c * a.seg0_chain_tokens * HD;
    v0 = reinterpret_cast<const bf16*>(a.seg0_v) + (int64_t)c * a.seg0_chain_tokens * HD;
    k1 = reinterpret_cast<const bf16*>(a.seg1_k) + (int64_t)c * a.seg1_chain_tokens * HD;
    v1 = reinterpret_cast<const bf16*>(a.seg1_v) + (int64_t)c * a.seg1_chain_tokens * HD;
    has_sinks = a.has_sinks != 0;
    has_bank = a.has_bank != 0;
    if (has_sinks) {
      sk = reinterpret_cast<const bf16*>(a.sink_k) + (int64_t)c * a.sink_chain_tokens * HD;
      sv = reinterpret_cast<const bf16*>(a.sink_v) + (int64_t)c * a.sink_chain_tokens * HD;
    }
  }
  const int64_t bofs = (int64_t)c * a.bank_cap + bank_idx;
  const bf16* bk = has_bank ? reinterpret_cast<const bf16*>(a.bank_ak_rope) + bofs * S * HD : nullptr;
  const bf16* bv = has_bank ? reinterpret_cast<const bf16*>(a.bank_av) + bofs * S * HD : nullptr;
  const bool seg_on[3] = {has_bank, L0 > 0, L1 > 0};
  const int seg_len[3] = {S, L0, L1};
  const bf16* seg_k[3] = {bk, k0, k1};
  const bf16* seg_v[3] = {bv, v0, v1};

  auto row_tok = [&](int r, int& g, int& i) {
    g = g0 + r / ntok;
    i = r % ntok;
  };
  auto q_row_ptr = [&](const void* base, int r) {
    int g, i;
    row_tok(r < n_rows ? r : 0, g, i);
    return reinterpret_cast<const bf16*>(base) + (((int64_t)c * G + g) * a.Tq + (int64_t)blk * 128 + i) * HD;
  };

  // ---- stage 1: Q (q_rope), K tiles, sinks, attractor bias
  {
    constexpr int CPR = HD / 8;
    for (int i = tid; i < 128 * CPR; i += NT) {
      const int r = i / CPR, ch = i % CPR;
      unsigned char* d = sm.q[ch >> 3] + r * 128 + (((ch & 7) ^ (r & 7)) << 4);
      cp_async16(d, q_row_ptr(a.q_rope, r) + ch * 8, r < n_rows);
    }
    for (int s = 0; s < 3; ++s) {
      if (!seg_on[s]) continue;
      if (s == 0 && a.prefill) copy_image<HD>(sm.kv[0], seg_k[0], tid, NT);
      else load_tile<HD>(sm.kv[s], seg_k[s], seg_len[s], tid, NT);
    }
    if (has_sinks) {
      for (int i = tid; i < 4 * HD / 8; i += NT) {
        cp_async16(&sm.sink_k[0][0] + i * 8, sk + i * 8, true);
        cp_async16(&sm.sink_v[0][0] + i * 8, sv + i * 8, true);
      }
    }
    cp_async_commit();
    if (has_bank)
      for (int i = tid; i < HD; i += NT) sm.res_w[i] = a.res_w[i];
    if (has_bank) {
      const float kappa = a.kappa[kvh];
      for (int s = tid; s < S; s += NT)
        sm.bias[s] = a.bank_act[bofs * S + s] ? __fmul_rn(kappa, logf(fmaxf(a.bank_mass[bofs * S + s], 1.0f)))
                                              : neg_inf();
    }
  }
  if (warp == 0) {
    tc5::tmem_alloc(&sm.tbase, 512);
    tc5::tmem_relinquish();
  }
  if (tid == 0) {
    tc5::mbar_init(&sm.bar_s, 1);
    tc5::mbar_init(&sm.bar_o, 1);
    tc5::mbar_fence_init();
    sm.err = 0;
  }
  cp_async_wait<0>();
  asm volatile("fence.proxy.async.shared::cta;\n" ::);
  tc5::fence_before_sync();
  __syncthreads();
  tc5::fence_after_sync();
  const uint32_t tb = sm.tbase;

  // ---- stage 2: S = Q K^T for every present segment
  constexpr uint32_t kIdS = tc5::idesc_bf16(128, 128, false, false);
  if (tid == 0) {
    const uint32_t qa = tc5::smem_u32(sm.q[0]);
    for (int s = 0; s < 3; ++s) {
      if (!seg_on[s]) continue;
      const uint32_t ka = tc5::smem_u32(sm.kv[s][0]);
      for (int ks = 0; ks < HD / 16; ++ks) {
        const uint32_t off = (ks >> 2) * 16384 + (ks & 3) * 32;
        tc5::mma_ss(tb + s * 128, tc5::sdesc(qa + off, 16, 1024), tc5::sdesc(ka + off, 16, 1024), kIdS, ks > 0);
      }
    }
    tc5::commit(&sm.bar_s);
  }

  constexpr float scale = HD == 128 ? 0.08838834764831845f : 0.125f;  // fp32(HD ** -0.5)
  constexpr float kLog2e = 1.4426950408889634f;
  // Both warpgroups work on every query row r (= TMEM lane): warpgroup wg takes columns
  // [wg*64, wg*64+64) of each key segment and [wg*HD/2, (wg+1)*HD/2) of the output.
  const int wg = warp >> 2;
  const int r = tid & 127;
  const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
  int gr, ir;
  row_tok(min(r, max(n_rows - 1, 0)), gr, ir);
  const int lim1 = len_before + ir;  // current-chunk key j is visible iff j <= lim1

  if (wg == 1) {
    // ---- warpgroup 1 prologue: the M_res operand and the sink scores
    if (has_bank && a.prefill) {
      // the consolidation scan wrote the split, swizzled operand image: copy it as is
      const unsigned char* img = reinterpret_cast<const unsigned char*>(a.bank_m) + bofs * (int64_t)HD * HD * 4;
      for (int i = r; i < HD * HD / 4; i += 128) cp_async16(&sm.m[0][0][0] + i * 16, img + i * 16, true);
      cp_async_commit();
    } else if (has_bank) {
      // M_res [d][e] fp32 row-major: split into bf16 hi/lo in the MN-major operand layout (rows d,
      // 64-column blocks of e); coalesced float4 loads, eight in flight per thread
      const float4* gm = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.bank_m) + bofs * HD * HD);
      constexpr int N4 = HD * HD / 4;
      for (int i0 = r; i0 < N4; i0 += 128 * 8) {
        float4 mv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) mv[u] = i0 + u * 128 < N4 ? gm[i0 + u * 128] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int i = i0 + u * 128;
          if (i >= N4) break;
          const int d = (i * 4) / HD, e = (i * 4) % HD;
          const float v4[4] = {mv[u].x, mv[u].y, mv[u].z, mv[u].w};
          uint32_t hi[2], lo[2];
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const bf16 h0 = __float2bfloat16_rn(v4[2 * q]), h1 = __float2bfloat16_rn(v4[2 * q + 1]);
            hi[q] = pack_bf16(bf2f(h0), bf2f(h1));
            lo[q] = pack_bf16(v4[2 * q] - bf2f(h0), v4[2 * q + 1] - bf2f(h1));
          }
          const uint32_t off = tc5::sw128_off(d, e & 63);
          *reinterpret_cast<uint2*>(sm.m[0][e >> 6] + off) = make_uint2(hi[0], hi[1]);
          *reinterpret_cast<uint2*>(sm.m[1][e >> 6] + off) = make_uint2(lo[0], lo[1]);
        }
      }
    }
    if (has_sinks) {
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      for (int ch = 0; ch < HD / 8; ++ch) {
        const uint4 qv = *reinterpret_cast<const uint4*>(sm.q[ch >> 3] + r * 128 + (((ch & 7) ^ (r & 7)) << 4));
        const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float2 qf = unpack_bf16(qw[u]);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 kf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&sm.sink_k[j][ch * 8 + 2 * u]));
            acc[j] = fmaf(qf.x, kf.x, acc[j]);
            acc[j] = fmaf(qf.y, kf.y, acc[j]);
          }
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) sm.sink_s[r][j] = __fmul_rn(acc[j], scale);
      for (int i = r; i < 4 * HD; i += 128) sm.sink_vf[i / HD][i % HD] = bf2f(sm.sink_v[i / HD][i % HD]);
    }
    asm volatile("bar.sync 2, 128;\n" ::);   // warpgroup 1 is done reading Q
    asm volatile("bar.arrive 1, 256;\n" ::); // sink scores are ready
  } else {
    asm volatile("bar.sync 1, 256;\n" ::);
  }
  float s_sink[4] = {neg_inf(), neg_inf(), neg_inf(), neg_inf()};
  if (has_sinks) {
#pragma unroll
    for (int j = 0; j < 4; ++j) s_sink[j] = sm.sink_s[r][j];
  }
  const bool ok = tc5::mbar_wait(&sm.bar_s, 0, kWaitIters);
  if (!ok) sm.err = 1;
  tc5::fence_after_sync();
  if (wg == 1 && ok) {
    // K tiles are consumed: stream V (and q_raw for the read-out) in behind them
    for (int s2 = 0; s2 < 3; ++s2) {
      if (!seg_on[s2]) continue;
      if (s2 == 0 && a.prefill) copy_image<HD>(sm.kv[0], seg_v[0], r, 128);
      else load_tile<HD>(sm.kv[s2], seg_v[s2], seg_len[s2], r, 128);
    }
    if (has_bank) {
      constexpr int CPR = HD / 8;
      for (int i = r; i < 128 * CPR; i += 128) {
        const int rr = i / CPR, ch = i % CPR;
        unsigned char* d = sm.q[ch >> 3] + rr * 128 + (((ch & 7) ^ (rr & 7)) << 4);
        cp_async16(d, q_row_ptr(a.q_raw, rr) + ch * 8, rr < n_rows);
      }
    }
    cp_async_commit();
  }

  // ---- softmax over this warpgroup's half of every segment
  const float* bias = sm.bias;
  auto row_pass = [&](auto seg_tag, auto&& body) {
    constexpr int SEG = decltype(seg_tag)::value;
    const int lim = SEG == 1 ? L0 - 1 : (SEG == 2 ? min(L1 - 1, lim1) : S - 1);
    for (int c0 = wg * 64; c0 < wg * 64 + 64; c0 += 32) {
      uint32_t v[32];
      tc5::ld32(tb + lane_off + SEG * 128 + c0, v);
      tc5::ld_wait();
      float x[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float sc = __fmul_rn(__uint_as_float(v[j]), scale);
        if (SEG == 0) x[j] = __fadd_rn(sc, bias[c0 + j]);
        else x[j] = (c0 + j <= lim) ? sc : neg_inf();
      }
      body(c0, x);
    }
  };
  auto for_each_seg = [&](auto&& body) {
    if (seg_on[0]) row_pass(std::integral_constant<int, 0>{}, [&](int c0, float (&x)[32]) { body(0, c0, x); });
    if (seg_on[1]) row_pass(std::integral_constant<int, 1>{}, [&](int c0, float (&x)[32]) { body(1, c0, x); });
    if (seg_on[2]) row_pass(std::integral_constant<int, 2>{}, [&](int c0, float (&x)[32]) { body(2, c0, x); });
  };
  // pass 1: row max (the sinks are counted by warpgroup 0)
  float mx = wg == 0 ? fmaxf(fmaxf(s_sink[0], s_sink[1]), fmaxf(s_sink[2], s_sink[3])) : neg_inf();
  if (ok) {
    for_each_seg([&](int, int, float (&x)[32]) {
#pragma unroll
      for (int j = 0; j < 32; ++j) mx = fmaxf(mx, x[j]);
    });
  }
  sm.red_max[wg][r] = mx;
  asm volatile("bar.sync 3, 256;\n" ::);
  mx = fmaxf(sm.red_max[0][r], sm.red_max[1][r]);
  // pass 2: row sum of exp(x - max); exp via exp2 of (x - max) * log2(e), within ~1e-6 relative
  float e_sink[4];
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    e_sink[j] = s_sink[j] == neg_inf() ? 0.f : expf(s_sink[j] - mx);
    if (wg == 0) sum += e_sink[j];
  }
  if (ok) {
    float part[4] = {0.f, 0.f, 0.f, 0.f};
    for_each_seg([&](int, int, float (&x)[32]) {
#pragma unroll
      for (int j = 0; j < 32; ++j) part[j & 3] += exp2f(__fmul_rn(x[j] - mx, kLog2e));
    });
    sum += (part[0] + part[1]) + (part[2] + part[3]);
  }
  sm.red_sum[wg][r] = sum;
  asm volatile("bar.sync 3, 256;\n" ::);
  sum = sm.red_sum[0][r] + sm.red_sum[1][r];
  // pass 3: p = bf16(exp(x - max) * (1 / sum)), two per column, into TMEM columns [0, 192); the
  // bf16 cast matches the reference's except within ~1e-6 of a rounding boundary. P of segment s
  // lands on score columns of earlier segments that either warpgroup may still be reading, so each
  // segment's P is written only after both warpgroups have read that segment's scores.
  const float inv_sum = 1.0f / sum;
  auto p_pass = [&](auto seg_tag) {
    constexpr int SEG = decltype(seg_tag)::value;
    uint32_t pk[2][16];
    int half = 0;
    if (ok) {
      row_pass(seg_tag, [&](int, float (&x)[32]) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float e0 = exp2f(__fmul_rn(x[2 * j] - mx, kLog2e));
          const float e1 = exp2f(__fmul_rn(x[2 * j + 1] - mx, kLog2e));
          pk[half][j] = pack_bf16(__fmul_rn(e0, inv_sum), __fmul_rn(e1, inv_sum));
        }
        ++half;
      });
    }
    asm volatile("bar.sync 3, 256;\n" ::);
    if (ok) {
      tc5::st16(tb + lane_off + (uint32_t)(SEG * 64 + wg * 32), pk[0]);
      tc5::st16(tb + lane_off + (uint32_t)(SEG * 64 + wg * 32 + 16), pk[1]);
    }
  };
  if (seg_on[0]) p_pass(std::integral_constant<int, 0>{});
  if (seg_on[1]) p_pass(std::integral_constant<int, 1>{});
  if (seg_on[2]) p_pass(std::integral_constant<int, 2>{});
  if (ok) tc5::st_wait();
  float p_sink[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) p_sink[j] = rbf(__fmul_rn(e_sink[j], inv_sum));
  if (wg == 1) {
    cp_async_wait<0>();
    asm volatile("fence.proxy.async.shared::cta;\n" ::);
  }
  tc5::fence_before_sync();
  __syncthreads();
  tc5::fence_after_sync();
  const bool ok_all = sm.err == 0;

  // ---- stage 3: O = P V; R = q_raw (M_hi + M_lo)
  if (tid == 0 && ok_all) {
    constexpr uint32_t kIdO = tc5::idesc_bf16(128, HD, false, true);
    bool first = true;
    for (int s2 = 0; s2 < 3; ++s2) {
      if (!seg_on[s2]) continue;
      const uint32_t va = tc5::smem_u32(sm.kv[s2][0]);
      for (int ks = 0; ks < 8; ++ks) {
        tc5::mma_ts(tb + kColO, tb + (uint32_t)(s2 * 64 + ks * 8), tc5::sdesc(va + ks * 2048, 16384, 1024), kIdO,
                    first ? 0u : 1u);
        first = false;
      }
    }
    if (has_bank) {
      constexpr uint32_t kIdR = tc5::idesc_bf16(128, HD, false, true);
      const uint32_t qa = tc5::smem_u32(sm.q[0]);
      for (int hl = 0; hl < 2; ++hl) {
        const uint32_t ma = tc5::smem_u32(sm.m[hl][0]);
        for (int ks = 0; ks < HD / 16; ++ks) {
          const uint32_t qo = (ks >> 2) * 16384 + (ks & 3) * 32;
          tc5::mma_ss(tb + kColR, tc5::sdesc(qa + qo, 16, 1024), tc5::sdesc(ma + ks * 2048, HD * 128, 1024), kIdR,
                      (hl | ks) ? 1u : 0u);
        }
      }
    }
    tc5::commit(&sm.bar_o);
  }

  // ---- epilogue: warpgroup wg writes columns [wg*HD/2, (wg+1)*HD/2) of row r
  {
    constexpr int HALF = HD / 2;
    const int cbeg = wg * HALF;
    float qn = 0.f;
    if (has_bank && a.q_l2 != nullptr) {
      qn = a.q_l2[((int64_t)c * G + gr) * a.Tq + (int64_t)blk * 128 + ir];
    } else if (has_bank) {
      float acc = 0.f;
      for (int ch = 0; ch < HD / 8; ++ch) {
        const uint4 qv = *reinterpret_cast<const uint4*>(sm.q[ch >> 3] + r * 128 + (((ch & 7) ^ (r & 7)) << 4));
        const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float2 f = unpack_bf16(qw[u]);
          acc = fmaf(f.x, f.x, fmaf(f.y, f.y, acc));
        }
      }
      qn = sqrtf(acc);
    }
    const float eta = has_bank ? a.eta[((int64_t)c * G + gr) * a.Tq + (int64_t)blk * 128 + ir] : 0.f;
    const float coef = has_bank ? a.coef[kvh] : 0.f;
    const bool ok2 = ok_all && tc5::mbar_wait(&sm.bar_o, 0, kWaitIters);
    if (!ok2 && ok_all) sm.err = 1;
    tc5::fence_after_sync();
    const float inv_qn = 1.0f / fmaxf(qn, 1e-12f);
    float ss = 0.f;
    if (ok2 && has_bank) {
      for (int c0 = cbeg; c0 < cbeg + HALF; c0 += 32) {
        uint32_t v[32];
        tc5::ld32(tb + lane_off + kColR + c0, v);
        tc5::ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float ym = __fmul_rn(__fmul_rn(__uint_as_float(v[j]), inv_qn), coef);
          ss = fmaf(ym, ym, ss);
        }
      }
    }
    sm.red_max[wg][r] = ss;
    asm volatile("bar.sync 3, 256;\n" ::);
    const float rs = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(sm.red_max[0][r] + sm.red_max[1][r], (float)HD), a.eps));
    if (ok2) {
      bf16* yrow = reinterpret_cast<bf16*>(a.y) +
                   (((int64_t)b * a.y_tokens + (int64_t)blk * 128 + ir) * H + kvh * G + gr) * HD;
      for (int c0 = cbeg; c0 < cbeg + HALF; c0 += 32) {
        uint32_t vo[32], vr[32];
        tc5::ld32(tb + lane_off + kColO + c0, vo);
        if (has_bank) tc5::ld32(tb + lane_off + kColR + c0, vr);
        tc5::ld_wait();
        uint32_t packed[16];
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          float o2[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int col = c0 + j + u;
            float o = __uint_as_float(vo[j + u]);
            if (has_sinks) {
#pragma unroll
              for (int q = 0; q < 4; ++q) o = fmaf(p_sink[q], sm.sink_vf[q][col], o);
            }
            o = rbf(o);
            if (has_bank) {
              const float ym = __fmul_rn(__fmul_rn(__uint_as_float(vr[j + u]), inv_qn), coef);
              o = rbf(__fadd_rn(o, rbf(__fmul_rn(eta, __fmul_rn(__fmul_rn(ym, rs), sm.res_w[col])))));
            }
            o2[u] = o;
          }
          packed[j >> 1] = pack_bf16(o2[0], o2[1]);
        }
        if (r < n_rows) {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            *reinterpret_cast<uint4*>(yrow + c0 + q * 8) =
                make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
        }
      }
    }
    tc5::fence_before_sync();
  }
  __syncthreads();
  tc5::fence_after_sync();
  if (warp == 0) tc5::tmem_dealloc(tb, 512);
  if (tid == 0 && sm.err && a.status) atomicOr(a.status, 2);
}

}  // namespace

extern "C" int bolt3_attend(const bolt3_attend_args* a, void* stream) {
  if (!a || !a->q_rope || !a->q_raw || !a->eta || !a->y || !a->kappa || !a->seg0_k || !a->seg0_v ||
      !a->seg1_k || !a->seg1_v)
    return BOLT3_ERR_ARG;
  if (a->n_chains <= 0 || a->n_chains > 65535 || a->hkv <= 0 || a->G <= 0 || a->G > 16 || a->Tq <= 0)
    return BOLT3_ERR_SHAPE;
  // the bank (and the read-out epilogue) is read by decode calls with has_bank, and by prefill
  // calls whose sequence has a third chunk
  const bool uses_bank = a->prefill ? a->Tq > 2 * CC : a->has_bank != 0;
  if (uses_bank && (!a->coef || !a->res_w || !a->bank_ak_rope || !a->bank_av || !a->bank_mass ||
                    !a->bank_act || !a->bank_m))
    return BOLT3_ERR_ARG;
  if (!a->prefill) {
    if (a->Tq > 128 || a->seg0_len < 0 || a->seg0_len > CC || a->seg1_len <= 0 || a->seg1_len > CC ||
        a->len_before < 0 || a->len_before + a->Tq != a->seg1_len)
      return BOLT3_ERR_SHAPE;
    if (a->has_sinks && (!a->sink_k || !a->sink_v)) return BOLT3_ERR_ARG;
  } else if (a->seg0_chain_tokens < a->Tq) {
    return BOLT3_ERR_CAPACITY;
  }
  const uintptr_t al = (uintptr_t)a->q_rope | (uintptr_t)a->q_raw | (uintptr_t)a->seg0_k | (uintptr_t)a->seg0_v |
                       (uintptr_t)a->seg1_k | (uintptr_t)a->seg1_v | (uintptr_t)a->sink_k |
                       (uintptr_t)a->sink_v | (uintptr_t)a->bank_ak_rope | (uintptr_t)a->bank_av |
                       (uintptr_t)a->bank_m | (uintptr_t)a->y;
  if (al & 15) return BOLT3_ERR_ALIGN;
  cudaStream_t s = (cudaStream_t)stream;
  dim3 grid;
  if (a->prefill) {
    const int64_t n_blk = (a->Tq + 127) / 128;
    const int64_t count = a->blk_count > 0 ? a->blk_count : n_blk - a->blk_begin;
    if (a->blk_begin < 0 || count <= 0 || a->blk_begin + count > n_blk) return BOLT3_ERR_SHAPE;
    grid = dim3((unsigned)a->G, (unsigned)count, (unsigned)a->n_chains);
  } else {
    const int gn = (int)std::max<int64_t>(1, std::min<int64_t>(a->G, 128 / a->Tq));
    grid = dim3((unsigned)((a->G + gn - 1) / gn), 1, (unsigned)a->n_chains);
  }
  // Each CTA allocates all 512 TMEM columns, so the shared-memory request keeps one CTA per SM.
  constexpr size_t kMinSmem = 120 * 1024;
  if (a->HD == 128) {
    const size_t smem = std::max(sizeof(Smem<128>) + 1024, kMinSmem);
    if (cudaFuncSetAttribute(attend_tc_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return BOLT3_ERR_CUDA;
    attend_tc_kernel<128><<<grid, NT, smem, s>>>(*a);
  } else if (a->HD == 64) {
    const size_t smem = std::max(sizeof(Smem<64>) + 1024, kMinSmem);
    if (cudaFuncSetAttribute(attend_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return BOLT3_ERR_CUDA;
    attend_tc_kernel<64><<<grid, NT, smem, s>>>(*a);
  } else {
    return BOLT3_ERR_SHAPE;
  }
  return cudaGetLastError() == cudaSuccess ? BOLT3_OK : BOLT3_ERR_CUDA;
}
