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
// [previous chunk] [current chunk, causal] (vsa_lm/config/bolt3.py:219-249). Every product is a
// tcgen05.mma with bf16 operands in 128-byte swizzled shared memory and fp32 accumulation; the 4
// sinks are a 16-row key tile (rows 4..15 zero and masked) whose scores land in TMEM columns
// [384, 400) before O is written there, and whose probabilities (columns [320, 328)) add one K step
// to the P@V product. Probabilities are normalised before their bf16 cast exactly
// as the reference does (F.softmax(...).to(dtype), bolt3.py:249). The epilogue reads M_res out
// (bolt3.py:251-256): y = bf16( bf16(P@V) + bf16( eta * RMSNorm_w( q_raw @ (M_hi + M_lo) / |q_raw|
// * (1-gamma)/sqrt(HD) ) ) ), with M split into two bf16 terms.
//
// All four warpgroups handle every query row (TMEM lane = row), each on a quarter of the columns,
// and swap row max / sum / RMS partials through shared memory. Thread 0 issues the MMAs. Prefill tiles arrive
// by TMA, issued by thread 0: Q and K tiles (3-D tensor maps, 128-byte swizzle, rows past the end of
// a sequence zero-filled), the scan's snapshot images as plain bulk copies, and V / q_raw into the
// K / Q tiles once the score MMAs have consumed them. Decode tiles (ring buffers) are gathered with
// cp.async by every thread, and warpgroup 1 converts the fp32 M_res into the split operand.
#include "../../include/bolt3.h"
#include "common.cuh"
#include "trace.h"
#include "tc5.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <type_traits>

namespace {

using namespace b3;

constexpr int S = 128;
constexpr int CC = 128;
constexpr int NT = 512;
constexpr int NWG = NT / 128;  // warpgroups; each covers all 128 query rows (TMEM lanes)
constexpr int CW = 128 / NWG;  // score columns per segment handled by one warpgroup
static_assert(CW == 32, "one 32-column TMEM chunk per segment and warpgroup");
constexpr uint32_t kWaitIters = 1u << 24;
constexpr uint32_t kColO = 384, kColR = 192, kColPSink = 320;
constexpr float kLog2e = 1.4426950408889634f;

// 2^x on the special-function unit (relative error ~2^-22; results below 2^-126 flush to zero)
B3_DEV float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

template <int HD>
struct __align__(1024) Smem {
  unsigned char q[HD / 64][16384];        // q_rope tile, then the q_raw tile (K-major SW128)
  unsigned char kv[3][HD / 64][16384];    // K tiles of attractors / prev / cur, then their V tiles
  unsigned char m[2][HD / 64][HD * 128];  // M_res hi / lo (MN-major B): rows = input dim d, N blocks of e
  unsigned char sink_k[HD / 64][2048];  // the 4 sink keys as a 16-row K-major tile, rows 4..15 zero
  unsigned char sink_v[HD / 64][2048];  // the 4 sink values as the 16-key B tile of P@V
  float res_w[HD];
  float red_max[NWG][128];  // per-row partial results exchanged between the warpgroups
  float red_sum[NWG][128];
  float bias[S];
  uint64_t bar_s, bar_o, bar_r;
  uint64_t bar_k, bar_v, bar_m;   // TMA completion: Q + K tiles, V + q_raw tiles, M_res image
  uint32_t tbase;
  int err;
};

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

// Tensor maps of the prefill operands: 3-D {HD, tokens, heads or chains}, box {64, 128, 1}, bf16,
// 128-byte swizzle.
struct __align__(64) AttendMaps {
  CUtensorMap q_rope, q_raw, k0, v0, k1, v1;
};

// PREFILL selects the prefill geometry and the TMA loads at compile time (a.prefill must agree), so
// that each instantiation carries only its own path's code
template <int HD, bool PREFILL>
__global__ void __launch_bounds__(NT, 1) attend_tc_kernel(const bolt3_attend_args a,
                                                          const __grid_constant__ AttendMaps tm) {
  extern __shared__ unsigned char smem_raw[];
  Smem<HD>& sm = *reinterpret_cast<Smem<HD>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5;
  if (a.wait_probe) {  // failure-path test hook: an expired bounded wait, reported as bit 2
    if (tid == 0 && !tc5::probe_wait(&sm.bar_s, a.wait_probe) && a.status) atomicOr(a.status, 2);
    return;
  }
  const int G = a.G;
  const int g_fast = blockIdx.x;  // head group within the KV head: the G CTAs of one chain-chunk run
  const int blk = (int)a.blk_begin + blockIdx.y;  // together and share K/V through L2
  const int c = blockIdx.z;
  const int kvh = c % a.hkv, b = c / a.hkv;
  const int H = a.hkv * G;

  // ---- geometry
  const int ntok = (int)min((int64_t)128, a.Tq - (int64_t)blk * 128);
  const int gn = PREFILL ? 1 : max(1, min(G, 128 / ntok));
  const int g0 = g_fast * gn;
  const int n_rows = min(gn, G - g0) * ntok;
  int L0, L1, len_before;
  const bf16 *k0, *v0, *k1, *v1, *sk = nullptr, *sv = nullptr;
  bool has_sinks, has_bank;
  int64_t bank_idx = 0;
  if constexpr (PREFILL) {
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
  constexpr bool use_tma = PREFILL;
  constexpr uint32_t kTileBytes = 128 * HD * 2;
  if (tid == 0) {
    tc5::mbar_init(&sm.bar_s, 1);
    tc5::mbar_init(&sm.bar_o, 1);
    tc5::mbar_init(&sm.bar_r, 1);
    tc5::mbar_init(&sm.bar_k, 1);
    tc5::mbar_init(&sm.bar_v, 1);
    tc5::mbar_init(&sm.bar_m, 1);
    tc5::mbar_fence_init();
    sm.err = 0;
    if (use_tma) {
      const int zq = c * G + g0;
      tc5::mbar_expect_tx(&sm.bar_k, kTileBytes * (1 + seg_on[0] + seg_on[1] + seg_on[2]));
      for (int h2 = 0; h2 < HD / 64; ++h2) tc5::tma_load_3d(sm.q[h2], &tm.q_rope, h2 * 64, blk * 128, zq, &sm.bar_k);
      if (seg_on[0]) tc5::bulk_load(sm.kv[0][0], seg_k[0], kTileBytes, &sm.bar_k);
      if (seg_on[1])
        for (int h2 = 0; h2 < HD / 64; ++h2) tc5::tma_load_3d(sm.kv[1][h2], &tm.k0, h2 * 64, (blk - 1) * 128, c, &sm.bar_k);
      for (int h2 = 0; h2 < HD / 64; ++h2) tc5::tma_load_3d(sm.kv[2][h2], &tm.k1, h2 * 64, blk * 128, c, &sm.bar_k);
      if (has_bank) {
        tc5::mbar_expect_tx(&sm.bar_m, HD * HD * 4);
        tc5::bulk_load(sm.m[0][0], reinterpret_cast<const unsigned char*>(a.bank_m) + bofs * (int64_t)HD * HD * 4,
                       HD * HD * 4, &sm.bar_m);
      }
    }
  }
  {
    constexpr int CPR = HD / 8;
    if (!use_tma) {
      for (int i = tid; i < 128 * CPR; i += NT) {
        const int r = i / CPR, ch = i % CPR;
        unsigned char* d = sm.q[ch >> 3] + r * 128 + (((ch & 7) ^ (r & 7)) << 4);
        cp_async16(d, q_row_ptr(a.q_rope, r) + ch * 8, r < n_rows);
      }
      for (int s = 0; s < 3; ++s)
        if (seg_on[s]) load_tile<HD>(sm.kv[s], seg_k[s], seg_len[s], tid, NT);
    }
    if (has_sinks) {
      constexpr int CPR = HD / 8;
      for (int i = tid; i < 16 * CPR; i += NT) {
        const int rr = i / CPR, ch = i % CPR;
        const uint32_t off = (ch >> 3) * 2048 + rr * 128 + (((ch & 7) ^ (rr & 7)) << 4);
        if (rr < 4) {
          cp_async16(&sm.sink_k[0][0] + off, sk + rr * HD + ch * 8, true);
          cp_async16(&sm.sink_v[0][0] + off, sv + rr * HD + ch * 8, true);
        } else {
          *reinterpret_cast<uint4*>(&sm.sink_k[0][0] + off) = make_uint4(0, 0, 0, 0);
          *reinterpret_cast<uint4*>(&sm.sink_v[0][0] + off) = make_uint4(0, 0, 0, 0);
        }
      }
    }
    cp_async_commit();
    if (has_bank)
      for (int i = tid; i < HD; i += NT) sm.res_w[i] = a.res_w[i];
    if (has_bank) {
      const float kappa = a.kappa[kvh];
      for (int s = tid; s < S; s += NT)
        sm.bias[s] = a.bank_act[bofs * S + s]
                         ? __fmul_rn(__fmul_rn(kappa, logf(fmaxf(a.bank_mass[bofs * S + s], 1.0f))), kLog2e)
                         : neg_inf();
    }
  }
  if (warp == 0) {
    tc5::tmem_alloc(&sm.tbase, 512);
    tc5::tmem_relinquish();
  }
  cp_async_wait<0>();
  asm volatile("fence.proxy.async.shared::cta;\n" ::);
  tc5::fence_before_sync();
  __syncthreads();
  tc5::fence_after_sync();
  const uint32_t tb = sm.tbase;

  // ---- stage 2: S = Q K^T for every present segment
  constexpr uint32_t kIdS = tc5::idesc_bf16(128, 128, false, false);
  // thread 0 tracks which TMA groups it has seen complete, so that it never leaves with copies in flight
  bool seen_k = !use_tma, seen_v = true, seen_m = !(use_tma && has_bank);
  if (tid == 0 && !seen_k) {
    seen_k = tc5::mbar_wait(&sm.bar_k, 0, kWaitIters);
    if (!seen_k) sm.err = 1;
  }
  if (tid == 0) {
    const uint32_t qa = tc5::smem_u32(sm.q[0]);
    for (int s = 0; s < 3; ++s) {
      if (!seg_on[s] || !seen_k) continue;
      const uint32_t ka = tc5::smem_u32(sm.kv[s][0]);
      for (int ks = 0; ks < HD / 16; ++ks) {
        const uint32_t off = (ks >> 2) * 16384 + (ks & 3) * 32;
        tc5::mma_ss(tb + s * 128, tc5::sdesc(qa + off, 16, 1024), tc5::sdesc(ka + off, 16, 1024), kIdS, ks > 0);
      }
    }
    if (has_sinks && seen_k) {
      constexpr uint32_t kIdSink = tc5::idesc_bf16(128, 16, false, false);
      const uint32_t sa = tc5::smem_u32(sm.sink_k[0]);
      for (int ks = 0; ks < HD / 16; ++ks) {
        const uint32_t qo = (ks >> 2) * 16384 + (ks & 3) * 32, so = (ks >> 2) * 2048 + (ks & 3) * 32;
        tc5::mma_ss(tb + kColO, tc5::sdesc(qa + qo, 16, 1024), tc5::sdesc(sa + so, 16, 1024), kIdSink, ks > 0);
      }
    }
    tc5::commit(&sm.bar_s);
  }

  // Every warpgroup works on every query row r (= TMEM lane): warpgroup wg takes columns
  // [wg*CW, wg*CW+CW) of each key segment and [wg*HD/NWG, (wg+1)*HD/NWG) of the output.
  const int wg = warp >> 2;
  const int r = tid & 127;
  const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
  int gr, ir;
  row_tok(min(r, max(n_rows - 1, 0)), gr, ir);
  const int lim1 = len_before + ir;  // current-chunk key j is visible iff j <= lim1

  if (wg == 1) {
    // ---- warpgroup 1 prologue (decode): the M_res operand
    if (has_bank && !use_tma) {
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
  }
  const bool ok = tc5::mbar_wait(&sm.bar_s, 0, kWaitIters);
  if (!ok) sm.err = 1;
  tc5::fence_after_sync();
  // K tiles are consumed: stream V (and q_raw for the read-out) in behind them
  if (use_tma && tid == 0 && ok && seen_k) {
    seen_v = false;
    tc5::mbar_expect_tx(&sm.bar_v, kTileBytes * (seg_on[0] + seg_on[1] + seg_on[2] + has_bank));
    if (seg_on[0]) tc5::bulk_load(sm.kv[0][0], seg_v[0], kTileBytes, &sm.bar_v);
    if (seg_on[1])
      for (int h2 = 0; h2 < HD / 64; ++h2) tc5::tma_load_3d(sm.kv[1][h2], &tm.v0, h2 * 64, (blk - 1) * 128, c, &sm.bar_v);
    for (int h2 = 0; h2 < HD / 64; ++h2) tc5::tma_load_3d(sm.kv[2][h2], &tm.v1, h2 * 64, blk * 128, c, &sm.bar_v);
    if (has_bank)
      for (int h2 = 0; h2 < HD / 64; ++h2) tc5::tma_load_3d(sm.q[h2], &tm.q_raw, h2 * 64, blk * 128, c * G + g0, &sm.bar_v);
  }
  if (!use_tma && wg == 1 && ok) {
    for (int s2 = 0; s2 < 3; ++s2)
      if (seg_on[s2]) load_tile<HD>(sm.kv[s2], seg_v[s2], seg_len[s2], r, 128);
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
  // The softmax runs in log2 units: t = S * (HD^-0.5 * log2 e) + bias * log2 e, p = 2^(t - max t) / sum,
  // which differs from exp(s - max s) by ~|s| * 1e-7 relative.
  constexpr float kScaleL2 = (float)((HD == 128 ? 0.08838834764831845 : 0.125) * 1.4426950408889634);
  const float* bias = sm.bias;
  // the 32 scores of this warpgroup in segment SEG: scaled, attractor bias added, masked keys -inf
  auto load_scores = [&](auto seg_tag, float (&x)[32]) {
    constexpr int SEG = decltype(seg_tag)::value;
    const int lim = SEG == 1 ? L0 - 1 : (SEG == 2 ? min(L1 - 1, lim1) : S - 1);
    const int c0 = wg * CW;
    uint32_t v[32];
    tc5::ld32(tb + lane_off + SEG * 128 + c0, v);
    tc5::ld_wait();
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (SEG == 0) x[j] = fmaf(__uint_as_float(v[j]), kScaleL2, bias[c0 + j]);
      else x[j] = (c0 + j <= lim) ? __fmul_rn(__uint_as_float(v[j]), kScaleL2) : neg_inf();
    }
  };
  // statistics pass: row max and sum of 2^(t - max) in one sweep, the sum rescaled whenever a block
  // raises the running max. Each block's 2^(t - running max) goes back to TMEM over its scores, with
  // that running max kept in mrun, so the P pass only rescales. Warpgroup 0 also counts the sinks
  // (TMEM columns [384, 388)).
  float mx = neg_inf(), sum = 0.f;
  auto stats = [&](const float (&x)[32], uint32_t (&ev)[32]) {
    float cm = x[0];
#pragma unroll
    for (int j = 1; j < 32; ++j) cm = fmaxf(cm, x[j]);
    if (cm == neg_inf()) {
#pragma unroll
      for (int j = 0; j < 32; ++j) ev[j] = 0u;
      return;
    }
    if (cm > mx) {
      sum = __fmul_rn(sum, ex2(mx - cm));
      mx = cm;
    }
    float part[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float e = ex2(x[j] - mx);
      part[j & 3] += e;
      ev[j] = __float_as_uint(e);
    }
    sum += (part[0] + part[1]) + (part[2] + part[3]);
  };
  float mrun[3] = {neg_inf(), neg_inf(), neg_inf()};
  auto stats_seg = [&](auto seg_tag) {
    constexpr int SEG = decltype(seg_tag)::value;
    float x[32];
    uint32_t ev[32];
    load_scores(seg_tag, x);
    stats(x, ev);
    mrun[SEG] = mx;
    tc5::st32(tb + lane_off + SEG * 128 + wg * CW, ev);
  };
  float s_sink[4] = {neg_inf(), neg_inf(), neg_inf(), neg_inf()};
  if (ok && has_sinks && wg == 0) {
    uint32_t v[32];
    tc5::ld32(tb + lane_off + kColO, v);
    tc5::ld_wait();
    float x[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) x[j] = neg_inf();
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] = s_sink[j] = __fmul_rn(__uint_as_float(v[j]), kScaleL2);
    stats(x, v);
  }
  if (ok) {
    if (seg_on[0]) stats_seg(std::integral_constant<int, 0>{});
    if (seg_on[1]) stats_seg(std::integral_constant<int, 1>{});
    if (seg_on[2]) stats_seg(std::integral_constant<int, 2>{});
    tc5::st_wait();
  }
  sm.red_max[wg][r] = mx;
  sm.red_sum[wg][r] = sum;
  asm volatile("bar.sync 3, %0;\n" ::"n"(NT));
  {
    mx = sm.red_max[0][r];
#pragma unroll
    for (int w = 1; w < NWG; ++w) mx = fmaxf(mx, sm.red_max[w][r]);
    sum = 0.f;
#pragma unroll
    for (int w = 0; w < NWG; ++w) sum += __fmul_rn(sm.red_sum[w][r], ex2(sm.red_max[w][r] - mx));
  }
  // P pass: p = bf16(2^(t - max) * (1 / sum)) = bf16(e * 2^(mrun - max) / sum) from the stored e,
  // two per column, into TMEM columns [0, 192); the bf16 cast matches the reference's except within
  // ~1e-6 of a rounding boundary. P of segment s lands on columns of earlier segments that another
  // warpgroup may still be reading, so each segment's P is written only after every warpgroup has
  // read that segment's values.
  const float inv_sum = 1.0f / sum;
  auto p_pass = [&](auto seg_tag) {
    constexpr int SEG = decltype(seg_tag)::value;
    uint32_t pk[16];
    if (ok) {
      uint32_t v[32];
      tc5::ld32(tb + lane_off + SEG * 128 + wg * CW, v);
      tc5::ld_wait();
      const float f = __fmul_rn(ex2(mrun[SEG] - mx), inv_sum);
#pragma unroll
      for (int j = 0; j < 16; ++j)
        pk[j] = pack_bf16(__fmul_rn(__uint_as_float(v[2 * j]), f), __fmul_rn(__uint_as_float(v[2 * j + 1]), f));
    }
    asm volatile("bar.sync 3, %0;\n" ::"n"(NT));
    if (ok) tc5::st16(tb + lane_off + (uint32_t)(SEG * 64 + wg * (CW / 2)), pk);
  };
  if (seg_on[0]) p_pass(std::integral_constant<int, 0>{});
  if (seg_on[1]) p_pass(std::integral_constant<int, 1>{});
  if (seg_on[2]) p_pass(std::integral_constant<int, 2>{});
  if (ok && has_sinks && wg == 0) {
    // sink probabilities, two per column, into columns [320, 328) (every score there has been read)
    uint32_t pk[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) pk[j] = 0u;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float e0 = ex2(s_sink[2 * j] - mx);
      const float e1 = ex2(s_sink[2 * j + 1] - mx);
      pk[j] = pack_bf16(__fmul_rn(e0, inv_sum), __fmul_rn(e1, inv_sum));
    }
    tc5::st16(tb + lane_off + kColPSink, pk);
  }
  if (ok) tc5::st_wait();
  if (wg == 1 && !use_tma) {
    cp_async_wait<0>();
    asm volatile("fence.proxy.async.shared::cta;\n" ::);
  }
  if (tid == 0 && !seen_v) {
    seen_v = tc5::mbar_wait(&sm.bar_v, 0, kWaitIters);
    if (!seen_v) sm.err = 1;
  }
  if (tid == 0 && !seen_m) {
    seen_m = tc5::mbar_wait(&sm.bar_m, 0, kWaitIters);
    if (!seen_m) sm.err = 1;
  }
  tc5::fence_before_sync();
  __syncthreads();
  tc5::fence_after_sync();
  const bool ok_all = sm.err == 0;

  // ---- stage 3: R = q_raw (M_hi + M_lo) first (the epilogue's RMS sweep overlaps P@V), then O = P V
  if (tid == 0 && ok_all) {
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
      tc5::commit(&sm.bar_r);
    }
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
    if (has_sinks) {
      tc5::mma_ts(tb + kColO, tb + kColPSink, tc5::sdesc(tc5::smem_u32(sm.sink_v[0]), 2048, 1024), kIdO,
                  first ? 0u : 1u);
      first = false;
    }
    tc5::commit(&sm.bar_o);
  }

  // ---- epilogue: warpgroup wg writes columns [wg*EW, (wg+1)*EW) of row r, EC at a time
  {
    constexpr int EW = HD / NWG;
    constexpr int EC = EW < 32 ? EW : 32;
    const int cbeg = wg * EW;
    float qn = 0.f;
    if (has_bank && a.q_l2 != nullptr) {
      qn = a.q_l2[((int64_t)c * G + gr) * a.Tq + (int64_t)blk * 128 + ir];
    } else if (has_bank && (!use_tma || tc5::mbar_wait(&sm.bar_v, 0, kWaitIters))) {
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
    const bool ok_r = ok_all && (!has_bank || tc5::mbar_wait(&sm.bar_r, 0, kWaitIters));
    if (!ok_r && ok_all) sm.err = 1;
    tc5::fence_after_sync();
    const float inv_qn = 1.0f / fmaxf(qn, 1e-12f);
    float ss = 0.f;
    if (ok_r && has_bank) {
      for (int c0 = cbeg; c0 < cbeg + EW; c0 += EC) {
        uint32_t v[EC];
        tc5::ld_cols(tb + lane_off + kColR + c0, v);
        tc5::ld_wait();
#pragma unroll
        for (int j = 0; j < EC; ++j) {
          const float ym = __fmul_rn(__fmul_rn(__uint_as_float(v[j]), inv_qn), coef);
          ss = fmaf(ym, ym, ss);
        }
      }
    }
    sm.red_max[wg][r] = ss;
    asm volatile("bar.sync 3, %0;\n" ::"n"(NT));
    float ss_all = 0.f;
#pragma unroll
    for (int w = 0; w < NWG; ++w) ss_all += sm.red_max[w][r];
    const float rs = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss_all, (float)HD), a.eps));
    const bool ok2 = ok_r && tc5::mbar_wait(&sm.bar_o, 0, kWaitIters);
    if (!ok2 && ok_r) sm.err = 1;
    tc5::fence_after_sync();
    if (ok2) {
      bf16* yrow = reinterpret_cast<bf16*>(a.y) +
                   (((int64_t)b * a.y_tokens + (int64_t)blk * 128 + ir) * H + kvh * G + gr) * HD;
      for (int c0 = cbeg; c0 < cbeg + EW; c0 += EC) {
        uint32_t vo[EC], vr[EC];
        tc5::ld_cols(tb + lane_off + kColO + c0, vo);
        if (has_bank) tc5::ld_cols(tb + lane_off + kColR + c0, vr);
        tc5::ld_wait();
        // y = bf16(bf16(O) + bf16(eta * (ym * rs) * w)), every rounding done two columns at a time
        uint32_t packed[EC / 2];
#pragma unroll
        for (int j = 0; j < EC; j += 2) {
          const float2 o = rbf2(__uint_as_float(vo[j]), __uint_as_float(vo[j + 1]), packed[j >> 1]);
          if (has_bank) {
            float t[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const float ym = __fmul_rn(__fmul_rn(__uint_as_float(vr[j + u]), inv_qn), coef);
              t[u] = __fmul_rn(eta, __fmul_rn(__fmul_rn(ym, rs), sm.res_w[c0 + j + u]));
            }
            uint32_t tmp;
            const float2 tr = rbf2(t[0], t[1], tmp);
            packed[j >> 1] = pack_bf16(__fadd_rn(o.x, tr.x), __fadd_rn(o.y, tr.y));
          }
        }
        if (r < n_rows) {
#pragma unroll
          for (int q = 0; q < EC / 8; ++q)
            *reinterpret_cast<uint4*>(yrow + c0 + q * 8) =
                make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
        }
      }
    }
    tc5::fence_before_sync();
  }
  __syncthreads();
  tc5::fence_after_sync();
  if (tid == 0) {
    // copies still in flight after a timed-out wait: give them one more bounded wait before leaving
    if (!seen_k) tc5::mbar_wait(&sm.bar_k, 0, kWaitIters);
    if (!seen_v) tc5::mbar_wait(&sm.bar_v, 0, kWaitIters);
    if (!seen_m) tc5::mbar_wait(&sm.bar_m, 0, kWaitIters);
  }
  if (warp == 0) tc5::tmem_dealloc(tb, 512);
  if (tid == 0 && sm.err && a.status) atomicOr(a.status, 2);
}

}  // namespace

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// bf16 rows [slices][rows][hd], slices `slice_stride` rows apart: box {64, box_rows, 1}, 128-byte
// swizzle; rows at or past `rows` read as zero. Also used by the decode kernels (attend_decode.cu).
bool b3_encode_bf16_rows(CUtensorMap* m, const void* base, int hd, int64_t rows, int64_t slice_stride,
                         int64_t slices, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)hd, (cuuint64_t)rows, (cuuint64_t)slices};
  const cuuint64_t strides[2] = {(cuuint64_t)hd * 2, (cuuint64_t)slice_stride * hd * 2};
  const cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// [slices][tokens][hd] bf16, box {64, 128, 1}
static bool encode_rows(CUtensorMap* m, const void* base, int hd, int64_t tokens, int64_t slices) {
  return b3_encode_bf16_rows(m, base, hd, tokens, tokens, slices, 128);
}

// decode steps with few query rows per chain (attend_decode.cu)
int b3_attend_decode_launch(const bolt3_attend_args* a, cudaStream_t s);

extern "C" int bolt3_attend(const bolt3_attend_args* a, void* stream) {
  const b3::TraceRange trace_range("bolt3_attend");
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
    // with a device step position, every size must hold for the largest shift as well
    const int64_t dmax = a->pos_dev != nullptr ? a->pos_span - 1 : 0;
    if (a->Tq > 128 || a->seg0_len < 0 || a->seg0_len > CC || a->seg1_len <= 0 || a->seg1_len + dmax > CC ||
        a->len_before < 0 || a->len_before + a->Tq != a->seg1_len)
      return BOLT3_ERR_SHAPE;
    if (a->has_sinks && (!a->sink_k || !a->sink_v)) return BOLT3_ERR_ARG;
    // only the decode kernels (at most 16 query rows per chain) read a device step position
    if (a->pos_dev != nullptr && (a->pos_span < 1 || (int64_t)a->G * a->Tq > 16)) return BOLT3_ERR_ARG;
  } else if (a->seg0_chain_tokens < a->Tq) {
    return BOLT3_ERR_CAPACITY;
  } else if (a->pos_dev != nullptr) {
    return BOLT3_ERR_ARG;
  }
  const uintptr_t al = (uintptr_t)a->q_rope | (uintptr_t)a->q_raw | (uintptr_t)a->seg0_k | (uintptr_t)a->seg0_v |
                       (uintptr_t)a->seg1_k | (uintptr_t)a->seg1_v | (uintptr_t)a->sink_k |
                       (uintptr_t)a->sink_v | (uintptr_t)a->bank_ak_rope | (uintptr_t)a->bank_av |
                       (uintptr_t)a->bank_m | (uintptr_t)a->y;
  if (al & 15) return BOLT3_ERR_ALIGN;
  cudaStream_t s = (cudaStream_t)stream;
  if (!a->prefill && (int64_t)a->G * a->Tq <= 16) return b3_attend_decode_launch(a, s);
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
  AttendMaps maps;
  memset(&maps, 0, sizeof(maps));
  if (a->prefill) {
    const int64_t nq = (int64_t)a->n_chains * a->G;
    if (!encode_rows(&maps.q_rope, a->q_rope, (int)a->HD, a->Tq, nq) ||
        !encode_rows(&maps.q_raw, a->q_raw, (int)a->HD, a->Tq, nq) ||
        !encode_rows(&maps.k0, a->seg0_k, (int)a->HD, a->seg0_chain_tokens, a->n_chains) ||
        !encode_rows(&maps.v0, a->seg0_v, (int)a->HD, a->seg0_chain_tokens, a->n_chains) ||
        !encode_rows(&maps.k1, a->seg1_k, (int)a->HD, a->seg1_chain_tokens, a->n_chains) ||
        !encode_rows(&maps.v1, a->seg1_v, (int)a->HD, a->seg1_chain_tokens, a->n_chains))
      return BOLT3_ERR_CUDA;
  }
  // Each CTA allocates all 512 TMEM columns, so the shared-memory request keeps one CTA per SM.
  constexpr size_t kMinSmem = 120 * 1024;
  if (a->HD == 128) {
    const size_t smem = std::max(sizeof(Smem<128>) + 1024, kMinSmem);
    auto kern = a->prefill ? attend_tc_kernel<128, true> : attend_tc_kernel<128, false>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return BOLT3_ERR_CUDA;
    kern<<<grid, NT, smem, s>>>(*a, maps);
  } else if (a->HD == 64) {
    const size_t smem = std::max(sizeof(Smem<64>) + 1024, kMinSmem);
    auto kern = a->prefill ? attend_tc_kernel<64, true> : attend_tc_kernel<64, false>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return BOLT3_ERR_CUDA;
    kern<<<grid, NT, smem, s>>>(*a, maps);
  } else {
    return BOLT3_ERR_SHAPE;
  }
  return cudaGetLastError() == cudaSuccess ? BOLT3_OK : BOLT3_ERR_CUDA;
}
