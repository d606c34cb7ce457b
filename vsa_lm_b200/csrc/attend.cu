// Phase C: three-field softmax attention with the fused M_res read-out epilogue.
//
// One CTA = one 128-row query tile of one chain: rows are (query head g, token i) pairs of the same
// KV head, so every key/value block loaded into shared memory serves all G query heads of the
// group (the reference materialises G copies with repeat_kv, surgery.py:96-100). Keys are visited
// block by block with an online (running-max) softmax:
//   [4 sinks] [S attractors: RoPE'd at their mean position, + kappa*log(mass), -inf if inactive]
//   [previous chunk] [current chunk, causal]                (vsa_lm/config/bolt3.py:219-249)
// The epilogue reads M_res out for the same rows (bolt3.py:251-256):
//   y = bf16( bf16(P@V) + bf16( eta * RMSNorm_w( q_raw @ (M_hi + M_lo) / |q_raw| * (1-gamma)/sqrt(HD) ) ) )
// with M split into two bf16 terms for the tensor cores.
#include "../../include/bolt3.h"
#include "common.cuh"

#include <algorithm>

namespace {

using namespace b3;

constexpr int S = 128;
constexpr int CC = 128;
constexpr int NT = 256;
constexpr int KB = 64;  // keys per block

template <int HD>
struct Smem {
  bf16 q[128 * HD];        // q_rope tile; q_raw tile in the epilogue
  bf16 k[2 * KB * HD];     // double-buffered key blocks; M_hi [HD][HD] in the epilogue
  bf16 v[2 * KB * HD];     // double-buffered value blocks; M_lo in the epilogue
  float bias[2][KB];
  float qn[128];
};

struct Job {
  const bf16* k;
  const bf16* v;
  int n;        // valid keys in this block
  int kind;     // 0 sinks, 1 attractors, 2 previous chunk, 3 current chunk (causal)
  int kbase;    // window position of the block's first key (kinds 2, 3)
  int slot0;    // first attractor slot (kind 1)
};

template <int HD>
B3_DEV void load_rows(bf16* s, const bf16* g, int rows, int rows_valid) {
  constexpr int CPR = HD / 8;
  for (int i = threadIdx.x; i < rows * CPR; i += NT) {
    const int r = i / CPR, ch = i % CPR;
    const bool ok = r < rows_valid;
    cp_async16(s + swz<HD>(r, ch * 8), ok ? g + (int64_t)r * HD + ch * 8 : g, ok);
  }
}

// Scores of one key block for the warp's 16 rows: s = q k^T * scale (+ bias), masked to -inf.
template <int HD, int NK>
B3_DEV void block_scores(float (&s)[NK / 8][4], const uint32_t (&qa)[HD / 16][4], const bf16* ks,
                         const float* bias, int nvalid, bool causal, int kbase, int lim0, int lim1,
                         int lane) {
  constexpr float scale = HD == 128 ? 0.08838834764831845f : 0.125f;  // fp32(HD ** -0.5)
  const int t4 = lane & 3;
#pragma unroll
  for (int n = 0; n < NK / 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
  for (int kt = 0; kt < HD / 16; ++kt) {
#pragma unroll
    for (int np = 0; np < NK / 16; ++np) {
      uint32_t b[4];
      ldsm_x4(b, ks + swz<HD>(np * 16 + (lane & 7) + (lane >> 4) * 8, kt * 16 + ((lane >> 3) & 1) * 8));
      mma16816(s[2 * np], qa[kt], b[0], b[1]);
      mma16816(s[2 * np + 1], qa[kt], b[2], b[3]);
    }
  }
#pragma unroll
  for (int n = 0; n < NK / 8; ++n) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int col = n * 8 + 2 * t4 + (q & 1);
      float x = __fmul_rn(s[n][q], scale);
      if (bias) x = __fadd_rn(x, bias[col]);
      const bool vis = col < nvalid && (!causal || kbase + col <= (q < 2 ? lim0 : lim1));
      s[n][q] = vis ? x : neg_inf();
    }
  }
}

// Pass 1: running row max and sum of exp over one block.
template <int HD, int NK>
B3_DEV void block_stats(float (&mrow)[2], float (&lrow)[2], const uint32_t (&qa)[HD / 16][4],
                        const bf16* ks, const float* bias, int nvalid, bool causal, int kbase, int lim0,
                        int lim1, int lane) {
  float s[NK / 8][4];
  block_scores<HD, NK>(s, qa, ks, bias, nvalid, causal, kbase, lim0, lim1, lane);
  float bm0 = neg_inf(), bm1 = neg_inf();
#pragma unroll
  for (int n = 0; n < NK / 8; ++n) {
    bm0 = fmaxf(bm0, fmaxf(s[n][0], s[n][1]));
    bm1 = fmaxf(bm1, fmaxf(s[n][2], s[n][3]));
  }
  bm0 = quad_max(bm0);
  bm1 = quad_max(bm1);
  const float mn0 = fmaxf(mrow[0], bm0), mn1 = fmaxf(mrow[1], bm1);
  float ps0 = 0.f, ps1 = 0.f;
  if (mn0 != neg_inf()) {
#pragma unroll
    for (int n = 0; n < NK / 8; ++n) ps0 += expf(s[n][0] - mn0) + expf(s[n][1] - mn0);
  }
  if (mn1 != neg_inf()) {
#pragma unroll
    for (int n = 0; n < NK / 8; ++n) ps1 += expf(s[n][2] - mn1) + expf(s[n][3] - mn1);
  }
  ps0 = quad_sum(ps0);
  ps1 = quad_sum(ps1);
  lrow[0] = (mn0 == neg_inf() ? 0.f : lrow[0] * expf(mrow[0] - mn0)) + ps0;
  lrow[1] = (mn1 == neg_inf() ? 0.f : lrow[1] * expf(mrow[1] - mn1)) + ps1;
  mrow[0] = mn0;
  mrow[1] = mn1;
}

// Pass 2: p = bf16(exp(s - max) / sum) exactly as the reference normalises before its bf16 cast
// (F.softmax(...).to(dtype), bolt3.py:249), then o += p v.
template <int HD, int NK>
B3_DEV void block_pv(float (&o)[HD / 8][4], const float (&mrow)[2], const float (&lrow)[2],
                     const uint32_t (&qa)[HD / 16][4], const bf16* ks, const bf16* vs, const float* bias,
                     int nvalid, bool causal, int kbase, int lim0, int lim1, int lane) {
  float s[NK / 8][4];
  block_scores<HD, NK>(s, qa, ks, bias, nvalid, causal, kbase, lim0, lim1, lane);
#pragma unroll
  for (int n = 0; n < NK / 8; ++n) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float m = mrow[q >> 1], l = lrow[q >> 1];
      s[n][q] = s[n][q] == neg_inf() ? 0.f : __fdiv_rn(expf(s[n][q] - m), l);
    }
  }
  uint32_t pk[NK / 16][4];
#pragma unroll
  for (int kt = 0; kt < NK / 16; ++kt) {
    pk[kt][0] = pack_bf16(s[2 * kt][0], s[2 * kt][1]);
    pk[kt][1] = pack_bf16(s[2 * kt][2], s[2 * kt][3]);
    pk[kt][2] = pack_bf16(s[2 * kt + 1][0], s[2 * kt + 1][1]);
    pk[kt][3] = pack_bf16(s[2 * kt + 1][2], s[2 * kt + 1][3]);
  }
#pragma unroll
  for (int kt = 0; kt < NK / 16; ++kt) {
#pragma unroll
    for (int np = 0; np < HD / 16; ++np) {
      uint32_t b[4];
      ldsm_x4_t(b, vs + swz<HD>(kt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, np * 16 + (lane >> 4) * 8));
      mma16816(o[2 * np], pk[kt], b[0], b[1]);
      mma16816(o[2 * np + 1], pk[kt], b[2], b[3]);
    }
  }
}

template <int HD>
__global__ void __launch_bounds__(NT, 1) attend_kernel(bolt3_attend_args a) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  Smem<HD>& sm = *reinterpret_cast<Smem<HD>*>(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int r0 = warp * 16;
  const int c = blockIdx.z;
  const int blk = blockIdx.x;
  const int G = a.G;
  const int kvh = c % a.hkv, b = c / a.hkv;
  const int H = a.hkv * G;

  // ---- geometry of this tile
  const int ntok = (int)min((int64_t)128, a.Tq - (int64_t)blk * 128);
  const int gn = a.prefill ? 1 : max(1, min(G, 128 / max(ntok, 1)));
  const int g0 = blockIdx.y * gn;
  const int ng = min(gn, G - g0);
  const int n_rows = ng * ntok;
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
  const int n_before = L0 + len_before;
  const int64_t bofs = ((int64_t)c * a.bank_cap + bank_idx);
  const bf16* bk = has_bank ? reinterpret_cast<const bf16*>(a.bank_ak_rope) + bofs * S * HD : nullptr;
  const bf16* bv = has_bank ? reinterpret_cast<const bf16*>(a.bank_av) + bofs * S * HD : nullptr;
  const float* bmass = has_bank ? a.bank_mass + bofs * S : nullptr;
  const uint8_t* bact = has_bank ? a.bank_act + bofs * S : nullptr;
  const float kappa = a.kappa[kvh];

  const int n_sink_jobs = has_sinks ? 1 : 0;
  const int n_attr_jobs = has_bank ? S / KB : 0;
  const int n_seg0_jobs = (L0 + KB - 1) / KB;
  const int n_seg1_jobs = (L1 + KB - 1) / KB;
  const int n_jobs = n_sink_jobs + n_attr_jobs + n_seg0_jobs + n_seg1_jobs;

  auto job_at = [&](int j) {
    Job jb;
    if (j < n_sink_jobs) {
      jb.k = sk; jb.v = sv; jb.n = 4; jb.kind = 0; jb.kbase = 0; jb.slot0 = 0;
      return jb;
    }
    j -= n_sink_jobs;
    if (j < n_attr_jobs) {
      jb.k = bk + (int64_t)j * KB * HD; jb.v = bv + (int64_t)j * KB * HD; jb.n = KB; jb.kind = 1;
      jb.kbase = 0; jb.slot0 = j * KB;
      return jb;
    }
    j -= n_attr_jobs;
    if (j < n_seg0_jobs) {
      jb.k = k0 + (int64_t)j * KB * HD; jb.v = v0 + (int64_t)j * KB * HD;
      jb.n = min(KB, L0 - j * KB); jb.kind = 2; jb.kbase = j * KB; jb.slot0 = 0;
      return jb;
    }
    j -= n_seg0_jobs;
    jb.k = k1 + (int64_t)j * KB * HD; jb.v = v1 + (int64_t)j * KB * HD;
    jb.n = min(KB, L1 - j * KB); jb.kind = 3; jb.kbase = L0 + j * KB; jb.slot0 = 0;
    return jb;
  };
  // step j < n_jobs: statistics pass (keys only); step j >= n_jobs: P@V pass (keys and values)
  auto issue = [&](int j, int buf) {
    const bool pv = j >= n_jobs;
    const Job jb = job_at(pv ? j - n_jobs : j);
    const int rows = jb.kind == 0 ? 16 : KB;
    load_rows<HD>(sm.k + buf * KB * HD, jb.k, rows, jb.n);
    if (pv) load_rows<HD>(sm.v + buf * KB * HD, jb.v, rows, jb.n);
    if (jb.kind == 1) {
      for (int i = tid; i < KB; i += NT) {
        const int s_ = jb.slot0 + i;
        sm.bias[buf][i] = bact[s_] ? __fmul_rn(kappa, logf(fmaxf(bmass[s_], 1.0f))) : neg_inf();
      }
    }
  };

  // ---- query tile (q_rope) and its A fragments
  auto row_head_tok = [&](int r, int& g, int& i) {
    g = g0 + r / max(ntok, 1);
    i = r % max(ntok, 1);
  };
  {
    constexpr int CPR = HD / 8;
    for (int i = tid; i < 128 * CPR; i += NT) {
      const int r = i / CPR, ch = i % CPR;
      const bool ok = r < n_rows;
      int g, ti;
      row_head_tok(ok ? r : 0, g, ti);
      const int64_t tq = (int64_t)blk * 128 + ti;
      const bf16* src = reinterpret_cast<const bf16*>(a.q_rope) + (((int64_t)c * G + g) * a.Tq + tq) * HD + ch * 8;
      cp_async16(sm.q + swz<HD>(r, ch * 8), ok ? src : reinterpret_cast<const bf16*>(a.q_rope), ok);
    }
  }
  if (n_jobs > 0) issue(0, 0);
  cp_async_commit();

  float o[HD / 8][4];
#pragma unroll
  for (int n = 0; n < HD / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float mrow[2] = {neg_inf(), neg_inf()}, lrow[2] = {0.f, 0.f};
  uint32_t qa[HD / 16][4];
  const bool warp_active = r0 < n_rows;
  int gA, iA, gB, iB;
  row_head_tok(min(r0 + g8, max(n_rows - 1, 0)), gA, iA);
  row_head_tok(min(r0 + g8 + 8, max(n_rows - 1, 0)), gB, iB);
  const int lim0 = n_before + iA, lim1 = n_before + iB;
  // largest token index among this warp's rows (for skipping fully masked causal blocks)
  int imax = 0;
  for (int r = r0; r < min(r0 + 16, n_rows); ++r) { int gg, ii; row_head_tok(r, gg, ii); imax = max(imax, ii); }

  const int n_steps = 2 * n_jobs;
  for (int j = 0; j < n_steps; ++j) {
    if (j + 1 < n_steps) {
      issue(j + 1, (j + 1) & 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (j == 0 && warp_active) {
#pragma unroll
      for (int kt = 0; kt < HD / 16; ++kt)
        ldsm_x4(qa[kt], sm.q + swz<HD>(r0 + (lane & 15), kt * 16 + (lane >> 4) * 8));
    }
    const bool pv = j >= n_jobs;
    const Job jb = job_at(pv ? j - n_jobs : j);
    const int buf = j & 1;
    const bool skip = !warp_active || (jb.kind == 3 && jb.kbase > n_before + imax);
    if (!skip) {
      const bf16* kt_ = sm.k + buf * KB * HD;
      const bf16* vt_ = sm.v + buf * KB * HD;
      const float* bs = jb.kind == 1 ? sm.bias[buf] : nullptr;
      if (!pv) {
        if (jb.kind == 0) block_stats<HD, 16>(mrow, lrow, qa, kt_, nullptr, jb.n, false, 0, lim0, lim1, lane);
        else block_stats<HD, KB>(mrow, lrow, qa, kt_, bs, jb.n, jb.kind == 3, jb.kbase, lim0, lim1, lane);
      } else {
        if (jb.kind == 0) block_pv<HD, 16>(o, mrow, lrow, qa, kt_, vt_, nullptr, jb.n, false, 0, lim0, lim1, lane);
        else block_pv<HD, KB>(o, mrow, lrow, qa, kt_, vt_, bs, jb.n, jb.kind == 3, jb.kbase, lim0, lim1, lane);
      }
    }
    __syncthreads();
  }

  // ---- P@V result rounded to the storage dtype (the probabilities were normalised already)
#pragma unroll
  for (int n = 0; n < HD / 8; ++n) {
    o[n][0] = rbf(o[n][0]); o[n][1] = rbf(o[n][1]);
    o[n][2] = rbf(o[n][2]); o[n][3] = rbf(o[n][3]);
  }

  if (has_bank) {
    // ---- M_res read-out epilogue: q_raw tile, M split, normalise, RMSNorm, eta gate
    const float* gm = a.bank_m + bofs * HD * HD;
    {
      constexpr int CPR = HD / 8;
      for (int i = tid; i < 128 * CPR; i += NT) {
        const int r = i / CPR, ch = i % CPR;
        const bool ok = r < n_rows;
        int g, ti;
        row_head_tok(ok ? r : 0, g, ti);
        const int64_t tq = (int64_t)blk * 128 + ti;
        const bf16* src = reinterpret_cast<const bf16*>(a.q_raw) + (((int64_t)c * G + g) * a.Tq + tq) * HD + ch * 8;
        cp_async16(sm.q + swz<HD>(r, ch * 8), ok ? src : reinterpret_cast<const bf16*>(a.q_raw), ok);
      }
      cp_async_commit();
      for (int i = tid; i < HD * HD / 4; i += NT) {
        const int d = (i * 4) / HD, e = (i * 4) % HD;
        const float4 m4 = *reinterpret_cast<const float4*>(gm + (int64_t)d * HD + e);
        const float mv[4] = {m4.x, m4.y, m4.z, m4.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const bf16 hi = __float2bfloat16_rn(mv[u]);
          sm.k[swz<HD>(d, e + u)] = hi;
          sm.v[swz<HD>(d, e + u)] = __float2bfloat16_rn(mv[u] - bf2f(hi));
        }
      }
      cp_async_wait<0>();
      __syncthreads();
    }
    for (int r = warp * 16; r < warp * 16 + 16; ++r) {
      constexpr int EPL = HD / 32;
      const bf16* p = sm.q + swz<HD>(r, lane * EPL);
      float acc = 0.f;
#pragma unroll
      for (int e = 0; e < EPL; ++e) { const float x = bf2f(p[e]); acc = fmaf(x, x, acc); }
      acc = warp_sum(acc);
      if (lane == 0) sm.qn[r] = sqrtf(acc);
    }
    __syncwarp();
    if (warp_active) {
      float ym[HD / 8][4];
#pragma unroll
      for (int n = 0; n < HD / 8; ++n) ym[n][0] = ym[n][1] = ym[n][2] = ym[n][3] = 0.f;
#pragma unroll
      for (int kt = 0; kt < HD / 16; ++kt) {
        uint32_t qr[4];
        ldsm_x4(qr, sm.q + swz<HD>(r0 + (lane & 15), kt * 16 + (lane >> 4) * 8));
#pragma unroll
        for (int np = 0; np < HD / 16; ++np) {
          uint32_t bb[4];
          ldsm_x4_t(bb, sm.k + swz<HD>(kt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, np * 16 + (lane >> 4) * 8));
          mma16816(ym[2 * np], qr, bb[0], bb[1]);
          mma16816(ym[2 * np + 1], qr, bb[2], bb[3]);
          ldsm_x4_t(bb, sm.v + swz<HD>(kt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, np * 16 + (lane >> 4) * 8));
          mma16816(ym[2 * np], qr, bb[0], bb[1]);
          mma16816(ym[2 * np + 1], qr, bb[2], bb[3]);
        }
      }
      const float coef = a.coef[kvh];
      const float qn0 = fmaxf(sm.qn[r0 + g8], 1e-12f), qn1 = fmaxf(sm.qn[r0 + g8 + 8], 1e-12f);
      float ss0 = 0.f, ss1 = 0.f;
#pragma unroll
      for (int n = 0; n < HD / 8; ++n) {
        ym[n][0] = __fmul_rn(__fdiv_rn(ym[n][0], qn0), coef);
        ym[n][1] = __fmul_rn(__fdiv_rn(ym[n][1], qn0), coef);
        ym[n][2] = __fmul_rn(__fdiv_rn(ym[n][2], qn1), coef);
        ym[n][3] = __fmul_rn(__fdiv_rn(ym[n][3], qn1), coef);
        ss0 = fmaf(ym[n][0], ym[n][0], fmaf(ym[n][1], ym[n][1], ss0));
        ss1 = fmaf(ym[n][2], ym[n][2], fmaf(ym[n][3], ym[n][3], ss1));
      }
      ss0 = quad_sum(ss0);
      ss1 = quad_sum(ss1);
      const float rs0 = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss0, (float)HD), a.eps));
      const float rs1 = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss1, (float)HD), a.eps));
      const float* eta = a.eta;
      const float e0 = eta[((int64_t)c * G + gA) * a.Tq + (int64_t)blk * 128 + iA];
      const float e1 = eta[((int64_t)c * G + gB) * a.Tq + (int64_t)blk * 128 + iB];
#pragma unroll
      for (int n = 0; n < HD / 8; ++n) {
        const int col = n * 8 + 2 * t4;
        const float w0 = a.res_w[col], w1 = a.res_w[col + 1];
        o[n][0] = rbf(__fadd_rn(o[n][0], rbf(__fmul_rn(e0, __fmul_rn(__fmul_rn(ym[n][0], rs0), w0)))));
        o[n][1] = rbf(__fadd_rn(o[n][1], rbf(__fmul_rn(e0, __fmul_rn(__fmul_rn(ym[n][1], rs0), w1)))));
        o[n][2] = rbf(__fadd_rn(o[n][2], rbf(__fmul_rn(e1, __fmul_rn(__fmul_rn(ym[n][2], rs1), w0)))));
        o[n][3] = rbf(__fadd_rn(o[n][3], rbf(__fmul_rn(e1, __fmul_rn(__fmul_rn(ym[n][3], rs1), w1)))));
      }
    }
  }

  // ---- store y [B][y_tokens][H][HD]
  if (warp_active) {
    bf16* y = reinterpret_cast<bf16*>(a.y);
    const int rA = r0 + g8, rB = r0 + g8 + 8;
    const int64_t tA = (int64_t)blk * 128 + iA, tB = (int64_t)blk * 128 + iB;
    bf16* yA = y + (((int64_t)b * a.y_tokens + tA) * H + kvh * G + gA) * HD;
    bf16* yB = y + (((int64_t)b * a.y_tokens + tB) * H + kvh * G + gB) * HD;
#pragma unroll
    for (int n = 0; n < HD / 8; ++n) {
      const int col = n * 8 + 2 * t4;
      if (rA < n_rows) *reinterpret_cast<uint32_t*>(yA + col) = pack_bf16(o[n][0], o[n][1]);
      if (rB < n_rows) *reinterpret_cast<uint32_t*>(yB + col) = pack_bf16(o[n][2], o[n][3]);
    }
  }
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
                       (uintptr_t)a->bank_m;
  if (al & 15) return BOLT3_ERR_ALIGN;
  cudaStream_t s = (cudaStream_t)stream;
  dim3 grid;
  if (a->prefill) {
    grid = dim3((unsigned)((a->Tq + 127) / 128), (unsigned)a->G, (unsigned)a->n_chains);
  } else {
    const int gn = (int)std::max<int64_t>(1, std::min<int64_t>(a->G, 128 / a->Tq));
    grid = dim3(1, (unsigned)((a->G + gn - 1) / gn), (unsigned)a->n_chains);
  }
  int rc;
  if (a->HD == 128) {
    const size_t smem = sizeof(Smem<128>);
    if (cudaFuncSetAttribute(attend_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return BOLT3_ERR_CUDA;
    attend_kernel<128><<<grid, NT, smem, s>>>(*a);
  } else if (a->HD == 64) {
    const size_t smem = sizeof(Smem<64>);
    if (cudaFuncSetAttribute(attend_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return BOLT3_ERR_CUDA;
    attend_kernel<64><<<grid, NT, smem, s>>>(*a);
  } else {
    return BOLT3_ERR_SHAPE;
  }
  rc = cudaGetLastError() == cudaSuccess ? BOLT3_OK : BOLT3_ERR_CUDA;
  return rc;
}
