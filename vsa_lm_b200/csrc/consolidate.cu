// Phase B: the sequential attractor-bank / M_res consolidation scan.
//
// One CTA (8 warps) owns one chain (sequence b, KV head h) for all of its consolidation steps, so
// the bank never leaves the SM between steps: ak / av live in shared memory, M_res lives in the
// registers of warps 0..HD/16-1 as the accumulator fragments of its own update GEMM. Every
// contraction of _consolidate_functional (vsa_lm/config/bolt3.py:68-192) is a 128 x 128 x HD
// tensor-core product with bf16 operands, fp32 accumulation:
//   sc   = kp . RoPE(ak, pm)^T            (:97-100, :169-171)   exact bf16 products
//   v^   = softmax(sc).bf16 @ av          (:101, :172)
//   cos  = kr . ak^T / (|kr| |ak|)        (:104-106, :175-176)
//   pair = ak . ak^T / (|ak| |ak|)        (:128-130)
//   gram = |kr . kr^T| / (|kr| |kr|)      (:156-157)
//   k^ M = kr . (M_hi + M_lo) / |kr|      (:159)   M split into two bf16 terms: ~2^-17 relative
//   M   <- gamma M + kr^T . (E_hi + E_lo)  (:162)   E = err / |kr|, split the same way
// Rankings count, per entry, the entries that sort before it (128 threads, one entry each); when
// exactly equal keys decide the result the CPU torch.topk order is reproduced with the emulation in
// stl_select.h (bolt3.py:133-134, 183).
#include "../../include/bolt3.h"
#include "common.cuh"
#include "stl_select.h"
#include "tc5.cuh"

#include <cstddef>
#include <type_traits>

namespace {

using namespace b3;

constexpr int S = 128;   // attractor slots
constexpr int CC = 128;  // chunk rows
constexpr int NT = 256;  // threads per CTA
constexpr float SIM_K = 0.88f, SIM_V = 0.80f, GAMMA_U = 0.995f;  // bolt3.py:31

template <int HD>
struct Smem {
  bf16 ak[S * HD];
  bf16 av[S * HD];
  bf16 kr[CC * HD];
  bf16 vv[CC * HD];
  bf16 x1[128 * HD];   // kp, then M_hi, then E_hi
  bf16 x2[128 * HD];   // RoPE(ak, pm), then M_lo, then E_lo
  float mass[S], util[S], pm[S], keep[S], na[S], rna[S], bias[S], botv[S];
  float rel[CC], score[CC], bsk[CC], beta[CC], nk[CC], rnk[CC], nv[CC], pos[CC], wgt[CC], topv[CC];
  int best[CC], tops[CC], bots[S], mlist[CC];
  unsigned char act[S], mrg[CC], ins[CC];
  int n_merged;
  b3sel::KV selA[128], selB[128];
  alignas(16) uint32_t keys[2][128];   // ranking scratch of the two thread groups (read as uint4)
  unsigned char dirty[S];   // slots whose key or mean position changed this step
  int dlist[S], n_dirty;
  uint32_t tbase;           // tensor memory holding RoPE(ak, pm) between steps
};
static_assert(offsetof(Smem<128>, keys) % 16 == 0 && offsetof(Smem<64>, keys) % 16 == 0,
              "group_rank reads the ranking keys 16 bytes at a time");

// ------------------------------------------------------------------------------------------
// shared-memory tile movement

template <int HD>
B3_DEV void g2s_rows(bf16* s, const bf16* g, int rows_valid) {
  constexpr int CPR = HD / 8;
  for (int i = threadIdx.x; i < 128 * CPR; i += NT) {
    const int r = i / CPR, ch = i % CPR;
    const bool ok = r < rows_valid;
    cp_async16(s + swz<HD>(r, ch * 8), ok ? g + (int64_t)r * HD + ch * 8 : g, ok);
  }
}

template <int HD>
B3_DEV void s2g_rows(bf16* g, const bf16* s) {
  constexpr int CPR = HD / 8;
  for (int i = threadIdx.x; i < 128 * CPR; i += NT) {
    const int r = i / CPR, ch = i % CPR;
    *reinterpret_cast<uint4*>(g + (int64_t)r * HD + ch * 8) =
        *reinterpret_cast<const uint4*>(s + swz<HD>(r, ch * 8));
  }
}

// Bulk (TMA engine) copy of `bytes` contiguous bytes of shared memory to global memory.
B3_DEV void bulk_s2g(void* gdst, const void* ssrc, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n" ::"l"(gdst),
               "r"((uint32_t)__cvta_generic_to_shared(ssrc)), "r"(bytes)
               : "memory");
}

// squared L2 norm of row r of a swizzled tile (whole warp)
template <int HD>
B3_DEV float row_sumsq(const bf16* s, int r, int lane) {
  constexpr int EPL = HD / 32;
  const bf16* p = s + swz<HD>(r, lane * EPL);
  float acc = 0.f;
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    const float x = bf2f(p[e]);
    acc = fmaf(x, x, acc);
  }
  return warp_sum(acc);
}

// Sum over one half of the 16-byte chunks of row r of x*y (swizzling only permutes chunks within a
// row, so the two halves of a row together cover it exactly once). Each row starts its sweep at a
// different chunk, so the lanes of a warp (consecutive rows) read different shared-memory banks.
template <int HD>
B3_DEV float half_row_dot(const bf16* x, const bf16* y, int r, int half) {
  constexpr int CPR = HD / 8, NH = CPR / 2;
  float acc = 0.f;
#pragma unroll
  for (int c = 0; c < NH; ++c) {
    const int ch = half * NH + ((c + r) & (NH - 1));                  // physical chunk of row r
    const int off = (ch >> 3) * (128 * 64) + r * 64 + (ch & 7) * 8;
    const uint4 a = *reinterpret_cast<const uint4*>(x + off);
    const uint4 b = *reinterpret_cast<const uint4*>(y + off);
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float2 fa = unpack_bf16(aw[u]), fb = unpack_bf16(bw[u]);
      acc = fmaf(fa.x, fb.x, fmaf(fa.y, fb.y, acc));
    }
  }
  return acc;
}

// ------------------------------------------------------------------------------------------
// warp-level GEMMs on 16 rows (r0 .. r0+15); fragments follow mma.m16n8k16 layouts

// acc[16 x 128] = A[r0.., K] . B[0..128, K]^T   (A, B swizzled tiles with K = HD columns)
template <int HD>
B3_DEV void gemm_nt(float (&acc)[16][4], const bf16* A, int r0, const bf16* B, int lane) {
#pragma unroll
  for (int n = 0; n < 16; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
#pragma unroll
  for (int kt = 0; kt < HD / 16; ++kt) {
    uint32_t a[4];
    ldsm_x4(a, A + swz<HD>(r0 + (lane & 15), kt * 16 + (lane >> 4) * 8));
#pragma unroll
    for (int np = 0; np < 8; ++np) {
      uint32_t b[4];
      ldsm_x4(b, B + swz<HD>(np * 16 + (lane & 7) + (lane >> 4) * 8, kt * 16 + ((lane >> 3) & 1) * 8));
      mma16816(acc[2 * np], a, b[0], b[1]);
      mma16816(acc[2 * np + 1], a, b[2], b[3]);
    }
  }
}

// acc[16 x HD] += P[16 x 128] . B[128 x HD]   (P as A fragments, B swizzled row-major [128][HD])
template <int HD>
B3_DEV void gemm_pv(float (&acc)[HD / 8][4], const uint32_t (&pa)[8][4], const bf16* B, int lane) {
#pragma unroll
  for (int kt = 0; kt < 8; ++kt) {
#pragma unroll
    for (int np = 0; np < HD / 16; ++np) {
      uint32_t b[4];
      ldsm_x4_t(b, B + swz<HD>(kt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, np * 16 + (lane >> 4) * 8));
      mma16816(acc[2 * np], pa[kt], b[0], b[1]);
      mma16816(acc[2 * np + 1], pa[kt], b[2], b[3]);
    }
  }
}

// acc[16 x HD] += A[r0.., 0..HD] . B[HD x HD]   (A swizzled [128][HD], B swizzled [HD][HD])
template <int HD>
B3_DEV void gemm_nn(float (&acc)[HD / 8][4], const bf16* A, int r0, const bf16* B, int lane) {
#pragma unroll
  for (int kt = 0; kt < HD / 16; ++kt) {
    uint32_t a[4];
    ldsm_x4(a, A + swz<HD>(r0 + (lane & 15), kt * 16 + (lane >> 4) * 8));
#pragma unroll
    for (int np = 0; np < HD / 16; ++np) {
      uint32_t b[4];
      ldsm_x4_t(b, B + swz<HD>(kt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, np * 16 + (lane >> 4) * 8));
      mma16816(acc[2 * np], a, b[0], b[1]);
      mma16816(acc[2 * np + 1], a, b[2], b[3]);
    }
  }
}

// acc[16 x HD] += A^T[m0.., 0..128] . B[128 x HD]   (A stored [128 tokens][HD], read transposed)
template <int HD>
B3_DEV void gemm_tn(float (&acc)[HD / 8][4], const bf16* A, int m0, const bf16* B, int lane) {
#pragma unroll 2
  for (int kt = 0; kt < 8; ++kt) {
    uint32_t a[4];
    ldsm_x4_t(a, A + swz<HD>(kt * 16 + (lane & 7) + (lane >> 4) * 8, m0 + ((lane >> 3) & 1) * 8));
#pragma unroll
    for (int np = 0; np < HD / 16; ++np) {
      uint32_t b[4];
      ldsm_x4_t(b, B + swz<HD>(kt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, np * 16 + (lane >> 4) * 8));
      mma16816(acc[2 * np], a, b[0], b[1]);
      mma16816(acc[2 * np + 1], a, b[2], b[3]);
    }
  }
}

// ------------------------------------------------------------------------------------------
// ranking of up to 128 (value, index) entries by 128 threads (t = 0..127 of a named-barrier group):
// thread t counts the entries that sort before entry t. Sorted order: "largest" = descending value,
// else ascending; equal values by ascending index; entries with index >= n are padding and sort
// last. group_rank writes out_idx/out_val[0..k) in that order; group_resolve then checks whether
// exactly equal values (or a NaN) decide any of the first `limit` positions and, if so, has thread 0
// recompute the CPU torch.topk order with the libstdc++-compatible emulation. Equal values sit on
// adjacent positions, so the order of ties never changes the value at a position, only the index.
// `keys` is 128 words of shared scratch for the group.
struct Rank {
  int rank, eq_after;  // position of entry t; entries with the same value and a larger index
  float v;
};

B3_DEV Rank group_rank(const float* vals, int n, int k, bool largest, int* out_idx, float* out_val,
                       uint32_t* keys, int t, int bar_id) {
  uint32_t kt = 0xffffffffu;
  float vt = 0.f;
  if (t < n) {
    vt = vals[t];
    // +0 and -0 compare equal: give them one key so that equal values have equal keys
    const uint32_t f = fkey(vt == 0.f ? 0.f : vt);
    kt = largest ? ~f : f;
    if (kt == 0xffffffffu) kt = 0xfffffffeu;
  }
  keys[t] = kt;
  asm volatile("bar.sync %0, 128;\n" ::"r"(bar_id) : "memory");
  int rank = 0, eq_after = 0;
#pragma unroll 4
  for (int j4 = 0; j4 < 128; j4 += 4) {
    const uint4 kq = *reinterpret_cast<const uint4*>(keys + j4);
    const uint32_t kk[4] = {kq.x, kq.y, kq.z, kq.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = j4 + u;
      rank += (kk[u] < kt) | ((kk[u] == kt) & (j < t));
      eq_after += (kk[u] == kt) & (j > t);
    }
  }
  if (rank < k) {
    out_idx[rank] = t;
    out_val[rank] = vt;
  }
  return Rank{rank, eq_after, vt};
}

B3_DEV void group_resolve(const Rank& rk, int limit, float ignore_below, const float* vals, int n, int k, bool largest,
                          int* out_idx, float* out_val, b3sel::KV* buf, int t, int bar_id, int32_t* status) {
  const bool tie_t =
      t < n && ((rk.v != rk.v) || (rk.rank < limit && rk.eq_after > 0 && rk.rank + 1 < n && rk.v >= ignore_below));
  int any_tie;
  asm volatile(
      "{\n.reg .pred p, q;\nsetp.ne.u32 p, %2, 0;\nbar.red.or.pred q, %1, 128, p;\nselp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(any_tie)
      : "r"(bar_id), "r"((uint32_t)tie_t)
      : "memory");
  if (any_tie && t == 0) {
    for (int i = 0; i < n; ++i) { buf[i].v = vals[i]; buf[i].i = i; }
    const int bad = b3sel::topk_order(buf, n, k, largest);
    if (bad && status) atomicOr(status, 1);
    for (int i = 0; i < k; ++i) {
      out_idx[i] = buf[i].i;
      out_val[i] = buf[i].v;
    }
  }
}

// copy one row of EPL bf16 per lane (lane * EPL .. + EPL - 1 lie in one 16-byte chunk)
template <int HD>
B3_DEV void copy_row_part(bf16* dst, int sd, const bf16* src, int ss, int lane) {
  constexpr int EPL = HD / 32;
  using V = typename std::conditional<EPL == 4, uint2, uint32_t>::type;
  *reinterpret_cast<V*>(dst + swz<HD>(sd, lane * EPL)) = *reinterpret_cast<const V*>(src + swz<HD>(ss, lane * EPL));
}

// ------------------------------------------------------------------------------------------

template <int HD>
__global__ void __launch_bounds__(NT, 1) consolidate_kernel(bolt3_consolidate_args a) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  Smem<HD>& sm = *reinterpret_cast<Smem<HD>*>(smem_raw);
  const int c = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int r0 = warp * 16;
  const int h = c % a.hkv;
  const float kappa = a.kappa[h];
  const float gam = a.gamma[h];
  constexpr float scale = HD == 128 ? 0.08838834764831845f : 0.125f;  // fp32(HD ** -0.5)
  const bool m_owner = warp < HD / 16;

  bf16* g_ak = reinterpret_cast<bf16*>(a.ak) + (int64_t)c * S * HD;
  bf16* g_av = reinterpret_cast<bf16*>(a.av) + (int64_t)c * S * HD;
  float* g_m = a.m_res + (int64_t)c * HD * HD;

  // ---- load or initialise the bank (bolt3.py:83-92)
  int n_filled;
  float mr[HD / 8][4];
  if (a.init_blank) {
    n_filled = 0;
    for (int i = tid; i < S * HD / 8; i += NT) {
      *reinterpret_cast<uint4*>(sm.ak + i * 8) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(sm.av + i * 8) = make_uint4(0, 0, 0, 0);
    }
    for (int s = tid; s < S; s += NT) {
      sm.mass[s] = 1.f; sm.util[s] = 0.f; sm.pm[s] = 0.f; sm.act[s] = 0;
    }
#pragma unroll
    for (int n = 0; n < HD / 8; ++n) mr[n][0] = mr[n][1] = mr[n][2] = mr[n][3] = 0.f;
  } else {
    n_filled = a.n_filled[c];
    g2s_rows<HD>(sm.ak, g_ak, S);
    g2s_rows<HD>(sm.av, g_av, S);
    cp_async_commit();
    for (int s = tid; s < S; s += NT) {
      sm.mass[s] = a.mass[(int64_t)c * S + s];
      sm.util[s] = a.util[(int64_t)c * S + s];
      sm.pm[s] = a.pm[(int64_t)c * S + s];
      sm.act[s] = a.act[(int64_t)c * S + s];
    }
    if (m_owner) {
#pragma unroll
      for (int n = 0; n < HD / 8; ++n) {
        const float2 u = *reinterpret_cast<const float2*>(g_m + (r0 + g) * HD + n * 8 + 2 * t4);
        const float2 w = *reinterpret_cast<const float2*>(g_m + (r0 + g + 8) * HD + n * 8 + 2 * t4);
        mr[n][0] = u.x; mr[n][1] = u.y; mr[n][2] = w.x; mr[n][3] = w.y;
      }
    } else {
#pragma unroll
      for (int n = 0; n < HD / 8; ++n) mr[n][0] = mr[n][1] = mr[n][2] = mr[n][3] = 0.f;
    }
    cp_async_wait<0>();
  }
  __syncthreads();

  // RoPE(ak, pm) of slots slot_of(0 .. n_slots-1) into x2 (bolt3.py:17-20 in the storage dtype: cos
  // and sin rounded, every product and sum rounded), two frequencies per item so that each pair of
  // roundings is one conversion
  auto rope_slots = [&](int n_slots, auto slot_of) {
    for (int i = tid; i < n_slots * (HD / 4); i += NT) {
      const int s = slot_of(i / (HD / 4)), d = (i % (HD / 4)) * 2;
      float sn0, cs0, sn1, cs1;
      sincosf(__fmul_rn(sm.pm[s], a.inv_freq[d]), &sn0, &cs0);
      sincosf(__fmul_rn(sm.pm[s], a.inv_freq[d + 1]), &sn1, &cs1);
      uint32_t t;
      const float2 cs = rbf2(cs0, cs1, t), sn = rbf2(sn0, sn1, t);
      const float2 x0 = unpack_bf16(*reinterpret_cast<const uint32_t*>(&sm.ak[swz<HD>(s, d)]));
      const float2 x1 = unpack_bf16(*reinterpret_cast<const uint32_t*>(&sm.ak[swz<HD>(s, d + HD / 2)]));
      const float2 a0 = rbf2(__fmul_rn(x0.x, cs.x), __fmul_rn(x0.y, cs.y), t);
      const float2 b0 = rbf2(__fmul_rn(-x1.x, sn.x), __fmul_rn(-x1.y, sn.y), t);
      const float2 a1 = rbf2(__fmul_rn(x1.x, cs.x), __fmul_rn(x1.y, cs.y), t);
      const float2 b1 = rbf2(__fmul_rn(x0.x, sn.x), __fmul_rn(x0.y, sn.y), t);
      *reinterpret_cast<uint32_t*>(&sm.x2[swz<HD>(s, d)]) = pack_bf16(__fadd_rn(a0.x, b0.x), __fadd_rn(a0.y, b0.y));
      *reinterpret_cast<uint32_t*>(&sm.x2[swz<HD>(s, d + HD / 2)]) =
          pack_bf16(__fadd_rn(a1.x, b1.x), __fadd_rn(a1.y, b1.y));
    }
  };
  // x2 <-> tensor memory between steps (x2 is scratch inside a step): warp w moves row
  // 32 * (w % 4) + lane (its TMEM lane), half w / 4 of the columns
  constexpr int NW2 = HD / 4;  // 32-bit words per half row
  const int x2_row = 32 * (warp & 3) + lane, x2_half = warp >> 2;
  auto x2_taddr = [&]() { return sm.tbase + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)(x2_half * NW2); };
  auto x2_save = [&]() {
    uint32_t w[NW2];
#pragma unroll
    for (int q = 0; q < NW2 / 4; ++q) {
      const uint4 u = *reinterpret_cast<const uint4*>(&sm.x2[swz<HD>(x2_row, x2_half * (HD / 2) + q * 8)]);
      w[4 * q] = u.x; w[4 * q + 1] = u.y; w[4 * q + 2] = u.z; w[4 * q + 3] = u.w;
    }
    if constexpr (NW2 == 32) tc5::st32(x2_taddr(), w);
    else tc5::st16(x2_taddr(), w);
    tc5::st_wait();
  };
  auto x2_restore = [&]() {
    uint32_t w[NW2];
    tc5::ld_cols(x2_taddr(), w);
    tc5::ld_wait();
#pragma unroll
    for (int q = 0; q < NW2 / 4; ++q)
      *reinterpret_cast<uint4*>(&sm.x2[swz<HD>(x2_row, x2_half * (HD / 2) + q * 8)]) =
          make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
  };
  if (warp == 0) {
    tc5::tmem_alloc(&sm.tbase, 64);
    tc5::tmem_relinquish();
  }
  for (int s = tid; s < S; s += NT) sm.dirty[s] = 0;
  tc5::fence_before_sync();
  __syncthreads();
  tc5::fence_after_sync();
  rope_slots(S, [](int i) { return i; });
  __syncthreads();
  x2_save();

  const bf16* g_kr = reinterpret_cast<const bf16*>(a.kr) + (int64_t)c * a.chain_tokens * HD;
  const bf16* g_kp = reinterpret_cast<const bf16*>(a.kp) + (int64_t)c * a.chain_tokens * HD;
  const bf16* g_v = reinterpret_cast<const bf16*>(a.v) + (int64_t)c * a.chain_tokens * HD;
  const float* g_beta = a.beta + (int64_t)c * a.chain_tokens;

  for (int st = 0; st < a.n_steps; ++st) {
    const int skip = st == 0 ? a.skip0 : 0;
    const int64_t t_begin = a.token0 + (int64_t)st * a.step_tokens + skip;
    const int l_tok = a.chunk_len - skip;

    // ---- load the chunk: kr, kp (x1), v; beta, positions
    g2s_rows<HD>(sm.kr, g_kr + t_begin * HD, l_tok);
    g2s_rows<HD>(sm.vv, g_v + t_begin * HD, l_tok);
    if (n_filled > 0) g2s_rows<HD>(sm.x1, g_kp + t_begin * HD, l_tok);
    cp_async_commit();
    if (tid == 0 && st + 1 < a.n_steps) {
      // pull the next chunk into L2 while this step computes
      const int64_t nb = a.token0 + (int64_t)(st + 1) * a.step_tokens;
      const uint32_t bytes = (uint32_t)a.chunk_len * HD * 2;
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(g_kr + nb * HD), "r"(bytes));
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(g_kp + nb * HD), "r"(bytes));
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(g_v + nb * HD), "r"(bytes));
    }
    for (int j = tid; j < CC; j += NT) {
      sm.beta[j] = j < l_tok ? g_beta[t_begin + j] : 0.f;
      sm.pos[j] = (float)(a.pos0 + t_begin + j);
      sm.mrg[j] = 0;
      sm.ins[j] = 0;
    }
    for (int s = tid; s < S; s += NT) sm.util[s] = __fmul_rn(sm.util[s], GAMMA_U);  // :94
    cp_async_wait<0>();
    __syncthreads();
    {
      // row norms of the chunk keys / values and of the slot keys: two threads per row
      const int r = tid >> 1, half = tid & 1;
      float kk = half_row_dot<HD>(sm.kr, sm.kr, r, half);
      float vv2 = half_row_dot<HD>(sm.vv, sm.vv, r, half);
      float aa = half_row_dot<HD>(sm.ak, sm.ak, r, half);
      kk += __shfl_xor_sync(0xffffffffu, kk, 1);
      vv2 += __shfl_xor_sync(0xffffffffu, vv2, 1);
      aa += __shfl_xor_sync(0xffffffffu, aa, 1);
      if (half == 0) {
        sm.nk[r] = sqrtf(kk);
        sm.nv[r] = sqrtf(vv2);
        sm.na[r] = sqrtf(aa);
        // F.normalize divides by max(|x|, 1e-12); the contractions multiply by the reciprocal
        sm.rnk[r] = 1.0f / fmaxf(sm.nk[r], 1e-12f);
        sm.rna[r] = 1.0f / fmaxf(sm.na[r], 1e-12f);
      }
    }
    __syncthreads();

    const bool full = n_filled >= S;
    if (n_filled == 0) {
      // ---- first fill: score = unbiased var(normalize(v)) (bolt3.py:180). The normalised values
      // are fp32 as in the reference; mean and variance accumulate in fp64 (the CPU reference's
      // variance reduction is exact to fp32 rounding given its inputs, which this reproduces).
      for (int r = warp; r < l_tok; r += 8) {
        constexpr int EPL = HD / 32;
        const bf16* p = sm.vv + swz<HD>(r, lane * EPL);
        const float den = fmaxf(sm.nv[r], 1e-12f);
        float xs[EPL];
        double sum = 0.0;
#pragma unroll
        for (int e = 0; e < EPL; ++e) { xs[e] = __fdiv_rn(bf2f(p[e]), den); sum += (double)xs[e]; }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        const double mean = sum / HD;
        double sq = 0.0;
#pragma unroll
        for (int e = 0; e < EPL; ++e) { const double d = (double)xs[e] - mean; sq += d * d; }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
        if (lane == 0) {
          sm.score[r] = (float)(sq / (HD - 1));
          sm.rel[r] = 0.15f;  // initial utility of the very first fill (:181)
        }
      }
      __syncthreads();
    } else {
      // ---- attractor prediction of each token's value (:97-103 / :169-174)
      for (int s = tid; s < S; s += NT) {
        const float lm = logf(fmaxf(sm.mass[s], 1.0f));
        sm.bias[s] = full ? __fmul_rn(kappa, lm) : lm;
      }
      __syncthreads();
      uint32_t pa[8][4];
      {
        float acc[16][4];
        gemm_nt<HD>(acc, sm.x1, r0, sm.x2, lane);
        float mx0 = neg_inf(), mx1 = neg_inf();
#pragma unroll
        for (int n = 0; n < 16; ++n) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int col = n * 8 + 2 * t4 + (q & 1);
            float sc = __fadd_rn(__fmul_rn(acc[n][q], scale), sm.bias[col]);
            if (!full && !sm.act[col]) sc = -1e9f;
            acc[n][q] = sc;
          }
          mx0 = fmaxf(mx0, fmaxf(acc[n][0], acc[n][1]));
          mx1 = fmaxf(mx1, fmaxf(acc[n][2], acc[n][3]));
        }
        mx0 = quad_max(mx0);
        mx1 = quad_max(mx1);
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int n = 0; n < 16; ++n) {
          acc[n][0] = expf(acc[n][0] - mx0); acc[n][1] = expf(acc[n][1] - mx0);
          acc[n][2] = expf(acc[n][2] - mx1); acc[n][3] = expf(acc[n][3] - mx1);
          s0 += acc[n][0] + acc[n][1];
          s1 += acc[n][2] + acc[n][3];
        }
        const float i0 = 1.0f / quad_sum(s0), i1 = 1.0f / quad_sum(s1);
#pragma unroll
        for (int kt = 0; kt < 8; ++kt) {
          pa[kt][0] = pack_bf16(__fmul_rn(acc[2 * kt][0], i0), __fmul_rn(acc[2 * kt][1], i0));
          pa[kt][1] = pack_bf16(__fmul_rn(acc[2 * kt][2], i1), __fmul_rn(acc[2 * kt][3], i1));
          pa[kt][2] = pack_bf16(__fmul_rn(acc[2 * kt + 1][0], i0), __fmul_rn(acc[2 * kt + 1][1], i0));
          pa[kt][3] = pack_bf16(__fmul_rn(acc[2 * kt + 1][2], i1), __fmul_rn(acc[2 * kt + 1][3], i1));
        }
      }
      {
        float acc2[HD / 8][4];
#pragma unroll
        for (int n = 0; n < HD / 8; ++n) acc2[n][0] = acc2[n][1] = acc2[n][2] = acc2[n][3] = 0.f;
        gemm_pv<HD>(acc2, pa, sm.av, lane);
        float e0 = 0.f, e1 = 0.f;
#pragma unroll
        for (int n = 0; n < HD / 8; ++n) {
          const int col = n * 8 + 2 * t4;
          const float2 va = unpack_bf16(*reinterpret_cast<const uint32_t*>(&sm.vv[swz<HD>(r0 + g, col)]));
          const float2 vb = unpack_bf16(*reinterpret_cast<const uint32_t*>(&sm.vv[swz<HD>(r0 + g + 8, col)]));
          const float v00 = va.x, v01 = va.y, v10 = vb.x, v11 = vb.y;
          float d;
          d = v00 - acc2[n][0]; e0 = fmaf(d, d, e0);
          d = v01 - acc2[n][1]; e0 = fmaf(d, d, e0);
          d = v10 - acc2[n][2]; e1 = fmaf(d, d, e1);
          d = v11 - acc2[n][3]; e1 = fmaf(d, d, e1);
        }
        e0 = quad_sum(e0);
        e1 = quad_sum(e1);
        if (t4 == 0) {
          sm.rel[r0 + g] = __fdiv_rn(sqrtf(e0), __fadd_rn(sm.nv[r0 + g], 1e-6f));
          sm.rel[r0 + g + 8] = __fdiv_rn(sqrtf(e1), __fadd_rn(sm.nv[r0 + g + 8], 1e-6f));
        }
      }
      // ---- cosine match against the slots (:104-106, :175-177)
      {
        float acc[16][4];
        gemm_nt<HD>(acc, sm.kr, r0, sm.ak, lane);
        const float rk0 = sm.rnk[r0 + g], rk1 = sm.rnk[r0 + g + 8];
        float b0 = neg_inf(), b1 = neg_inf();
        int i0 = 0x7fffffff, i1 = 0x7fffffff;
#pragma unroll
        for (int n = 0; n < 16; ++n) {
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const int col = n * 8 + 2 * t4 + q;
            const float ra = sm.rna[col];
            float c0 = __fmul_rn(acc[n][q], __fmul_rn(rk0, ra));
            float c1 = __fmul_rn(acc[n][2 + q], __fmul_rn(rk1, ra));
            if (!full && !sm.act[col]) { c0 = 0.f; c1 = 0.f; }
            if (c0 > b0) { b0 = c0; i0 = col; }
            if (c1 > b1) { b1 = c1; i1 = col; }
          }
        }
#pragma unroll
        for (int o = 1; o <= 2; o <<= 1) {
          const float ob0 = __shfl_xor_sync(0xffffffffu, b0, o);
          const int oi0 = __shfl_xor_sync(0xffffffffu, i0, o);
          const float ob1 = __shfl_xor_sync(0xffffffffu, b1, o);
          const int oi1 = __shfl_xor_sync(0xffffffffu, i1, o);
          if (ob0 > b0 || (ob0 == b0 && oi0 < i0)) { b0 = ob0; i0 = oi0; }
          if (ob1 > b1 || (ob1 == b1 && oi1 < i1)) { b1 = ob1; i1 = oi1; }
        }
        if (t4 == 0) {
          sm.bsk[r0 + g] = b0; sm.best[r0 + g] = i0;
          sm.bsk[r0 + g + 8] = b1; sm.best[r0 + g + 8] = i1;
        }
      }
      __syncthreads();
      if (!full) {
        for (int j = tid; j < CC; j += NT)
          sm.score[j] = __fmul_rn(sm.rel[j], 1.0f - fminf(fmaxf(sm.bsk[j], 0.f), 1.f));  // :177
        __syncthreads();
      }
    }

    if (!full) {
      // ---- fill: the m best tokens take the next empty slots (:183-192)
      const int m = min(S - n_filled, l_tok);
      if (tid < 128) {
        const Rank rk = group_rank(sm.score, l_tok, m, true, sm.tops, sm.topv, sm.keys[0], tid, 1);
        group_resolve(rk, m, neg_inf(), sm.score, l_tok, m, true, sm.tops, sm.topv, sm.selA, tid, 1, a.status);
      }
      __syncthreads();
      for (int i = warp; i < m; i += 8) {
        const int j = sm.tops[i], s = n_filled + i;
        copy_row_part<HD>(sm.ak, s, sm.kr, j, lane);
        copy_row_part<HD>(sm.av, s, sm.vv, j, lane);
        if (lane == 0) {
          sm.pm[s] = sm.pos[j];
          sm.mass[s] = 1.f;
          sm.util[s] = sm.rel[j];
          sm.act[s] = 1;
          sm.dirty[s] = 1;
        }
      }
      n_filled += m;
      __syncthreads();
    } else {
      // ---- sim_v, score, merge mask (:107-110): two threads per row
      {
        const int r = tid >> 1, half = tid & 1;
        const int sb = sm.best[r];
        float dot = 0.f, aa = 0.f;
        if (r < l_tok) {
          constexpr int CPR = HD / 8;
#pragma unroll
          for (int h = 0; h < CPR / 2; ++h) {
            // logical chunk ch of row r sits at physical chunk ch ^ (row & 7) of that row
            const int ch = half * CPR / 2 + h;
            const uint4 a4 = *reinterpret_cast<const uint4*>(&sm.vv[swz<HD>(r, ch * 8)]);
            const uint4 b4 = *reinterpret_cast<const uint4*>(&sm.av[swz<HD>(sb, ch * 8)]);
            const uint32_t aw[4] = {a4.x, a4.y, a4.z, a4.w}, bw[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const float2 fa = unpack_bf16(aw[u]), fb = unpack_bf16(bw[u]);
              dot = fmaf(fa.x, fb.x, fmaf(fa.y, fb.y, dot));
              aa = fmaf(fb.x, fb.x, fmaf(fb.y, fb.y, aa));
            }
          }
        }
        dot += __shfl_xor_sync(0xffffffffu, dot, 1);
        aa += __shfl_xor_sync(0xffffffffu, aa, 1);
        if (half == 0 && r < l_tok) {
          const float sv = __fdiv_rn(dot, __fmul_rn(fmaxf(sm.nv[r], 1e-8f), fmaxf(sqrtf(aa), 1e-8f)));
          const float bs = sm.bsk[r];
          sm.score[r] = __fmul_rn(sm.rel[r], 1.0f - fminf(fmaxf(bs, 0.f), 1.f));
          sm.mrg[r] = (bs >= SIM_K) && (sv >= SIM_V);
        }
      }
      __syncthreads();
      // ---- merge: running means of the matched slots (:112-123)
      if (warp == 0) {
        int base = 0;
        for (int j0 = 0; j0 < CC; j0 += 32) {
          const int j = j0 + lane;
          const bool mm = j < l_tok && sm.mrg[j];
          const unsigned bal = __ballot_sync(0xffffffffu, mm);
          if (mm) sm.mlist[base + __popc(bal & ((1u << lane) - 1))] = j;
          base += __popc(bal);
        }
        if (lane == 0) sm.n_merged = base;
      }
      __syncthreads();
      const int n_m = sm.n_merged;
      if (n_m > 0) {
        for (int s = warp; s < S; s += 8) {
          int cnt = 0;
          for (int q = 0; q < n_m; ++q) cnt += sm.best[sm.mlist[q]] == s;
          if (cnt == 0) continue;
          constexpr int EPL = HD / 32;
          float ks[EPL], vs[EPL];
          float ps = 0.f;
#pragma unroll
          for (int e = 0; e < EPL; ++e) ks[e] = vs[e] = 0.f;
          for (int q = 0; q < n_m; ++q) {
            const int j = sm.mlist[q];
            if (sm.best[j] != s) continue;
#pragma unroll
            for (int e = 0; e < EPL; ++e) {
              ks[e] = __fadd_rn(ks[e], bf2f(sm.kr[swz<HD>(j, lane * EPL + e)]));
              vs[e] = __fadd_rn(vs[e], bf2f(sm.vv[swz<HD>(j, lane * EPL + e)]));
            }
            ps = __fadd_rn(ps, sm.pos[j]);
          }
          const float ms = sm.mass[s];
          const float nm = __fadd_rn(ms, (float)cnt);
#pragma unroll
          for (int e = 0; e < EPL; ++e) {
            const int d = lane * EPL + e;
            const float ka = __fadd_rn(__fmul_rn(ms, bf2f(sm.ak[swz<HD>(s, d)])), ks[e]);
            const float va = __fadd_rn(__fmul_rn(ms, bf2f(sm.av[swz<HD>(s, d)])), vs[e]);
            sm.ak[swz<HD>(s, d)] = __float2bfloat16_rn(__fdiv_rn(ka, nm));
            sm.av[swz<HD>(s, d)] = __float2bfloat16_rn(__fdiv_rn(va, nm));
          }
          __syncwarp();
          const float aa = row_sumsq<HD>(sm.ak, s, lane);
          if (lane == 0) {
            sm.pm[s] = __fdiv_rn(__fadd_rn(__fmul_rn(ms, sm.pm[s]), ps), nm);
            sm.mass[s] = nm;
            sm.dirty[s] = 1;
            sm.na[s] = sqrtf(aa);
            sm.rna[s] = 1.0f / fmaxf(sm.na[s], 1e-12f);
          }
        }
        __syncthreads();
      }
      // ---- diversity eviction (:125-152)
      {
        float acc[16][4];
        gemm_nt<HD>(acc, sm.ak, r0, sm.ak, lane);
        const float ra0 = sm.rna[r0 + g], ra1 = sm.rna[r0 + g + 8];
        float m0 = neg_inf(), m1 = neg_inf();
#pragma unroll
        for (int n = 0; n < 16; ++n) {
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const int col = n * 8 + 2 * t4 + q;
            // (ra_s * ra_s') is symmetric, so equal cosines of a mutual pair stay bit-identical
            const float rb = sm.rna[col];
            float p0 = __fmul_rn(acc[n][q], __fmul_rn(ra0, rb));
            float p1 = __fmul_rn(acc[n][2 + q], __fmul_rn(ra1, rb));
            if (col == r0 + g) p0 = -1.0f;
            if (col == r0 + g + 8) p1 = -1.0f;
            m0 = fmaxf(m0, p0);
            m1 = fmaxf(m1, p1);
          }
        }
        m0 = quad_max(m0);
        m1 = quad_max(m1);
        if (t4 == 0) {
          sm.keep[r0 + g] = __fmul_rn(sm.util[r0 + g], 1.0f - fminf(fmaxf(m0, 0.f), 0.98f));
          sm.keep[r0 + g + 8] = __fmul_rn(sm.util[r0 + g + 8], 1.0f - fminf(fmaxf(m1, 0.f), 0.98f));
        }
      }
      for (int j = tid; j < CC; j += NT) sm.wgt[j] = sm.mrg[j] ? -1e9f : sm.score[j];
      __syncthreads();
      const int k_cand = min(l_tok, S);
      // token candidates by weight (threads 0..127) and slots by keep value (128..255), both at once
      const bool grp_a = tid < 128;
      const Rank rk = grp_a ? group_rank(sm.wgt, l_tok, k_cand, true, sm.tops, sm.topv, sm.keys[0], tid, 1)
                            : group_rank(sm.keep, S, k_cand, false, sm.bots, sm.botv, sm.keys[1], tid - 128, 2);
      __syncthreads();
      // replacements take a prefix of the pairs (weights descend, keep values ascend); ties can only
      // matter inside it
      const int n_rep = __syncthreads_count(tid < k_cand && sm.topv[tid] > sm.botv[tid] && sm.topv[tid] > -1e8f);
      if (grp_a)
        group_resolve(rk, n_rep, -1e8f, sm.wgt, l_tok, k_cand, true, sm.tops, sm.topv, sm.selA, tid, 1, a.status);
      else
        group_resolve(rk, n_rep, neg_inf(), sm.keep, S, k_cand, false, sm.bots, sm.botv, sm.selB, tid - 128, 2,
                      a.status);
      __syncthreads();
      for (int i = warp; i < k_cand; i += 8) {
        const float tv = sm.topv[i];
        if (!((tv > sm.botv[i]) && (tv > -1e8f))) continue;  // :135
        const int j = sm.tops[i], s = sm.bots[i];
        copy_row_part<HD>(sm.ak, s, sm.kr, j, lane);
        copy_row_part<HD>(sm.av, s, sm.vv, j, lane);
        if (lane == 0) {
          sm.pm[s] = sm.pos[j];
          sm.mass[s] = 1.f;
          sm.util[s] = sm.rel[j];
          sm.ins[j] = 1;
          sm.dirty[s] = 1;
        }
      }
      __syncthreads();
      // ---- Gershgorin-normalised delta rule into M_res (:154-162)
      for (int j = tid; j < CC; j += NT)
        sm.wgt[j] = (j < l_tok && !sm.mrg[j] && !sm.ins[j]) ? sm.beta[j] : 0.f;
      __syncthreads();
      float bsafe0, bsafe1;
      {
        float acc[16][4];
        gemm_nt<HD>(acc, sm.kr, r0, sm.kr, lane);
        const float rk0 = sm.rnk[r0 + g], rk1 = sm.rnk[r0 + g + 8];
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int n = 0; n < 16; ++n) {
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const int col = n * 8 + 2 * t4 + q;
            const float rb = sm.rnk[col];
            const float w = sm.wgt[col];
            s0 = fmaf(fabsf(__fmul_rn(acc[n][q], __fmul_rn(rk0, rb))), w, s0);
            s1 = fmaf(fabsf(__fmul_rn(acc[n][2 + q], __fmul_rn(rk1, rb))), w, s1);
          }
        }
        s0 = fmaxf(quad_sum(s0), 1.0f);
        s1 = fmaxf(quad_sum(s1), 1.0f);
        bsafe0 = __fdiv_rn(sm.wgt[r0 + g], s0);
        bsafe1 = __fdiv_rn(sm.wgt[r0 + g + 8], s1);
      }
      // M split into two bf16 terms, stored [d_in][d_out] in x1 (hi) and x2 (lo)
      if (m_owner) {
#pragma unroll
        for (int n = 0; n < HD / 8; ++n) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int row = r0 + g + (q >> 1) * 8, col = n * 8 + 2 * t4 + (q & 1);
            const bf16 hi = __float2bfloat16_rn(mr[n][q]);
            sm.x1[swz<HD>(row, col)] = hi;
            sm.x2[swz<HD>(row, col)] = __float2bfloat16_rn(mr[n][q] - bf2f(hi));
          }
        }
      }
      __syncthreads();
      float err[HD / 8][4];
      {
#pragma unroll
        for (int n = 0; n < HD / 8; ++n) err[n][0] = err[n][1] = err[n][2] = err[n][3] = 0.f;
        gemm_nn<HD>(err, sm.kr, r0, sm.x1, lane);
        gemm_nn<HD>(err, sm.kr, r0, sm.x2, lane);
        const float rk0 = sm.rnk[r0 + g], rk1 = sm.rnk[r0 + g + 8];
#pragma unroll
        for (int n = 0; n < HD / 8; ++n) {
#pragma unroll
          for (int hr = 0; hr < 2; ++hr) {
            const int row = r0 + g + hr * 8, col = n * 8 + 2 * t4;
            const float rk = hr ? rk1 : rk0;
            const float bs = hr ? bsafe1 : bsafe0;
            const float2 vv = unpack_bf16(*reinterpret_cast<const uint32_t*>(&sm.vv[swz<HD>(row, col)]));
            const float e0 = __fmul_rn(vv.x - __fmul_rn(err[n][2 * hr], rk), bs);
            const float e1 = __fmul_rn(vv.y - __fmul_rn(err[n][2 * hr + 1], rk), bs);
            err[n][2 * hr] = __fmul_rn(e0, rk);  // E = err / |k| so that kr^T E = k^T err
            err[n][2 * hr + 1] = __fmul_rn(e1, rk);
          }
        }
      }
      __syncthreads();  // every warp is done reading the M split
#pragma unroll
      for (int n = 0; n < HD / 8; ++n) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int row = r0 + g + (q >> 1) * 8, col = n * 8 + 2 * t4 + (q & 1);
          const bf16 hi = __float2bfloat16_rn(err[n][q]);
          sm.x1[swz<HD>(row, col)] = hi;
          sm.x2[swz<HD>(row, col)] = __float2bfloat16_rn(err[n][q] - bf2f(hi));
        }
      }
      __syncthreads();
      if (m_owner) {
#pragma unroll
        for (int n = 0; n < HD / 8; ++n) {
          mr[n][0] = __fmul_rn(mr[n][0], gam); mr[n][1] = __fmul_rn(mr[n][1], gam);
          mr[n][2] = __fmul_rn(mr[n][2], gam); mr[n][3] = __fmul_rn(mr[n][3], gam);
        }
        gemm_tn<HD>(mr, sm.kr, r0, sm.x1, lane);
        gemm_tn<HD>(mr, sm.kr, r0, sm.x2, lane);
      }
      __syncthreads();
    }

    // ---- state the attention of a later chunk reads: RoPE(ak, pm), av, mass, act, M_res. The
    // shared-memory tiles already have the operand layout the attention's tensor cores read, so
    // the snapshot is a handful of bulk copies: k_read (x2), av, M_hi (rebuilt in x1), M_lo (kr).
    // k_read: last step's, from tensor memory, with the slots this step changed recomputed.
    x2_restore();
    if (warp == 0) {
      int base = 0;
      for (int s0 = 0; s0 < S; s0 += 32) {
        const bool dd = sm.dirty[s0 + lane] != 0;
        const unsigned bal = __ballot_sync(0xffffffffu, dd);
        if (dd) sm.dlist[base + __popc(bal & ((1u << lane) - 1))] = s0 + lane;
        base += __popc(bal);
        sm.dirty[s0 + lane] = 0;
      }
      if (lane == 0) sm.n_dirty = base;
    }
    __syncthreads();
    rope_slots(sm.n_dirty, [&](int i) { return sm.dlist[i]; });
    if (a.snap_ak_rope && m_owner) {
#pragma unroll
      for (int n = 0; n < HD / 8; ++n) {
#pragma unroll
        for (int hrow = 0; hrow < 2; ++hrow) {
          const int d = r0 + g + hrow * 8, e = n * 8 + 2 * t4;
          const float m0 = mr[n][2 * hrow], m1 = mr[n][2 * hrow + 1];
          const bf16 h0 = __float2bfloat16_rn(m0), h1 = __float2bfloat16_rn(m1);
          *reinterpret_cast<uint32_t*>(&sm.x1[swz<HD>(d, e)]) = pack_bf16(bf2f(h0), bf2f(h1));
          *reinterpret_cast<uint32_t*>(&sm.kr[swz<HD>(d, e)]) = pack_bf16(m0 - bf2f(h0), m1 - bf2f(h1));
        }
      }
    }
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    __syncthreads();
    x2_save();
    if (a.snap_ak_rope) {
      const int64_t sn = (int64_t)c * a.snap_cap + a.snap0 + st;
      constexpr uint32_t kTile = 128 * HD * 2;
      if (tid == 0) {
        unsigned char* gm = reinterpret_cast<unsigned char*>(a.snap_m) + sn * (int64_t)HD * HD * 4;
        bulk_s2g(reinterpret_cast<unsigned char*>(a.snap_ak_rope) + sn * kTile, sm.x2, kTile);
        bulk_s2g(reinterpret_cast<unsigned char*>(a.snap_av) + sn * kTile, sm.av, kTile);
        bulk_s2g(gm, sm.x1, (uint32_t)HD * HD * 2);
        bulk_s2g(gm + (int64_t)HD * HD * 2, sm.kr, (uint32_t)HD * HD * 2);
        asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
      }
      for (int s = tid; s < S; s += NT) {
        a.snap_mass[sn * S + s] = sm.mass[s];
        a.snap_act[sn * S + s] = sm.act[s];
      }
      // the next step overwrites these tiles: wait until the copies have read them
      if (tid == 0) asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory");
      __syncthreads();
    }
  }

  // ---- write the bank back
  s2g_rows<HD>(g_ak, sm.ak);
  s2g_rows<HD>(g_av, sm.av);
  if (a.ak_rope) s2g_rows<HD>(reinterpret_cast<bf16*>(a.ak_rope) + (int64_t)c * S * HD, sm.x2);
  for (int s = tid; s < S; s += NT) {
    a.mass[(int64_t)c * S + s] = sm.mass[s];
    a.util[(int64_t)c * S + s] = sm.util[s];
    a.pm[(int64_t)c * S + s] = sm.pm[s];
    a.act[(int64_t)c * S + s] = sm.act[s];
  }
  if (m_owner) {
#pragma unroll
    for (int n = 0; n < HD / 8; ++n) {
      *reinterpret_cast<float2*>(g_m + (r0 + g) * HD + n * 8 + 2 * t4) = make_float2(mr[n][0], mr[n][1]);
      *reinterpret_cast<float2*>(g_m + (r0 + g + 8) * HD + n * 8 + 2 * t4) = make_float2(mr[n][2], mr[n][3]);
    }
  }
  if (tid == 0) {
    a.n_filled[c] = n_filled;
    asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory");  // snapshot copies have landed
  }
  tc5::fence_before_sync();
  __syncthreads();
  tc5::fence_after_sync();
  if (warp == 0) tc5::tmem_dealloc(sm.tbase, 64);
}

template <int HD>
int launch(const bolt3_consolidate_args& a, cudaStream_t s) {
  const size_t smem = sizeof(Smem<HD>);
  // the attribute is per function and per device; setting it again is harmless
  if (cudaFuncSetAttribute(consolidate_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return BOLT3_ERR_CUDA;
  consolidate_kernel<HD><<<a.n_chains, NT, smem, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? BOLT3_OK : BOLT3_ERR_CUDA;
}

}  // namespace

extern "C" int bolt3_consolidate(const bolt3_consolidate_args* a, void* stream) {
  if (!a || !a->ak || !a->av || !a->mass || !a->util || !a->pm || !a->act || !a->m_res ||
      !a->n_filled || !a->kr || !a->kp || !a->v || !a->beta || !a->kappa || !a->gamma || !a->inv_freq)
    return BOLT3_ERR_ARG;
  if (a->n_chains <= 0 || a->hkv <= 0 || a->n_steps < 0) return BOLT3_ERR_SHAPE;
  if (a->chunk_len <= 0 || a->chunk_len > CC || a->skip0 < 0 || a->skip0 >= a->chunk_len)
    return BOLT3_ERR_SHAPE;
  if (a->snap_ak_rope && (!a->snap_av || !a->snap_mass || !a->snap_act || !a->snap_m ||
                          a->snap0 < 0 || a->snap0 + a->n_steps > a->snap_cap))
    return BOLT3_ERR_CAPACITY;
  if (a->n_steps > 0 &&
      a->token0 + (int64_t)(a->n_steps - 1) * a->step_tokens + a->chunk_len > a->chain_tokens)
    return BOLT3_ERR_CAPACITY;
  const uintptr_t al = (uintptr_t)a->ak | (uintptr_t)a->av | (uintptr_t)a->kr | (uintptr_t)a->kp |
                       (uintptr_t)a->v | (uintptr_t)a->ak_rope | (uintptr_t)a->snap_ak_rope |
                       (uintptr_t)a->snap_av | (uintptr_t)a->m_res | (uintptr_t)a->snap_m;
  if (al & 15) return BOLT3_ERR_ALIGN;
  if (a->n_steps == 0) return BOLT3_OK;
  cudaStream_t s = (cudaStream_t)stream;
  if (a->HD == 128) return launch<128>(*a, s);
  if (a->HD == 64) return launch<64>(*a, s);
  return BOLT3_ERR_SHAPE;
}
