// Phase B: the sequential attractor-bank / M_res consolidation scan.
//
// One CTA (8 warps) owns one chain (sequence b, KV head h) for all of its consolidation steps, so
// the bank never leaves the SM between steps: ak / av live in shared memory, M_res (fp32) lives in
// tensor memory as the accumulator of its own update. Every contraction of _consolidate_functional
// (vsa_lm/config/bolt3.py:68-192) is a tcgen05.mma over 128-byte-swizzled shared-memory tiles with
// bf16 operands and fp32 accumulation in tensor memory:
//   sc   = kp . RoPE(ak, pm)^T            (:97-100, :169-171)   exact bf16 products
//   v^   = softmax(sc).bf16 @ av          (:101, :172)          P written to tensor memory
//   cos  = kr . ak^T / (|kr| |ak|)        (:104-106, :175-176)
//   pair = ak . ak^T / (|ak| |ak|)        (:128-130)
//   gram = |kr . kr^T| / (|kr| |kr|)      (:156-157)
//   k^ M = kr . (M_hi + M_lo) / |kr|      (:159)   M split into two bf16 terms: ~2^-17 relative
//   M   <- gamma M + kr^T . (E_hi + E_lo)  (:162)   E = err / |kr|, split the same way
// Thread 0 issues the MMAs; the row-wise work that follows each one (softmax, argmax, maxima, sums,
// the error rows) reads tensor-memory lanes, one thread per row and column half. Rankings count,
// per entry, the entries that sort before it (128 threads, one entry each); when exactly equal keys
// decide the result the CPU torch.topk order is reproduced with the emulation in stl_select.h
// (bolt3.py:133-134, 183).
#include "../../include/bolt3.h"
#include "common.cuh"
#include "trace.h"
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
struct __align__(1024) Smem {
  bf16 ak[S * HD];     // every tile: 128 rows, 128-byte-swizzled blocks of 64 columns (tcgen05 operands)
  bf16 av[S * HD];
  bf16 kr[CC * HD];
  bf16 vv[CC * HD];
  bf16 x1[128 * HD];   // kp, then M_hi, then E_hi
  bf16 x2[128 * HD];   // RoPE(ak, pm), then M_lo, then E_lo
  bf16 zpad[HD == 64 ? 128 * 64 : 8];  // HD = 64: zero rows 64..127 of the M update's A operand
  float mass[S], util[S], pm[S], keep[S], na[S], rna[S], bias[S], botv[S];
  float rel[CC], score[CC], bsk[CC], beta[CC], nk[CC], rnk[CC], nv[CC], pos[CC], wgt[CC], topv[CC], bsafe[CC];
  float red[2][128], red2[2][128];  // per-row partial results of the two column halves
  int redi[2][128];
  int best[CC], tops[CC], bots[S], mlist[CC], mbest[CC], hlist[S];
  unsigned char act[S], mrg[CC], ins[CC], hit[S];
  int n_merged, n_hit;
  b3sel::KV selA[128], selB[128];
  alignas(16) uint32_t keys[2][128];   // ranking scratch of the two thread groups (read as uint4)
  unsigned char dirty[S];   // slots whose key or mean position changed this step
  int dlist[S], n_dirty;
  uint64_t bar[2];          // MMA completion: results in D1 (bar[0]); in D2 or M (bar[1])
  uint32_t tbase;
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

// tensor-memory columns: M_res, the RoPE(ak, pm) cache, two fp32 result tiles, P (bf16 pairs)
constexpr uint32_t TM_M = 0, TM_X2 = 128, TM_D1 = 192, TM_D2 = 320, TM_P = 448;
constexpr uint32_t kWaitIters = 1u << 24;

template <int HD>
__global__ void __launch_bounds__(NT, 1) consolidate_kernel(bolt3_consolidate_args a) {
  extern __shared__ unsigned char smem_raw[];
  Smem<HD>& sm = *reinterpret_cast<Smem<HD>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int c = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (a.wait_probe) {  // failure-path test hook: an expired bounded wait, reported as bit 4
    if (tid == 0 && !tc5::probe_wait(&sm.bar[0], a.wait_probe) && a.status) atomicOr(a.status, 4);
    return;
  }
  const int h = c % a.hkv;
  const float kappa = a.kappa[h];
  const float gam = a.gamma[h];
  constexpr float scale = HD == 128 ? 0.08838834764831845f : 0.125f;  // fp32(HD ** -0.5)
  // row view of tensor memory: this thread owns row (lane) `row` and column half `half`
  const int row = 32 * (warp & 3) + lane, half = warp >> 2;
  const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
  constexpr int HH = HD / 2;  // columns of an HD-wide tile per half

  bf16* g_ak = reinterpret_cast<bf16*>(a.ak) + (int64_t)c * S * HD;
  bf16* g_av = reinterpret_cast<bf16*>(a.av) + (int64_t)c * S * HD;
  float* g_m = a.m_res + (int64_t)c * HD * HD;

  // ---- tensor memory, barriers
  if (warp == 0) {
    tc5::tmem_alloc(&sm.tbase, 512);
    tc5::tmem_relinquish();
  }
  if (tid == 0) {
    tc5::mbar_init(&sm.bar[0], 1);
    tc5::mbar_init(&sm.bar[1], 1);
    tc5::mbar_fence_init();
  }
  if constexpr (HD == 64)
    for (int i = tid; i < 128 * 64 / 8; i += NT) reinterpret_cast<uint4*>(sm.zpad)[i] = make_uint4(0, 0, 0, 0);
  for (int s2 = tid; s2 < S; s2 += NT) sm.dirty[s2] = 0;
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
  tc5::fence_before_sync();
  __syncthreads();
  tc5::fence_after_sync();
  const uint32_t tb = sm.tbase;
  uint32_t ph[2] = {0u, 0u};
  bool timed_out = false;
  auto wait_mma = [&](int i) {
    if (!tc5::mbar_wait(&sm.bar[i], ph[i], kWaitIters)) timed_out = true;
    ph[i] ^= 1u;
    tc5::fence_after_sync();
  };
  // every thread's shared-memory and tensor-memory writes are visible to the MMAs issued next
  auto handoff = [&]() {
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    tc5::fence_before_sync();
    __syncthreads();
    tc5::fence_after_sync();
  };
  // 32-column tensor-memory access of this thread's row
  auto tld = [&](uint32_t col, uint32_t (&v)[32]) { tc5::ld32(tb + lane_off + col, v); };
  auto tst = [&](uint32_t col, const uint32_t (&v)[32]) { tc5::st32(tb + lane_off + col, v); };

  // ---- MMA issue (thread 0). Tiles are [128 rows][HD] in 64-column blocks of 16 KB.
  const uint32_t s_ak = tc5::smem_u32(sm.ak), s_av = tc5::smem_u32(sm.av), s_kr = tc5::smem_u32(sm.kr);
  const uint32_t s_x1 = tc5::smem_u32(sm.x1), s_x2 = tc5::smem_u32(sm.x2);
  // D[128 x 128] = A . B^T, both K-major (K = HD)
  auto mma_abt = [&](uint32_t dcol, uint32_t sa, uint32_t sb) {
    constexpr uint32_t id = tc5::idesc_bf16(128, 128, false, false);
    for (int ks = 0; ks < HD / 16; ++ks) {
      const uint32_t off = (ks >> 2) * 16384 + (ks & 3) * 32;
      tc5::mma_ss(tb + dcol, tc5::sdesc(sa + off, 16, 1024), tc5::sdesc(sb + off, 16, 1024), id, ks > 0);
    }
  };
  // D[128 x HD] (+)= A . B, A K-major [128][HD], B [HD rows = K][HD columns = N] (MN-major)
  auto mma_ab = [&](uint32_t dcol, uint32_t sa, uint32_t sb, bool acc) {
    constexpr uint32_t id = tc5::idesc_bf16(128, HD, false, true);
    for (int ks = 0; ks < HD / 16; ++ks) {
      const uint32_t off = (ks >> 2) * 16384 + (ks & 3) * 32;
      tc5::mma_ss(tb + dcol, tc5::sdesc(sa + off, 16, 1024), tc5::sdesc(sb + ks * 2048, 16384, 1024), id,
                  acc || ks > 0);
    }
  };

  // fp32 M_res staged in x1..x2 (64 KB at HD = 128, 16 KB at 64: x1 and x2 are consecutive): row r,
  // 16-byte chunk ch at chunk ch ^ (r & 7), so that a warp's 32 rows read or write one chunk each
  // without bank conflicts
  float* const m_stage = reinterpret_cast<float*>(sm.x1);
  auto m_swz = [](int r, int ch) { return r * HD + ((ch ^ (r & 7)) << 2); };

  // ---- load or initialise the bank (bolt3.py:83-92); M_res into tensor memory rows d
  int n_filled;
  if (a.init_blank) {
    n_filled = 0;
    for (int i = tid; i < S * HD / 8; i += NT) {
      *reinterpret_cast<uint4*>(sm.ak + i * 8) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(sm.av + i * 8) = make_uint4(0, 0, 0, 0);
    }
    for (int s2 = tid; s2 < S; s2 += NT) {
      sm.mass[s2] = 1.f; sm.util[s2] = 0.f; sm.pm[s2] = 0.f; sm.act[s2] = 0;
    }
  } else {
    n_filled = a.n_filled[c];
    g2s_rows<HD>(sm.ak, g_ak, S);
    g2s_rows<HD>(sm.av, g_av, S);
    // M_res through shared memory (x1, x2 are free until the chunk arrives): coalesced copies in,
    // then each thread takes its row (below)
    for (int i = tid; i < HD * HD / 4; i += NT) {
      const int r = i / (HD / 4), ch = i % (HD / 4);
      cp_async16(m_stage + m_swz(r, ch), g_m + (int64_t)r * HD + ch * 4, true);
    }
    cp_async_commit();
    for (int s2 = tid; s2 < S; s2 += NT) {
      sm.mass[s2] = a.mass[(int64_t)c * S + s2];
      sm.util[s2] = a.util[(int64_t)c * S + s2];
      sm.pm[s2] = a.pm[(int64_t)c * S + s2];
      sm.act[s2] = a.act[(int64_t)c * S + s2];
    }
    cp_async_wait<0>();
  }
  __syncthreads();
#pragma unroll
  for (int q = 0; q < HH / 32; ++q) {
    uint32_t v[32];
#pragma unroll
    for (int c4 = 0; c4 < 8; ++c4) {
      float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
      if (!a.init_blank && row < HD) f = *reinterpret_cast<const float4*>(m_stage + m_swz(row, (half * HH + q * 32) / 4 + c4));
      v[4 * c4] = __float_as_uint(f.x);
      v[4 * c4 + 1] = __float_as_uint(f.y);
      v[4 * c4 + 2] = __float_as_uint(f.z);
      v[4 * c4 + 3] = __float_as_uint(f.w);
    }
    tst(TM_M + half * HH + q * 32, v);
  }
  tc5::st_wait();
  __syncthreads();

  // RoPE(ak, pm) of slots slot_of(0 .. n_slots-1) into x2 (bolt3.py:17-20 in the storage dtype: cos
  // and sin rounded, every product and sum rounded), two frequencies per item so that each pair of
  // roundings is one conversion
  auto rope_slots = [&](int n_slots, auto slot_of) {
    for (int i = tid; i < n_slots * (HD / 4); i += NT) {
      const int s2 = slot_of(i / (HD / 4)), d = (i % (HD / 4)) * 2;
      float sn0, cs0, sn1, cs1;
      sincosf(__fmul_rn(sm.pm[s2], a.inv_freq[d]), &sn0, &cs0);
      sincosf(__fmul_rn(sm.pm[s2], a.inv_freq[d + 1]), &sn1, &cs1);
      uint32_t t;
      const float2 cs = rbf2(cs0, cs1, t), sn = rbf2(sn0, sn1, t);
      const float2 x0 = unpack_bf16(*reinterpret_cast<const uint32_t*>(&sm.ak[swz<HD>(s2, d)]));
      const float2 x1 = unpack_bf16(*reinterpret_cast<const uint32_t*>(&sm.ak[swz<HD>(s2, d + HD / 2)]));
      const float2 a0 = rbf2(__fmul_rn(x0.x, cs.x), __fmul_rn(x0.y, cs.y), t);
      const float2 b0 = rbf2(__fmul_rn(-x1.x, sn.x), __fmul_rn(-x1.y, sn.y), t);
      const float2 a1 = rbf2(__fmul_rn(x1.x, cs.x), __fmul_rn(x1.y, cs.y), t);
      const float2 b1 = rbf2(__fmul_rn(x0.x, sn.x), __fmul_rn(x0.y, sn.y), t);
      *reinterpret_cast<uint32_t*>(&sm.x2[swz<HD>(s2, d)]) = pack_bf16(__fadd_rn(a0.x, b0.x), __fadd_rn(a0.y, b0.y));
      *reinterpret_cast<uint32_t*>(&sm.x2[swz<HD>(s2, d + HD / 2)]) =
          pack_bf16(__fadd_rn(a1.x, b1.x), __fadd_rn(a1.y, b1.y));
    }
  };
  // x2 <-> tensor memory between steps (x2 is scratch inside a step): this thread moves its row,
  // its half of the columns (HD/4 32-bit words)
  constexpr int NW2 = HD / 4;
  auto x2_save = [&]() {
    uint32_t w[NW2];
#pragma unroll
    for (int q = 0; q < NW2 / 4; ++q) {
      const uint4 u = *reinterpret_cast<const uint4*>(&sm.x2[swz<HD>(row, half * HH + q * 8)]);
      w[4 * q] = u.x; w[4 * q + 1] = u.y; w[4 * q + 2] = u.z; w[4 * q + 3] = u.w;
    }
    if constexpr (NW2 == 32) tc5::st32(tb + lane_off + TM_X2 + half * NW2, w);
    else tc5::st16(tb + lane_off + TM_X2 + half * NW2, w);
    tc5::st_wait();
  };
  auto x2_restore = [&]() {
    uint32_t w[NW2];
    tc5::ld_cols(tb + lane_off + TM_X2 + half * NW2, w);
    tc5::ld_wait();
#pragma unroll
    for (int q = 0; q < NW2 / 4; ++q)
      *reinterpret_cast<uint4*>(&sm.x2[swz<HD>(row, half * HH + q * 8)]) =
          make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
  };
  // M_res (tensor memory) split into two bf16 terms, written as [d][e] operand images
  auto m_split = [&](bf16* hi_t, bf16* lo_t) {
    if (row < HD) {
#pragma unroll
      for (int q = 0; q < HH / 32; ++q) {
        uint32_t v[32];
        tld(TM_M + half * HH + q * 32, v);
        tc5::ld_wait();
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
          uint32_t hw[4], lw[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float m0 = __uint_as_float(v[ch * 8 + 2 * u]), m1 = __uint_as_float(v[ch * 8 + 2 * u + 1]);
            const float2 hh = rbf2(m0, m1, hw[u]);
            lw[u] = pack_bf16(m0 - hh.x, m1 - hh.y);
          }
          const int col = half * HH + q * 32 + ch * 8;
          *reinterpret_cast<uint4*>(&hi_t[swz<HD>(row, col)]) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
          *reinterpret_cast<uint4*>(&lo_t[swz<HD>(row, col)]) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
      }
    }
  };
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
    for (int s2 = tid; s2 < S; s2 += NT) sm.util[s2] = __fmul_rn(sm.util[s2], GAMMA_U);  // :94
    cp_async_wait<0>();
    handoff();
    {
      // row norms of the chunk keys / values and of the slot keys: two threads per row
      const int r = tid >> 1, hf = tid & 1;
      float kk = half_row_dot<HD>(sm.kr, sm.kr, r, hf);
      float vv2 = half_row_dot<HD>(sm.vv, sm.vv, r, hf);
      float aa = half_row_dot<HD>(sm.ak, sm.ak, r, hf);
      kk += __shfl_xor_sync(0xffffffffu, kk, 1);
      vv2 += __shfl_xor_sync(0xffffffffu, vv2, 1);
      aa += __shfl_xor_sync(0xffffffffu, aa, 1);
      if (hf == 0) {
        sm.nk[r] = sqrtf(kk);
        sm.nv[r] = sqrtf(vv2);
        sm.na[r] = sqrtf(aa);
        // F.normalize divides by max(|x|, 1e-12); the contractions multiply by the reciprocal
        sm.rnk[r] = 1.0f / fmaxf(sm.nk[r], 1e-12f);
        sm.rna[r] = 1.0f / fmaxf(sm.na[r], 1e-12f);
      }
    }
    const bool full = n_filled >= S;
    if (n_filled > 0) {
      // attractor prediction: sc = kp . RoPE(ak)^T into D1
      if (tid == 0) {
        mma_abt(TM_D1, s_x1, s_x2);
        tc5::commit(&sm.bar[0]);
      }
      for (int s2 = tid; s2 < S; s2 += NT) {
        const float lm = logf(fmaxf(sm.mass[s2], 1.0f));
        sm.bias[s2] = full ? __fmul_rn(kappa, lm) : lm;
      }
    }
    __syncthreads();

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
      // ---- attractor prediction of each token's value (:97-103 / :169-174): softmax over the
      // slots, P = bf16(p) into tensor memory
      wait_mma(0);
      {
        float x[64];
        {
          uint32_t v[32];
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            tld(TM_D1 + half * 64 + q * 32, v);
            tc5::ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int col = half * 64 + q * 32 + j;
              float sc = __fadd_rn(__fmul_rn(__uint_as_float(v[j]), scale), sm.bias[col]);
              if (!full && !sm.act[col]) sc = -1e9f;
              x[q * 32 + j] = sc;
            }
          }
        }
        float mx = x[0];
#pragma unroll
        for (int j = 1; j < 64; ++j) mx = fmaxf(mx, x[j]);
        sm.red[half][row] = mx;
        __syncthreads();
        mx = fmaxf(sm.red[0][row], sm.red[1][row]);
        float sum = 0.f;
#pragma unroll
        for (int j = 0; j < 64; ++j) {
          x[j] = expf(x[j] - mx);
          sum += x[j];
        }
        sm.red2[half][row] = sum;
        __syncthreads();
        const float inv = 1.0f / (sm.red2[0][row] + sm.red2[1][row]);
        uint32_t pk[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) pk[j] = pack_bf16(__fmul_rn(x[2 * j], inv), __fmul_rn(x[2 * j + 1], inv));
        tst(TM_P + half * 32, pk);
        tc5::st_wait();
      }
      handoff();
      if (tid == 0) {
        // v^ = P . av into D2; cos = kr . ak^T into D1
        constexpr uint32_t id = tc5::idesc_bf16(128, HD, false, true);
        for (int ks = 0; ks < S / 16; ++ks)
          tc5::mma_ts(tb + TM_D2, tb + TM_P + ks * 8, tc5::sdesc(s_av + ks * 2048, 16384, 1024), id, ks > 0);
        tc5::commit(&sm.bar[1]);
        mma_abt(TM_D1, s_kr, s_ak);
        tc5::commit(&sm.bar[0]);
      }
      // rel_err = |v - v^| / (|v| + 1e-6)
      wait_mma(1);
      {
        float e = 0.f;
#pragma unroll
        for (int q = 0; q < HH / 32; ++q) {
          uint32_t v[32];
          tld(TM_D2 + half * HH + q * 32, v);
          tc5::ld_wait();
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) {
            const uint4 u = *reinterpret_cast<const uint4*>(&sm.vv[swz<HD>(row, half * HH + q * 32 + ch * 8)]);
            const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int w2 = 0; w2 < 4; ++w2) {
              const float2 vf = unpack_bf16(uw[w2]);
              float d = vf.x - __uint_as_float(v[ch * 8 + 2 * w2]);
              e = fmaf(d, d, e);
              d = vf.y - __uint_as_float(v[ch * 8 + 2 * w2 + 1]);
              e = fmaf(d, d, e);
            }
          }
        }
        sm.red[half][row] = e;
      }
      // cosine match against the slots (:104-106, :175-177): best slot, first index on ties
      wait_mma(0);
      {
        const float rk = sm.rnk[row];
        float b = neg_inf();
        int bi = 0x7fffffff;
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          uint32_t v[32];
          tld(TM_D1 + half * 64 + q * 32, v);
          tc5::ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int col = half * 64 + q * 32 + j;
            float cv = __fmul_rn(__uint_as_float(v[j]), __fmul_rn(rk, sm.rna[col]));
            if (!full && !sm.act[col]) cv = 0.f;
            if (cv > b) { b = cv; bi = col; }
          }
        }
        sm.red2[half][row] = b;
        sm.redi[half][row] = bi;
      }
      tc5::fence_before_sync();
      __syncthreads();
      tc5::fence_after_sync();
      if (half == 0) {
        sm.rel[row] = __fdiv_rn(sqrtf(sm.red[0][row] + sm.red[1][row]), __fadd_rn(sm.nv[row], 1e-6f));
        const float b0 = sm.red2[0][row], b1 = sm.red2[1][row];
        const bool second = b1 > b0;
        sm.bsk[row] = second ? b1 : b0;
        sm.best[row] = second ? sm.redi[1][row] : sm.redi[0][row];
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
        const int j = sm.tops[i], s2 = n_filled + i;
        copy_row_part<HD>(sm.ak, s2, sm.kr, j, lane);
        copy_row_part<HD>(sm.av, s2, sm.vv, j, lane);
        if (lane == 0) {
          sm.pm[s2] = sm.pos[j];
          sm.mass[s2] = 1.f;
          sm.util[s2] = sm.rel[j];
          sm.act[s2] = 1;
          sm.dirty[s2] = 1;
        }
      }
      n_filled += m;
      __syncthreads();
    } else {
      // ---- sim_v, score, merge mask (:107-110): two threads per row
      {
        const int r = tid >> 1, hf = tid & 1;
        const int sb = sm.best[r];
        float dot = 0.f, aa = 0.f;
        if (r < l_tok) {
          constexpr int CPR = HD / 8;
#pragma unroll
          for (int hh = 0; hh < CPR / 2; ++hh) {
            // logical chunk ch of row r sits at physical chunk ch ^ (row & 7)
            const int ch = hf * CPR / 2 + hh;
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
        if (hf == 0 && r < l_tok) {
          const float sv = __fdiv_rn(dot, __fmul_rn(fmaxf(sm.nv[r], 1e-8f), fmaxf(sqrtf(aa), 1e-8f)));
          const float bs = sm.bsk[r];
          sm.score[r] = __fmul_rn(sm.rel[r], 1.0f - fminf(fmaxf(bs, 0.f), 1.f));
          sm.mrg[r] = (bs >= SIM_K) && (sv >= SIM_V);
        }
      }
      __syncthreads();
      // ---- merge: running means of the matched slots (:112-123). The merged tokens are listed in
      // token order, each with its slot; each slot that receives tokens is one warp's, which sums
      // them in token order.
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
      for (int s2 = tid; s2 < S; s2 += NT) sm.hit[s2] = 0;
      __syncthreads();
      const int n_m = sm.n_merged;
      if (n_m > 0) {
        for (int q = tid; q < n_m; q += NT) {
          const int sb = sm.best[sm.mlist[q]];
          sm.mbest[q] = sb;
          sm.hit[sb] = 1;
        }
        __syncthreads();
        if (warp == 0) {
          int base = 0;
          for (int s0 = 0; s0 < S; s0 += 32) {
            const bool hh = sm.hit[s0 + lane] != 0;
            const unsigned bal = __ballot_sync(0xffffffffu, hh);
            if (hh) sm.hlist[base + __popc(bal & ((1u << lane) - 1))] = s0 + lane;
            base += __popc(bal);
          }
          if (lane == 0) sm.n_hit = base;
        }
        __syncthreads();
        for (int hi = warp; hi < sm.n_hit; hi += 8) {
          const int s2 = sm.hlist[hi];
          constexpr int EPL = HD / 32;
          float ks[EPL], vs[EPL];
          float ps = 0.f;
          int cnt = 0;
#pragma unroll
          for (int e = 0; e < EPL; ++e) ks[e] = vs[e] = 0.f;
          for (int q = 0; q < n_m; ++q) {
            if (sm.mbest[q] != s2) continue;
            const int j = sm.mlist[q];
            ++cnt;
#pragma unroll
            for (int e = 0; e < EPL; ++e) {
              ks[e] = __fadd_rn(ks[e], bf2f(sm.kr[swz<HD>(j, lane * EPL + e)]));
              vs[e] = __fadd_rn(vs[e], bf2f(sm.vv[swz<HD>(j, lane * EPL + e)]));
            }
            ps = __fadd_rn(ps, sm.pos[j]);
          }
          const float ms = sm.mass[s2];
          const float nm = __fadd_rn(ms, (float)cnt);
#pragma unroll
          for (int e = 0; e < EPL; ++e) {
            const int d = lane * EPL + e;
            const float ka = __fadd_rn(__fmul_rn(ms, bf2f(sm.ak[swz<HD>(s2, d)])), ks[e]);
            const float va = __fadd_rn(__fmul_rn(ms, bf2f(sm.av[swz<HD>(s2, d)])), vs[e]);
            sm.ak[swz<HD>(s2, d)] = __float2bfloat16_rn(__fdiv_rn(ka, nm));
            sm.av[swz<HD>(s2, d)] = __float2bfloat16_rn(__fdiv_rn(va, nm));
          }
          __syncwarp();
          const float aa = row_sumsq<HD>(sm.ak, s2, lane);
          if (lane == 0) {
            sm.pm[s2] = __fdiv_rn(__fadd_rn(__fmul_rn(ms, sm.pm[s2]), ps), nm);
            sm.mass[s2] = nm;
            sm.dirty[s2] = 1;
            sm.na[s2] = sqrtf(aa);
            sm.rna[s2] = 1.0f / fmaxf(sm.na[s2], 1e-12f);
          }
        }
      }
      // ---- diversity eviction (:125-152): pair = ak . ak^T into D1, and already the Gershgorin
      // gram = kr . kr^T (:156) into D2
      handoff();
      if (tid == 0) {
        mma_abt(TM_D1, s_ak, s_ak);
        tc5::commit(&sm.bar[0]);
        mma_abt(TM_D2, s_kr, s_kr);
        tc5::commit(&sm.bar[1]);
      }
      wait_mma(0);
      {
        const float ra = sm.rna[row];
        float m = neg_inf();
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          uint32_t v[32];
          tld(TM_D1 + half * 64 + q * 32, v);
          tc5::ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int col = half * 64 + q * 32 + j;
            // (ra_s * ra_s') is symmetric, so equal cosines of a mutual pair stay bit-identical
            float p = __fmul_rn(__uint_as_float(v[j]), __fmul_rn(ra, sm.rna[col]));
            if (col == row) p = -1.0f;
            m = fmaxf(m, p);
          }
        }
        sm.red[half][row] = m;
      }
      __syncthreads();
      if (half == 0) {
        const float m = fmaxf(sm.red[0][row], sm.red[1][row]);
        sm.keep[row] = __fmul_rn(sm.util[row], 1.0f - fminf(fmaxf(m, 0.f), 0.98f));
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
        const int j = sm.tops[i], s2 = sm.bots[i];
        copy_row_part<HD>(sm.ak, s2, sm.kr, j, lane);
        copy_row_part<HD>(sm.av, s2, sm.vv, j, lane);
        if (lane == 0) {
          sm.pm[s2] = sm.pos[j];
          sm.mass[s2] = 1.f;
          sm.util[s2] = sm.rel[j];
          sm.ins[j] = 1;
          sm.dirty[s2] = 1;
        }
      }
      __syncthreads();
      // ---- Gershgorin-normalised delta rule into M_res (:154-162)
      for (int j = tid; j < CC; j += NT)
        sm.wgt[j] = (j < l_tok && !sm.mrg[j] && !sm.ins[j]) ? sm.beta[j] : 0.f;
      __syncthreads();
      wait_mma(1);
      {
        const float rk0 = sm.rnk[row];
        float s0 = 0.f;
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          uint32_t v[32];
          tld(TM_D2 + half * 64 + q * 32, v);
          tc5::ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int col = half * 64 + q * 32 + j;
            s0 = fmaf(fabsf(__fmul_rn(__uint_as_float(v[j]), __fmul_rn(rk0, sm.rnk[col]))), sm.wgt[col], s0);
          }
        }
        sm.red[half][row] = s0;
      }
      // M split into x1 (hi) and x2 (lo) for k^ M
      m_split(sm.x1, sm.x2);
      handoff();
      if (half == 0) sm.bsafe[row] = __fdiv_rn(sm.wgt[row], fmaxf(sm.red[0][row] + sm.red[1][row], 1.0f));
      if (tid == 0) {
        mma_ab(TM_D1, s_kr, s_x1, false);
        mma_ab(TM_D1, s_kr, s_x2, true);
        tc5::commit(&sm.bar[0]);
      }
      __syncthreads();
      wait_mma(0);
      {
        // E = ((v - (kr . M) / |kr|) * beta_safe) / |kr|, so that kr^T E = k^T err; split into x1/x2
        const float rk = sm.rnk[row], bs = sm.bsafe[row];
#pragma unroll
        for (int q = 0; q < HH / 32; ++q) {
          uint32_t v[32];
          tld(TM_D1 + half * HH + q * 32, v);
          tc5::ld_wait();
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) {
            const int col = half * HH + q * 32 + ch * 8;
            const uint4 u = *reinterpret_cast<const uint4*>(&sm.vv[swz<HD>(row, col)]);
            const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
            uint32_t hw[4], lw[4];
#pragma unroll
            for (int w2 = 0; w2 < 4; ++w2) {
              const float2 vf = unpack_bf16(uw[w2]);
              const float e0 = __fmul_rn(__fmul_rn(vf.x - __fmul_rn(__uint_as_float(v[ch * 8 + 2 * w2]), rk), bs), rk);
              const float e1 = __fmul_rn(__fmul_rn(vf.y - __fmul_rn(__uint_as_float(v[ch * 8 + 2 * w2 + 1]), rk), bs), rk);
              const float2 hh = rbf2(e0, e1, hw[w2]);
              lw[w2] = pack_bf16(e0 - hh.x, e1 - hh.y);
            }
            *reinterpret_cast<uint4*>(&sm.x1[swz<HD>(row, col)]) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *reinterpret_cast<uint4*>(&sm.x2[swz<HD>(row, col)]) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
          }
        }
        // M <- gamma M (rows d; the padding rows of HD = 64 stay zero)
#pragma unroll
        for (int q = 0; q < HH / 32; ++q) {
          uint32_t v[32];
          tld(TM_M + half * HH + q * 32, v);
          tc5::ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(__fmul_rn(__uint_as_float(v[j]), gam));
          tst(TM_M + half * HH + q * 32, v);
        }
        tc5::st_wait();
      }
      handoff();
      if (tid == 0) {
        // M += kr^T . E_hi + kr^T . E_lo: A = kr read transposed (rows d = the MN-major M side; at
        // HD = 64 the second block of 64 rows is the zero tile), B = E [tokens][e]
        constexpr uint32_t id = tc5::idesc_bf16(128, HD, true, true);
        const uint32_t lbo_a = HD == 128 ? 16384u : tc5::smem_u32(sm.zpad) - s_kr;
        for (int hl = 0; hl < 2; ++hl) {
          const uint32_t sb = hl ? s_x2 : s_x1;
          for (int ks = 0; ks < CC / 16; ++ks)
            tc5::mma_ss(tb + TM_M, tc5::sdesc(s_kr + ks * 2048, lbo_a, 1024), tc5::sdesc(sb + ks * 2048, 16384, 1024),
                        id, 1u);
        }
        tc5::commit(&sm.bar[1]);
      }
      wait_mma(1);
    }

    // ---- state the attention of a later chunk reads: RoPE(ak, pm), av, mass, act, M_res. The
    // shared-memory tiles already have the operand layout the attention's tensor cores read, so
    // the snapshot is a handful of bulk copies: k_read (x2), av, M_hi (x1), M_lo (kr).
    // k_read: last step's, from tensor memory, with the slots this step changed recomputed.
    __syncthreads();
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
    if (a.snap_ak_rope) m_split(sm.x1, sm.kr);
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
      for (int s2 = tid; s2 < S; s2 += NT) {
        a.snap_mass[sn * S + s2] = sm.mass[s2];
        a.snap_act[sn * S + s2] = sm.act[s2];
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
  for (int s2 = tid; s2 < S; s2 += NT) {
    a.mass[(int64_t)c * S + s2] = sm.mass[s2];
    a.util[(int64_t)c * S + s2] = sm.util[s2];
    a.pm[(int64_t)c * S + s2] = sm.pm[s2];
    a.act[(int64_t)c * S + s2] = sm.act[s2];
  }
  if (row < HD) {
#pragma unroll
    for (int q = 0; q < HH / 32; ++q) {
      uint32_t v[32];
      tld(TM_M + half * HH + q * 32, v);
      tc5::ld_wait();
      float4* dst = reinterpret_cast<float4*>(g_m + (int64_t)row * HD + half * HH + q * 32);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        dst[j] = make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]), __uint_as_float(v[4 * j + 2]),
                             __uint_as_float(v[4 * j + 3]));
    }
  }
  if (tid == 0) {
    a.n_filled[c] = n_filled;
    asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory");  // snapshot copies have landed
    if (timed_out && a.status) atomicOr(a.status, 4);
  }
  tc5::fence_before_sync();
  __syncthreads();
  tc5::fence_after_sync();
  if (warp == 0) tc5::tmem_dealloc(tb, 512);
}

template <int HD>
int launch(const bolt3_consolidate_args& a, cudaStream_t s) {
  const size_t smem = sizeof(Smem<HD>) + 1024;  // + alignment of the tiles to 1024 bytes
  // the attribute is per function and per device; setting it again is harmless
  if (cudaFuncSetAttribute(consolidate_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return BOLT3_ERR_CUDA;
  consolidate_kernel<HD><<<a.n_chains, NT, smem, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? BOLT3_OK : BOLT3_ERR_CUDA;
}

}  // namespace

extern "C" int bolt3_consolidate(const bolt3_consolidate_args* a, void* stream) {
  const b3::TraceRange trace_range("bolt3_consolidate");
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
