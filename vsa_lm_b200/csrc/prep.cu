// Phase A epilogue: from the fused projection output to head-major q/k/v with RoPE and gates.
//
// Mirrors Bolt3Attn.head_qkv (vsa_lm/config/bolt3.py:59-66: per-head LlamaRMSNorm when qk_norm,
// surgery.py:43-53), LlamaRoPE (surgery.py:80-93) in the storage dtype (cos/sin cast to bf16, every
// product and the sum rounded to bf16), beta = sigmoid(beta_proj x) and eta = tanh(eta_proj x)
// (bolt3.py:198-199) computed from the bf16 logits and rounded to bf16.
//
// HBM-bound elementwise work with 16-byte loads and stores: a block takes 16 tokens (1 for small
// calls such as decode steps) and every head row of them; a head row of HD values is handled by HD/8 lanes, each owning 8 consecutive elements;
// the lane holding elements i and the lane holding i + HD/2 (the pair rotate-half RoPE couples) swap
// values with one shuffle. cos/sin are computed once per (token, frequency) into shared memory.
#include "../../include/bolt3.h"
#include "common.cuh"
#include "trace.h"

namespace {

using namespace b3;

template <int HD, int TB>
__global__ void __launch_bounds__(256) prep_kernel(const bolt3_prep_args a) {
  constexpr int LPR = HD / 8;          // lanes per head row
  constexpr int RPW = 32 / LPR;        // rows per warp pass
  constexpr int HALF = LPR / 2;        // lane offset between the RoPE partners
  constexpr int NW = 8;                // warps
  const int64_t n_tok = (int64_t)a.B * a.T;
  const int64_t tok0 = (int64_t)blockIdx.x * TB;  // this block's tokens: tok0 .. tok0 + ntb - 1
  const int ntb = (int)min((int64_t)TB, n_tok - tok0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane / LPR, l = lane % LPR;   // row slot within the warp, lane within the row
  const bool first = l < HALF;         // holds elements of the first half
  // the attention kernel that follows a decode step's prep may start its set-up now (it waits for
  // this grid's completion before it reads any of its outputs)
  grid_dep_launch();
  // device step position (a step replayed from a CUDA graph): shift the RoPE position and the k/v
  // write offset by d; a d outside the range the launch was checked for skips the step
  int64_t dpos = 0;
  if (a.pos_dev != nullptr) {
    dpos = *a.pos_dev - a.pos_ref;
    if (dpos < 0 || dpos >= a.pos_span) return;
  }
  const int64_t k_t_off = a.k_t_off + dpos, beta_t_off = a.beta_t_off + dpos;

  // bf16 cos/sin of the HD/2 frequencies for each of the block's tokens, shared by all their
  // heads, stored as pairs of adjacent frequencies (the operands of the packed RoPE below)
  __shared__ uint32_t s_cos[TB][HD / 4], s_sin[TB][HD / 4];
  // each token's sequence and position, once per block (64-bit divisions kept out of the item loop)
  __shared__ int s_b[TB], s_t[TB];
  for (int i = threadIdx.x; i < ntb; i += blockDim.x) {
    s_b[i] = (int)((tok0 + i) / a.T);
    s_t[i] = (int)((tok0 + i) % a.T);
  }
  for (int i = threadIdx.x; i < ntb * (HD / 4); i += blockDim.x) {
    const int tl = i / (HD / 4), fp = i % (HD / 4);
    const float pos = (float)(a.pos0 + dpos + (tok0 + tl) % a.T);
    float s0, c0, s1, c1;
    sincosf(__fmul_rn(pos, a.inv_freq[2 * fp]), &s0, &c0);
    sincosf(__fmul_rn(pos, a.inv_freq[2 * fp + 1]), &s1, &c1);
    s_cos[tl][fp] = pack_bf16(c0, c1);
    s_sin[tl][fp] = pack_bf16(s0, s1);
  }

  // head rows per token: [0, H) q when parts & 1, then HKV k and HKV v rows when parts & 2
  const bool do_q = a.parts & 1, do_kv = (a.parts & 2) != 0;
  const bool want_l2 = do_q && a.q_l2 != nullptr;
  const int n_rows = (do_q ? a.H : 0) + (do_kv ? 2 * a.HKV : 0);
  // one-token blocks (decode steps) split the token's rows over blockIdx.y, one warp pass each, so
  // that a block's work is one dependent pass; multi-token blocks take every row of their tokens
  constexpr int kRowGroup = NW * RPW;
  const int row_base = TB == 1 ? (int)blockIdx.y * kRowGroup : 0;
  const int n_items = TB == 1 ? min(kRowGroup, n_rows - row_base)
                              : ntb * n_rows;  // (token, row) pairs; consecutive rows of a token are adjacent
  // it / n_rows as a multiply and shift: with m = ceil(2^20 / n_rows), floor(it m / 2^20) is exact
  // for it * (m n_rows - 2^20) < 2^20, which holds for it < n_items (at most 16 tokens x a few
  // hundred rows; the launcher checks the bound)
  const uint32_t div_m = ((1u << 20) + (uint32_t)n_rows - 1) / (uint32_t)n_rows;
  auto token_of = [&](int it) { return (int)(((uint32_t)it * div_m) >> 20); };
  // this lane's eight RMSNorm weights of q and k rows (constant over the items)
  float wq[8], wk[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    wq[e] = a.q_norm_w != nullptr ? a.q_norm_w[l * 8 + e] : 0.f;
    wk[e] = a.k_norm_w != nullptr ? a.k_norm_w[l * 8 + e] : 0.f;
  }
  auto row_col = [&](int r, int& kind, int& head) -> int64_t {
    if (do_q && r < a.H) { kind = 0; head = r; return a.q_col + (int64_t)head * HD; }
    const int rk = r - (do_q ? a.H : 0);
    if (rk < a.HKV) { kind = 1; head = rk; return a.k_col + (int64_t)head * HD; }
    kind = 2; head = rk - a.HKV;
    return a.v_col + (int64_t)head * HD;
  };
  auto src = [&](int it) -> const uint4* {
    const int tl = token_of(it);
    int kd, hd_;
    const int64_t col = row_col(row_base + it - tl * n_rows, kd, hd_);
    return reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(a.proj) + (tok0 + tl) * a.ld + col + l * 8);
  };
  // the row item a lane handles in warp pass `pass`
  auto item = [&](int pass) { return warp * RPW + pass * NW * RPW + sub; };
  auto process = [&](int it, const uint4 u) {
    const bool live = it < n_items;
    const int tl = live ? token_of(it) : 0;
    const int b = s_b[tl], t = s_t[tl];
    int kind = 2, head = 0;  // 0 = q, 1 = k, 2 = v
    if (live) row_col(row_base + it - tl * n_rows, kind, head);
    float x[8];
    {
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = unpack_bf16(w[q]);
        x[2 * q] = f.x;
        x[2 * q + 1] = f.y;
      }
    }
    const int nh = kind == 0 ? a.H : a.HKV;
    const int64_t hs = kind == 0 ? a.q_head_stride : a.k_head_stride;
    const int64_t to = kind == 0 ? a.q_t_off : k_t_off;
    const int64_t off = (((int64_t)b * nh + head) * hs + to + t) * HD + l * 8;
    // per-row reductions stay inside the LPR lanes of the row
    auto row_sum = [&](float v) {
#pragma unroll
      for (int o = LPR / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      return v;
    };
    const bool has_norm = (kind == 0 ? a.q_norm_w : a.k_norm_w) != nullptr;
    // all lanes take part in the shuffles below, whatever their row's kind
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) ss = fmaf(x[e], x[e], ss);
    ss = row_sum(ss);
    // the stored row: the loaded bf16 values as they are, or their RMSNorm rounded to bf16
    uint32_t raw[4] = {u.x, u.y, u.z, u.w};
    if (kind != 2 && has_norm) {
      const float rr = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, (float)HD), a.eps));
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float w0 = kind == 0 ? wq[2 * q] : wk[2 * q], w1 = kind == 0 ? wq[2 * q + 1] : wk[2 * q + 1];
        const float2 r2 = rbf2(__fmul_rn(__fmul_rn(x[2 * q], rr), w0), __fmul_rn(__fmul_rn(x[2 * q + 1], rr), w1), raw[q]);
        x[2 * q] = r2.x;
        x[2 * q + 1] = r2.y;
      }
    }
    float l2 = 0.f;  // |q_raw| of the stored (bf16) row, for the M_res read-out
    if (want_l2) {   // uniform over the grid: every lane takes part in the shuffles
#pragma unroll
      for (int e = 0; e < 8; ++e) l2 = fmaf(x[e], x[e], l2);
      l2 = row_sum(l2);
    }
    // RoPE partner values (element i <-> i + HD/2), exchanged as the stored bf16 pairs
    uint32_t yp[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) yp[q] = __shfl_xor_sync(0xffffffffu, raw[q], HALF);
    if (!live) return;
    if (kind == 2) {
      *reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(a.v) + off) = make_uint4(raw[0], raw[1], raw[2], raw[3]);
      return;
    }
    if (kind == 0 && a.q_l2 != nullptr && l == 0)
      a.q_l2[((int64_t)b * a.H + head) * a.eta_head_stride + a.eta_t_off + t] = sqrtf(l2);
    const uint32_t* cs = &s_cos[tl][(l % HALF) * 4];  // frequency index: element index mod HD/2
    const uint32_t* sn = &s_sin[tl][(l % HALF) * 4];
    // rope = bf16(bf16(x cos) + bf16(partner sin)), two elements per packed bf16 operation: the
    // product of two bf16 values is exact in fp32, so one rounding of it is the reference's
    // fp32-product-then-bf16 value, and the sum of two bf16 values rounds the same way directly
    // or through fp32 (exact in fp32 unless one term is below the other's rounding unit, when both
    // give the larger). rotate_half: the first half pairs with -x[i + HD/2], the second with x[i - HD/2].
    uint32_t rot[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t ps = mul_bf16x2(yp[q], sn[q]);
      rot[q] = add_bf16x2(mul_bf16x2(raw[q], cs[q]), first ? neg_bf16x2(ps) : ps);
    }
    *reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(kind == 0 ? a.q_raw : a.k_raw) + off) =
        make_uint4(raw[0], raw[1], raw[2], raw[3]);
    *reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(kind == 0 ? a.q_rope : a.k_rope) + off) =
        make_uint4(rot[0], rot[1], rot[2], rot[3]);
  };
  // rolling prefetch: each lane keeps kPre 16-byte loads in flight (this kernel is bound by HBM
  // latency x bytes in flight); the load for pass p + kPre is issued before pass p is processed
  constexpr int kPre = 4;
  auto fetch = [&](int it) { return it < n_items ? *src(it) : make_uint4(0, 0, 0, 0); };
  uint4 buf[kPre];
  // launched overlapped with the projection GEMM (decode steps): everything above reads only the
  // layer's constants; the projection is read from here on
  grid_dep_wait();
#pragma unroll
  for (int p = 0; p < kPre; ++p) buf[p] = fetch(item(p));
  __syncthreads();  // trig table
  const int n_pass = (n_items + NW * RPW - 1) / (NW * RPW);
  for (int p0 = 0; p0 < n_pass; p0 += kPre) {
#pragma unroll
    for (int p = 0; p < kPre; ++p) {
      const uint4 u = buf[p];
      buf[p] = fetch(item(p0 + kPre + p));
      process(item(p0 + p), u);
    }
  }

  // gates: HKV beta logits and H eta logits per token
  const int n_gates = blockIdx.y == 0 ? (do_kv ? a.HKV : 0) + (do_q ? a.H : 0) : 0;  // the first row group's
  for (int i = threadIdx.x; i < ntb * n_gates; i += blockDim.x) {
    const int tl = i / n_gates, gi = i % n_gates;
    const int64_t tok = tok0 + tl;
    const int b = s_b[tl], t = s_t[tl];
    const bf16* row = reinterpret_cast<const bf16*>(a.proj) + tok * a.ld;
    if (do_kv && gi < a.HKV) {
      const float z = bf2f(row[a.beta_col + gi]);
      a.beta[((int64_t)b * a.HKV + gi) * a.beta_head_stride + beta_t_off + t] = rbf(1.0f / (1.0f + expf(-z)));
    } else {
      const int h = gi - (do_kv ? a.HKV : 0);
      const float z = bf2f(row[a.eta_col + h]);
      a.eta[((int64_t)b * a.H + h) * a.eta_head_stride + a.eta_t_off + t] = rbf(tanhf(z));
    }
  }
}

}  // namespace

extern "C" int bolt3_prep(const bolt3_prep_args* a, void* stream) {
  const b3::TraceRange trace_range("bolt3_prep");
  if (!a || !a->proj || !a->inv_freq) return BOLT3_ERR_ARG;
  if (a->parts < 1 || a->parts > 3) return BOLT3_ERR_ARG;
  if ((a->parts & 1) && (!a->q_raw || !a->q_rope || !a->eta)) return BOLT3_ERR_ARG;
  if ((a->parts & 2) && (!a->k_raw || !a->k_rope || !a->v || !a->beta)) return BOLT3_ERR_ARG;
  if (a->B <= 0 || a->T <= 0 || a->H <= 0 || a->HKV <= 0 || a->H % a->HKV) return BOLT3_ERR_SHAPE;
  if ((a->parts & 1) && (a->q_col < 0 || a->q_col + (int64_t)a->H * a->HD > a->ld || a->eta_col < 0 ||
                         a->eta_col + a->H > a->ld))
    return BOLT3_ERR_CAPACITY;
  if ((a->parts & 2) && (a->k_col < 0 || a->k_col + (int64_t)a->HKV * a->HD > a->ld || a->v_col < 0 ||
                         a->v_col + (int64_t)a->HKV * a->HD > a->ld || a->beta_col < 0 ||
                         a->beta_col + a->HKV > a->ld))
    return BOLT3_ERR_CAPACITY;
  if ((a->parts & 1) && (a->q_head_stride < a->q_t_off + a->T || a->eta_head_stride < a->eta_t_off + a->T))
    return BOLT3_ERR_CAPACITY;
  if (a->pos_dev != nullptr && a->pos_span < 1) return BOLT3_ERR_ARG;
  const int64_t dmax = a->pos_dev != nullptr ? a->pos_span - 1 : 0;  // largest device step shift
  if ((a->parts & 2) && (a->k_head_stride < a->k_t_off + dmax + a->T || a->beta_head_stride < a->beta_t_off + dmax + a->T))
    return BOLT3_ERR_CAPACITY;
  // 16-byte vector access: rows of proj, and every output row, start on 16-byte boundaries
  const uintptr_t al = (uintptr_t)a->proj |
                       ((a->parts & 1) ? ((uintptr_t)a->q_raw | (uintptr_t)a->q_rope) : 0) |
                       ((a->parts & 2) ? ((uintptr_t)a->k_raw | (uintptr_t)a->k_rope | (uintptr_t)a->v) : 0);
  const bool cols_ok = !((a->parts & 1) && a->q_col % 8) && !((a->parts & 2) && (a->k_col % 8 || a->v_col % 8));
  if ((al & 15) || (a->ld % 8) || !cols_ok) return BOLT3_ERR_ALIGN;
  const int64_t n_tok = (int64_t)a->B * a->T;
  if (n_tok > 0x7fffffff) return BOLT3_ERR_SHAPE;
  // 16 tokens per block when there are enough tokens to fill the GPU several times over (prefill);
  // one token per block otherwise (decode steps), so that every SM gets work
  // (token, row) pairs per block: the kernel's multiply-shift division by the row count is exact
  // while pairs x (row count - 1) < 2^20 (16-token blocks hold for up to ~250 rows)
  const int64_t rows = a->H + 2 * a->HKV;
  const auto fits = [&](int64_t tb) { return tb * rows * (rows - 1) < ((int64_t)1 << 20); };
  if (!fits(1)) return BOLT3_ERR_SHAPE;
  const bool big = n_tok >= 16 * 1024 && fits(16);
  const int tb = big ? 16 : 1;
  // one-token blocks: the rows in groups of a warp pass (16 rows at HD = 128, 32 at 64)
  const int row_group = 8 * (32 / (a->HD / 8));
  const dim3 grid((unsigned)((n_tok + tb - 1) / tb), big ? 1u : (unsigned)((rows + row_group - 1) / row_group));
  cudaStream_t s = (cudaStream_t)stream;
  // one-token blocks (decode steps, a few microseconds of work): launched overlapped with the
  // projection GEMM before them, so that their blocks are scheduled as the GEMM's leave
  cudaError_t e = cudaSuccess;
  if (a->HD == 128) {
    if (big) prep_kernel<128, 16><<<grid, 256, 0, s>>>(*a);
    else e = launch_overlapped(prep_kernel<128, 1>, grid, dim3(256), 0, s, *a);
  } else if (a->HD == 64) {
    if (big) prep_kernel<64, 16><<<grid, 256, 0, s>>>(*a);
    else e = launch_overlapped(prep_kernel<64, 1>, grid, dim3(256), 0, s, *a);
  } else {
    return BOLT3_ERR_SHAPE;
  }
  return e == cudaSuccess && cudaGetLastError() == cudaSuccess ? BOLT3_OK : BOLT3_ERR_CUDA;
}
