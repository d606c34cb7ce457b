// Phase A epilogue: from the fused projection output to head-major q/k/v with RoPE and gates.
//
// Mirrors Bolt3Attn.head_qkv (vsa_lm/config/bolt3.py:59-66: per-head LlamaRMSNorm when qk_norm,
// surgery.py:43-53), LlamaRoPE (surgery.py:80-93) in the storage dtype (cos/sin cast to bf16, every
// product and the sum rounded to bf16), beta = sigmoid(beta_proj x) and eta = tanh(eta_proj x)
// (bolt3.py:198-199) computed from the bf16 logits and rounded to bf16.
//
// HBM-bound elementwise work with 16-byte loads and stores: a head row of HD values is handled by
// HD/8 lanes, each owning 8 consecutive elements; the lane holding elements i and the lane holding
// i + HD/2 (the pair rotate-half RoPE couples) swap values with one shuffle.
#include "../../include/bolt3.h"
#include "common.cuh"

namespace {

using namespace b3;

template <int HD>
__global__ void __launch_bounds__(256) prep_kernel(const bolt3_prep_args a) {
  constexpr int LPR = HD / 8;          // lanes per head row
  constexpr int RPW = 32 / LPR;        // rows per warp pass
  constexpr int HALF = LPR / 2;        // lane offset between the RoPE partners
  const int tok = blockIdx.x;          // b * T + t
  const int b = tok / a.T, t = tok % a.T;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane / LPR, l = lane % LPR;   // row slot within the warp, lane within the row
  const bf16* row = reinterpret_cast<const bf16*>(a.proj) + (int64_t)tok * a.ld;
  const float pos = (float)(a.pos0 + t);
  const bool first = l < HALF;         // holds elements of the first half

  // cos/sin of the HD/2 frequencies, once per token, shared by every head through shared memory
  __shared__ float s_cos[HD / 2], s_sin[HD / 2];
  for (int i = threadIdx.x; i < HD / 2; i += blockDim.x) {
    float sv, cv;
    sincosf(__fmul_rn(pos, a.inv_freq[i]), &sv, &cv);
    s_cos[i] = rbf(cv);
    s_sin[i] = rbf(sv);
  }
  __syncthreads();
  float cs[8], sn[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int fi = (l % HALF) * 8 + e;  // frequency index: element index mod HD/2
    cs[e] = s_cos[fi];
    sn[e] = s_sin[fi];
  }

  // head rows this call handles: [0, H) q when parts & 1, then HKV k and HKV v rows when parts & 2
  const bool do_q = a.parts & 1, do_kv = (a.parts & 2) != 0;
  const int n_rows = (do_q ? a.H : 0) + (do_kv ? 2 * a.HKV : 0);
  auto row_col = [&](int r, int& kind, int& head) -> int64_t {
    if (do_q && r < a.H) { kind = 0; head = r; return a.q_col + (int64_t)head * HD; }
    const int rk = r - (do_q ? a.H : 0);
    if (rk < a.HKV) { kind = 1; head = rk; return a.k_col + (int64_t)head * HD; }
    kind = 2; head = rk - a.HKV;
    return a.v_col + (int64_t)head * HD;
  };
  // issue the loads of up to kPre passes before any use, so each lane keeps several 16-byte loads
  // in flight (this kernel is bound by HBM latency x bytes in flight)
  constexpr int kPre = 4;
  uint4 pre[kPre];
#pragma unroll
  for (int p = 0; p < kPre; ++p) {
    const int r = warp * RPW + p * 8 * RPW + sub;
    pre[p] = make_uint4(0, 0, 0, 0);
    int kd, hd_;
    if (r < n_rows) pre[p] = *reinterpret_cast<const uint4*>(row + row_col(r, kd, hd_) + l * 8);
  }
  int pass = 0;
  for (int r0 = warp * RPW; r0 < n_rows; r0 += 8 * RPW, ++pass) {
    const int r = r0 + sub;
    const bool live = r < n_rows;
    int kind = 2, head = 0;  // 0 = q, 1 = k, 2 = v
    int64_t col = 0;
    if (live) col = row_col(r, kind, head);
    float x[8];
    {
      uint4 u = make_uint4(0, 0, 0, 0);
      if (pass < kPre) {
#pragma unroll
        for (int p = 0; p < kPre; ++p)
          if (p == pass) u = pre[p];
      } else if (live) {
        u = *reinterpret_cast<const uint4*>(row + col + l * 8);
      }
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
    const int64_t to = kind == 0 ? a.q_t_off : a.k_t_off;
    const int64_t off = (((int64_t)b * nh + head) * hs + to + t) * HD + l * 8;
    // per-row reductions stay inside the LPR lanes of the row
    auto row_sum = [&](float v) {
#pragma unroll
      for (int o = LPR / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      return v;
    };
    const float* nw = kind == 0 ? a.q_norm_w : a.k_norm_w;
    // all lanes take part in the shuffles below, whatever their row's kind
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) ss = fmaf(x[e], x[e], ss);
    ss = row_sum(ss);
    if (kind != 2 && nw != nullptr) {
      const float rr = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, (float)HD), a.eps));
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = rbf(__fmul_rn(__fmul_rn(x[e], rr), nw[l * 8 + e]));
    }
    float l2 = 0.f;  // |q_raw| of the stored (bf16) row, for the M_res read-out
#pragma unroll
    for (int e = 0; e < 8; ++e) l2 = fmaf(x[e], x[e], l2);
    l2 = row_sum(l2);
    // RoPE partner values (element i <-> i + HD/2)
    float y[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) y[e] = __shfl_xor_sync(0xffffffffu, x[e], HALF);
    if (!live) continue;
    uint32_t raw[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) raw[q] = pack_bf16(x[2 * q], x[2 * q + 1]);
    if (kind == 2) {
      *reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(a.v) + off) = make_uint4(raw[0], raw[1], raw[2], raw[3]);
      continue;
    }
    if (kind == 0 && a.q_l2 != nullptr && l == 0)
      a.q_l2[((int64_t)b * a.H + head) * a.eta_head_stride + a.eta_t_off + t] = sqrtf(l2);
    uint32_t rot[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float o2[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int e = 2 * q + u;
        // rotate_half: the first half pairs with -x[i + HD/2], the second half with x[i - HD/2]
        const float partner = first ? -y[e] : y[e];
        o2[u] = rbf(__fadd_rn(rbf(__fmul_rn(x[e], cs[e])), rbf(__fmul_rn(partner, sn[e]))));
      }
      rot[q] = pack_bf16(o2[0], o2[1]);
    }
    *reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(kind == 0 ? a.q_raw : a.k_raw) + off) =
        make_uint4(raw[0], raw[1], raw[2], raw[3]);
    *reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(kind == 0 ? a.q_rope : a.k_rope) + off) =
        make_uint4(rot[0], rot[1], rot[2], rot[3]);
  }

  // gates: HKV beta logits and H eta logits
  const int n_gates = (do_kv ? a.HKV : 0) + (do_q ? a.H : 0);
  for (int i = threadIdx.x; i < n_gates; i += blockDim.x) {
    if (do_kv && i < a.HKV) {
      const float z = bf2f(row[a.beta_col + i]);
      a.beta[((int64_t)b * a.HKV + i) * a.beta_head_stride + a.beta_t_off + t] = rbf(1.0f / (1.0f + expf(-z)));
    } else {
      const int h = i - (do_kv ? a.HKV : 0);
      const float z = bf2f(row[a.eta_col + h]);
      a.eta[((int64_t)b * a.H + h) * a.eta_head_stride + a.eta_t_off + t] = rbf(tanhf(z));
    }
  }
}

}  // namespace

extern "C" int bolt3_prep(const bolt3_prep_args* a, void* stream) {
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
  if ((a->parts & 2) && (a->k_head_stride < a->k_t_off + a->T || a->beta_head_stride < a->beta_t_off + a->T))
    return BOLT3_ERR_CAPACITY;
  // 16-byte vector access: rows of proj, and every output row, start on 16-byte boundaries
  const uintptr_t al = (uintptr_t)a->proj |
                       ((a->parts & 1) ? ((uintptr_t)a->q_raw | (uintptr_t)a->q_rope) : 0) |
                       ((a->parts & 2) ? ((uintptr_t)a->k_raw | (uintptr_t)a->k_rope | (uintptr_t)a->v) : 0);
  const bool cols_ok = !((a->parts & 1) && a->q_col % 8) && !((a->parts & 2) && (a->k_col % 8 || a->v_col % 8));
  if ((al & 15) || (a->ld % 8) || !cols_ok) return BOLT3_ERR_ALIGN;
  const int64_t n_tok = (int64_t)a->B * a->T;
  if (n_tok > 0x7fffffff) return BOLT3_ERR_SHAPE;
  cudaStream_t s = (cudaStream_t)stream;
  if (a->HD == 128) prep_kernel<128><<<(unsigned)n_tok, 256, 0, s>>>(*a);
  else if (a->HD == 64) prep_kernel<64><<<(unsigned)n_tok, 256, 0, s>>>(*a);
  else return BOLT3_ERR_SHAPE;
  return cudaGetLastError() == cudaSuccess ? BOLT3_OK : BOLT3_ERR_CUDA;
}
