// C-ABI utilities and the two-phase prefill driver (consolidation scan, then attention).
#include "../../include/bolt3.h"
#include "common.cuh"
#include "trace.h"
#include "stl_select.h"

namespace {

constexpr int S = 128, CC = 128, N_SINKS = 4;

int64_t n_consolidations(int64_t T) {  // bolt3.py:262: full, non-final chunks consolidate prev
  const int64_t full = T / CC;
  return T % CC == 0 ? (full > 2 ? full - 2 : 0) : (full > 1 ? full - 1 : 0);
}

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

struct SnapLayout {
  size_t ak_rope, av, mass, act, m, total;
};

SnapLayout snap_layout(int n_chains, int64_t T, int HD) {
  const size_t ns = (size_t)n_chains * (size_t)n_consolidations(T);
  SnapLayout L;
  size_t off = 0;
  L.ak_rope = off; off = align256(off + ns * S * HD * 2);
  L.av = off;      off = align256(off + ns * S * HD * 2);
  L.mass = off;    off = align256(off + ns * S * 4);
  L.act = off;     off = align256(off + ns * S);
  L.m = off;       off = align256(off + ns * (size_t)HD * HD * 4);
  L.total = off;
  return L;
}

}  // namespace

extern "C" int bolt3_abi_version(void) { return BOLT3_ABI_VERSION; }

extern "C" size_t bolt3_args_size(int which) {
  switch (which) {
    case 0: return sizeof(bolt3_prep_args);
    case 1: return sizeof(bolt3_consolidate_args);
    case 2: return sizeof(bolt3_attend_args);
    case 3: return sizeof(bolt3_prefill_args);
    case 4: return sizeof(bolt3_anchor_args);
    case 5: return sizeof(bolt3_rmsnorm_args);
    case 6: return sizeof(bolt3_silu_mul_args);
    default: return 0;
  }
}

extern "C" const char* bolt3_status_string(int st) {
  switch (st) {
    case BOLT3_OK: return "ok";
    case BOLT3_ERR_ARG: return "invalid argument (null pointer or negative size)";
    case BOLT3_ERR_SHAPE: return "unsupported shape (HD must be 64 or 128, S = C = 128, G <= 16)";
    case BOLT3_ERR_ALIGN: return "pointer not 16-byte aligned";
    case BOLT3_ERR_CAPACITY: return "buffer too small for the described work";
    case BOLT3_ERR_CUDA: return "CUDA launch or runtime error";
    default: return "unknown status";
  }
}

extern "C" int bolt3_topk_order_host(const float* vals, int n, int k, int largest, int32_t* out_idx) {
  if (!vals || !out_idx || n <= 0 || k <= 0 || k > n || n > 4096) return 1;
  b3sel::KV buf[4096];
  for (int i = 0; i < n; ++i) { buf[i].v = vals[i]; buf[i].i = i; }
  const int bad = b3sel::topk_order(buf, n, k, largest != 0);
  for (int i = 0; i < k; ++i) out_idx[i] = buf[i].i;
  return bad;
}

extern "C" size_t bolt3_prefill_workspace_size(int n_chains, int64_t T, int HD) {
  if (n_chains <= 0 || T <= 0 || (HD != 64 && HD != 128)) return 0;
  return snap_layout(n_chains, T, HD).total;
}

extern "C" int bolt3_prefill_fwd(const bolt3_prefill_args* a, void* stream) {
  const b3::TraceRange trace_range("bolt3_prefill_fwd");
  if (!a) return BOLT3_ERR_ARG;
  if (a->B <= 0 || a->T <= 0 || a->HKV <= 0 || a->H % a->HKV || (a->HD != 64 && a->HD != 128))
    return BOLT3_ERR_SHAPE;
  const int n_chains = a->B * a->HKV;
  const int64_t n_cons = n_consolidations(a->T);
  const SnapLayout L = snap_layout(n_chains, a->T, a->HD);
  if (n_cons > 0 && (!a->workspace || a->workspace_bytes < L.total)) return BOLT3_ERR_CAPACITY;
  unsigned char* ws = reinterpret_cast<unsigned char*>(a->workspace);

  if (n_cons > 0) {
    bolt3_consolidate_args c = {};
    c.n_chains = n_chains; c.hkv = a->HKV; c.HD = a->HD;
    c.ak = a->ak; c.av = a->av; c.ak_rope = a->ak_rope;
    c.mass = a->mass; c.util = a->util; c.pm = a->pm; c.act = a->act; c.m_res = a->m_res;
    c.n_filled = a->n_filled;
    c.init_blank = 1;
    c.kr = a->k_raw; c.kp = a->k_rope; c.v = a->v; c.beta = a->beta;
    c.chain_tokens = a->T;
    c.token0 = 0; c.step_tokens = CC; c.skip0 = N_SINKS; c.chunk_len = CC; c.pos0 = 0;
    c.n_steps = (int)n_cons;
    c.kappa = a->kappa; c.gamma = a->gamma; c.inv_freq = a->inv_freq;
    c.snap_ak_rope = ws + L.ak_rope; c.snap_av = ws + L.av;
    c.snap_mass = reinterpret_cast<float*>(ws + L.mass);
    c.snap_act = reinterpret_cast<uint8_t*>(ws + L.act);
    c.snap_m = ws + L.m;
    c.snap_cap = n_cons; c.snap0 = 0;
    c.status = a->status;
    const int rc = bolt3_consolidate(&c, stream);
    if (rc != BOLT3_OK) return rc;
  }
  bolt3_attend_args t = {};
  t.n_chains = n_chains; t.hkv = a->HKV; t.G = a->H / a->HKV; t.HD = a->HD;
  t.q_rope = a->q_rope; t.q_raw = a->q_raw; t.eta = a->eta; t.Tq = a->T;
  t.prefill = 1;
  t.seg0_k = a->k_rope; t.seg0_v = a->v; t.seg0_chain_tokens = a->T;
  t.seg1_k = a->k_rope; t.seg1_v = a->v; t.seg1_chain_tokens = a->T;
  if (n_cons > 0) {
    t.bank_ak_rope = ws + L.ak_rope; t.bank_av = ws + L.av;
    t.bank_mass = reinterpret_cast<const float*>(ws + L.mass);
    t.bank_act = reinterpret_cast<const uint8_t*>(ws + L.act);
    t.bank_m = ws + L.m;
    t.bank_cap = n_cons;
  }
  t.kappa = a->kappa; t.coef = a->coef; t.res_w = a->res_w; t.eps = a->eps;
  t.y = a->y; t.y_tokens = a->T;
  t.status = a->status;
  t.q_l2 = a->q_l2;
  return bolt3_attend(&t, stream);
}
