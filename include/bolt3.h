/* C-ABI of the B200-native Bolt-3 dual-field attention hot path.
 *
 * The reference implements this path in eager PyTorch (vsa_lm/config/bolt3.py); it has no FFI of
 * its own. These entry points are what a binding of that module's hot loops calls instead: plain
 * device pointers, int64 sizes/strides, a cudaStream_t passed as void*, an int status return.
 * No entry point allocates device memory, throws, or synchronises the stream; all work is
 * stream-ordered. bf16 arrays are passed as `void*` holding IEEE bfloat16 values.
 *
 * Array layouts (row-major, innermost last). A "chain" is one (sequence b, KV head h) pair,
 * chain = b * HKV + h; a query head index is chain * G + g (head h*G + g of sequence b).
 *   q_raw, q_rope : [B*H][Tq][HD] bf16         k_raw, k_rope, v : [B*HKV][Tk][HD] bf16
 *   beta          : [B*HKV][Tk] fp32           eta              : [B*H][Tq] fp32
 *   bank ak, av, ak_rope : [chains][S][HD] bf16; mass, util, pm : [chains][S] fp32;
 *   act : [chains][S] uint8; m_res : [chains][HD][HD] fp32 (= the reference's states[li]);
 *   n_filled : [chains] int32.
 * Supported shapes: HD in {64, 128}, S = C = 128, n_sinks = 4, G = H / HKV in [1, 16].
 */
#ifndef BOLT3_H_
#define BOLT3_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BOLT3_ABI_VERSION 10

enum bolt3_status {
  BOLT3_OK = 0,
  BOLT3_ERR_ARG = 1,       /* null pointer where one is required, or a negative size */
  BOLT3_ERR_SHAPE = 2,     /* unsupported HD / S / C / G / token count */
  BOLT3_ERR_ALIGN = 3,     /* a pointer or stride is not 16-byte aligned */
  BOLT3_ERR_CAPACITY = 4,  /* a buffer described by the arguments is too small */
  BOLT3_ERR_CUDA = 5       /* a kernel launch or CUDA runtime call failed */
};

/* ---- Phase A epilogue: per-head RMSNorm (optional), RoPE, beta = sigmoid, eta = tanh.
 * Replaces Bolt3Attn.head_qkv + rope + gates (vsa_lm/config/bolt3.py:59-66, 196-199;
 * vsa_lm/surgery.py:43-53, 80-93) and the same lines of Bolt3Decoder.step (bolt3.py:346-350).
 * Input `proj` is a token-major projection output [B*T][ld] (ld a multiple of 8, 16-byte aligned).
 * `parts` selects what it holds: bit 0 = q (H*HD columns at q_col) and eta logits (H at eta_col);
 * bit 1 = k and v (HKV*HD each at k_col, v_col) and beta logits (HKV at beta_col). The q and k/v
 * column blocks must start on multiples of 8.
 * Output element (b, head, t) of a head-major array lives at
 *   ((b * n_heads + head) * head_stride + t_off + t) * HD      (q_*: n_heads = H, k/v: HKV). */
/* Device step position. A one-token decode step replayed from a CUDA graph cannot take its
 * position as a launch argument; bolt3_prep and bolt3_attend (prefill = 0) then read it from the
 * device. With pos_dev non-NULL the kernel reads d = *pos_dev - pos_ref, which must lie in
 * [0, pos_span): bolt3_prep uses RoPE position pos0 + d and writes k / v / beta at k_t_off + d and
 * beta_t_off + d (q and eta offsets are unchanged); bolt3_attend uses seg1_len + d keys of segment 1
 * and len_before + d. The launch checks every size for the largest d, pos_span - 1; segment 1's
 * rows past seg1_len + d must hold finite values (they are read and masked). A d outside the range
 * makes both kernels skip the step, and bolt3_attend ORs 8 into its status word. */
typedef struct bolt3_prep_args {
  const void* proj; int64_t ld;       /* bf16 [B*T][ld] */
  int B, T, H, HKV, HD;
  const float* q_norm_w;              /* [HD] or NULL (no qk_norm) */
  const float* k_norm_w;              /* [HD] or NULL */
  float eps;
  const float* inv_freq;              /* [HD/2] */
  int64_t pos0;                       /* RoPE position of token t is pos0 + t */
  void* q_raw; void* q_rope; int64_t q_head_stride; int64_t q_t_off;
  float* eta; int64_t eta_head_stride; int64_t eta_t_off;
  void* k_raw; void* k_rope; void* v; int64_t k_head_stride; int64_t k_t_off;
  float* beta; int64_t beta_head_stride; int64_t beta_t_off;
  float* q_l2;                        /* optional: |q_raw| per (head, token), laid out like eta */
  int parts;                          /* 1 = q/eta, 2 = k/v/beta, 3 = both */
  int64_t q_col, k_col, v_col, beta_col, eta_col;
  /* optional step position on the device (see "Device step position" below); NULL otherwise */
  const int64_t* pos_dev; int64_t pos_ref; int64_t pos_span;
} bolt3_prep_args;
int bolt3_prep(const bolt3_prep_args* a, void* stream);

/* ---- Phase B: sequential consolidation scan, one CTA per chain.
 * Runs `n_steps` consecutive _consolidate_functional calls (vsa_lm/config/bolt3.py:68-192) on
 * every chain: fill path, or full path = attractor prediction, cosine match, merge, diversity
 * eviction (torch.topk tie order reproduced exactly) and the Gershgorin-normalised delta rule
 * into M_res. Step i consolidates the chunk of array tokens
 *   [token0 + i*step_tokens + (i == 0 ? skip0 : 0), token0 + i*step_tokens + chunk_len)
 * whose RoPE position is pos0 + token index. The bank is read from / written back to the state
 * arrays (init_blank = 1 starts from the empty bank of bolt3.py:83-92). After each step the
 * state the attention reads is optionally written to snapshot slot snap0 + i:
 *   snap_ak_rope, snap_av [chains][snap_cap] x S*HD*2 bytes; snap_mass [chains][snap_cap][S] fp32;
 *   snap_act [chains][snap_cap][S] uint8; snap_m [chains][snap_cap] x HD*HD*4 bytes.
 *   The bf16 snapshots are tensor-core operand images that bolt3_attend copies as is: a tile of
 *   R rows x HD columns is HD/64 blocks of [R rows][64 columns], each row 128 bytes whose 16-byte
 *   chunk c sits at chunk c ^ (row & 7). ak_rope and av: R = S rows of slots. snap_m: M_res split
 *   into bf16 hi then lo terms, each an image with R = HD rows d and columns e. The final bank
 *   (ak, av, ak_rope, m_res) is written in the plain row-major layouts listed at the top.
 * `ak_rope` (optional) receives RoPE(ak, pm) of the final bank. `status` (optional, device int)
 * is OR-ed with 1 when a kernel-side bounds check of the tie-order emulation fires, and with 4 when
 * a bounded wait for a tensor-core product expired.
 * `wait_probe` is a failure-path test hook and 0 in normal use. When nonzero, every CTA's first
 * thread polls a barrier that nothing arrives at `wait_probe` times; the wait runs out, status
 * bit 4 is set, and the kernel returns without touching the bank or starting any copy or MMA. */
typedef struct bolt3_consolidate_args {
  int n_chains, hkv, HD;
  void* ak; void* av; void* ak_rope;
  float* mass; float* util; float* pm; uint8_t* act; float* m_res; int32_t* n_filled;
  int init_blank;
  const void* kr; const void* kp; const void* v; const float* beta;
  int64_t chain_tokens;               /* tokens between chains in kr / kp / v / beta */
  int64_t token0; int64_t step_tokens; int skip0; int chunk_len; int64_t pos0; int n_steps;
  const float* kappa; const float* gamma; const float* inv_freq;   /* [hkv], [hkv], [HD/2] */
  void* snap_ak_rope; void* snap_av; float* snap_mass; uint8_t* snap_act; void* snap_m;
  int64_t snap_cap; int64_t snap0;
  int32_t* status;
  uint32_t wait_probe;                /* test hook, 0 in normal use (see above) */
} bolt3_consolidate_args;
int bolt3_consolidate(const bolt3_consolidate_args* a, void* stream);

/* ---- Phase C: three-field softmax attention + fused M_res read-out epilogue.
 * Replaces the chunk body of Bolt3Attn.forward (vsa_lm/config/bolt3.py:219-256) and the
 * attention of Bolt3Decoder.step (bolt3.py:365-402): softmax over
 * [n_sinks sinks | S attractors (RoPE at mean position, + kappa*log(mass), -inf if inactive) |
 * causal local window], then y = bf16(bf16(P@V) + bf16(eta * RMSNorm(normalize(q_raw) @ M_res *
 * (1 - gamma) / sqrt(HD)))). Query block r (blockIdx.x) holds query tokens [r*128, r*128+128) of
 * q arrays with Tq tokens per head. Window keys are two segments (previous chunk, current chunk)
 * of [chains][*][HD] arrays; a key at window position j is visible to query row i of the block
 * iff j <= n_before + i.
 *   prefill = 1: block r is chunk r of a sequence of Tq tokens held in k_rope / v (Tk = Tq);
 *     segment 0 = chunk r-1, segment 1 = chunk r, sinks = tokens 0..3, bank = snapshot r-2.
 *   prefill = 0: one query block (Tq <= 128 new tokens); segment pointers, lengths, sinks and the
 *     bank (slot 0 of [chains][bank_cap] arrays) are given explicitly.
 * bank_m: prefill = 1 reads the split bf16 image bolt3_consolidate writes to snap_m; prefill = 0
 * reads M_res itself, fp32 [chains][HD][HD]. q_l2 (optional, [B*H][Tq] fp32) holds |q_raw| per row
 * as bolt3_prep writes it; without it the kernel computes the norms.
 * `wait_probe` is a failure-path test hook and 0 in normal use. When nonzero, the kernels that
 * have bounded waits (the tensor-core prefill tile and the streaming one-token decode kernel) poll
 * a barrier that nothing arrives at `wait_probe` times, set status bit 2 and return without
 * writing y. The warp-per-chain decode kernel has no waits and ignores it. */
typedef struct bolt3_attend_args {
  int n_chains, hkv, G, HD;
  const void* q_rope; const void* q_raw; const float* eta; int64_t Tq;
  int prefill;
  /* window segments (prefill: seg0_k = seg1_k = k_rope, seg*_v = v, chain_tokens = Tk) */
  const void* seg0_k; const void* seg0_v; int64_t seg0_chain_tokens; int seg0_len;
  const void* seg1_k; const void* seg1_v; int64_t seg1_chain_tokens; int seg1_len;
  int len_before;                      /* keys of segment 1 that precede the first query */
  const void* sink_k; const void* sink_v; int64_t sink_chain_tokens; int has_sinks;
  /* attractor bank: [chains][snap_cap][S]... as written by bolt3_consolidate */
  const void* bank_ak_rope; const void* bank_av; const float* bank_mass; const uint8_t* bank_act;
  const void* bank_m; int64_t bank_cap; int has_bank;
  const float* kappa;                  /* [hkv] */
  const float* coef;                   /* [hkv]: (1 - gamma) / sqrt(HD), fp32 */
  const float* res_w; float eps;       /* res_norm weight [HD] (fp32), eps */
  void* y; int64_t y_tokens;           /* bf16 [B][y_tokens][H][HD]; row of query token t: t */
  int32_t* status;                     /* optional device int: OR-ed with 2 if a bounded wait expired,
                                          with 8 if a device step position was out of range */
  const float* q_l2;                   /* optional |q_raw| per row, [B*H][Tq] */
  int64_t blk_begin, blk_count;        /* prefill: query blocks [blk_begin, blk_begin + blk_count)
                                          (blk_count = 0: every block) */
  uint32_t wait_probe;                 /* test hook, 0 in normal use (see above) */
  /* optional step position on the device (prefill = 0 only; see "Device step position") */
  const int64_t* pos_dev; int64_t pos_ref; int64_t pos_span;
} bolt3_attend_args;
int bolt3_attend(const bolt3_attend_args* a, void* stream);

/* ---- Softmax anchor layers of the hybrid model: one-token decode step.
 * Replaces the anchor branch of Bolt3Decoder.step for one new token (vsa_lm/config/bolt3.py:426-445:
 * the cache append of vsa_lm/decode.py:88-106, then scaled_dot_product_attention with enable_gqa).
 * For every (sequence b, KV head): writes k_new / v_new at cache position n, then the exact softmax
 * attention of its G = H / HKV query heads over cache positions 0..n (scores q.k * scale in fp32),
 * y rounded to bf16 once. q: bf16 [B][H][HD]; k_new, v_new: bf16 [B][HKV][HD]; k_cache, v_cache:
 * bf16 [B][HKV][cap][HD]; y: bf16 [B][H][HD]. HD 64 or 128, G <= 8. inv_freq NULL: q and k_new
 * come with RoPE applied. inv_freq non-NULL (fp32 [HD/2]): the kernel applies rotate-half RoPE to q
 * and k_new at position pos0 as LlamaRoPE does in bf16 (vsa_lm/surgery.py:80-93: cos and sin rounded
 * to bf16, each product and the sum rounded to bf16). With pos_dev (the device step position of
 * bolt3_prep), d = *pos_dev - pos_ref shifts both the cache position (n + d) and pos0 (pos0 + d),
 * within [0, pos_span); outside it the step is skipped and status gets 8. */
typedef struct bolt3_anchor_args {
  int B, H, HKV, HD;
  const void* q; const void* k_new; const void* v_new;
  void* k_cache; void* v_cache; int64_t cap; int64_t n;
  void* y; float scale;
  int32_t* status;                     /* optional device int (bit 8: device position out of range) */
  const int64_t* pos_dev; int64_t pos_ref; int64_t pos_span;
  const float* inv_freq; int64_t pos0;  /* optional RoPE of q and k_new (see above) */
} bolt3_anchor_args;
int bolt3_anchor_decode(const bolt3_anchor_args* a, void* stream);

/* ---- RMSNorm of bf16 rows (the hybrid model's block, final and per-head q/k norms).
 * Replaces LlamaRMSNorm.forward (vsa_lm/surgery.py:43-53) for bf16 inputs: y[r] = bf16(x[r] *
 * rsqrt(mean(x[r]^2) + eps) * w), in fp32 inside; one kernel instead of torch's casts and norm.
 * x: bf16 rows of D values, row r at x + r * x_stride (elements); y: bf16 [rows][D]; w: [D], bf16
 * (w_fp32 = 0) or fp32 (w_fp32 = 1). D a multiple of 8 up to 4096; pointers 16-byte aligned.
 * With r (bf16 [rows][D]) the row normalised is the residual sum s = bf16(x + r), each element added
 * in fp32 and rounded once as torch's bf16 addition does, and s is written to sum (bf16 [rows][D]):
 * the hybrid model's `x = x + branch; h = norm(x)` in one kernel. */
typedef struct bolt3_rmsnorm_args {
  const void* x; const void* w; void* y;
  int64_t rows; int64_t x_stride;
  int D; int w_fp32; float eps;
  const void* r; void* sum;             /* optional residual input and sum output (see above) */
} bolt3_rmsnorm_args;
int bolt3_rmsnorm(const bolt3_rmsnorm_args* a, void* stream);

/* ---- SwiGLU's elementwise step (the hybrid model's MLP, vsa_lm/surgery.py:202-211).
 * gu: bf16 [rows][2I], the gate projection in columns [0, I) and the up projection in [I, 2I) (both
 * projections as one GEMM); y: bf16 [rows][I] = bf16(bf16(silu(g)) * u), silu in fp32 as torch
 * computes it. I a multiple of 8; pointers 16-byte aligned. */
typedef struct bolt3_silu_mul_args {
  const void* gu; void* y;
  int64_t rows; int64_t I;
} bolt3_silu_mul_args;
int bolt3_silu_mul(const bolt3_silu_mul_args* a, void* stream);

/* Bytes of snapshot workspace bolt3_prefill_fwd needs for n_chains chains of T tokens. */
size_t bolt3_prefill_workspace_size(int n_chains, int64_t T, int HD);

/* ---- Phases B + C of Bolt3Attn.forward (vsa_lm/config/bolt3.py:194-274) for sequences of T
 * tokens whose projections bolt3_prep has written (q_*: Tq = T, k_* / v / beta: Tk = T).
 * Runs the consolidation scan (chunk i consolidated after chunk i+1 when chunk i+1 is full and
 * not last, sinks = first 4 tokens) into caller-provided snapshot workspace, then the attention
 * over all chunks. The final bank is written to the state arrays (which may be scratch). */
typedef struct bolt3_prefill_args {
  int B, T, H, HKV, HD;
  const void* q_rope; const void* q_raw; const float* eta;
  const void* k_raw; const void* k_rope; const void* v; const float* beta;
  const float* kappa; const float* gamma; const float* coef; const float* inv_freq;
  const float* res_w; float eps;
  void* workspace; size_t workspace_bytes;
  /* final bank (chains = B*HKV) */
  void* ak; void* av; void* ak_rope; float* mass; float* util; float* pm; uint8_t* act;
  float* m_res; int32_t* n_filled;
  void* y;                            /* bf16 [B][T][H][HD] */
  int32_t* status;
  const float* q_l2;                  /* optional |q_raw| per row from bolt3_prep, [B*H][T] */
} bolt3_prefill_args;
int bolt3_prefill_fwd(const bolt3_prefill_args* a, void* stream);

/* ---- bolt3_prefill_fwd without a caller-provided workspace. No counterpart in the reference.
 * For hosts that cannot allocate device memory on their hot path (an engine that pools all of HBM
 * itself, a C-ABI host without a device allocator, a loop that cannot afford cudaMalloc's implicit
 * device synchronisation). The snapshot workspace is a fixed BOLT3_NOALLOC_SCRATCH_BYTES array
 * inside the library: CUDA reserves it in a context when the library's device code is first used
 * there (lazy module loading) and holds it until the process exits. `workspace` and
 * `workspace_bytes` of the arguments are ignored. Work needing more than that returns
 * BOLT3_ERR_CAPACITY (32 MiB covers 254 chain-consolidations at HD = 128: e.g. one Qwen3-4B-shape
 * sequence of up to 4224 tokens, or configs[0] whole). The first call in a context (each device's
 * primary context, or a context the host created) looks up the array's device address with that
 * context current and caches it under the context's unique id; make that first call before any
 * stream capture. Calls share the array: two calls that overlap on the GPU (different streams, or
 * different host threads) race and must be ordered by the caller. Allocates nothing (no
 * cudaMalloc / cudaFree). */
#define BOLT3_NOALLOC_SCRATCH_BYTES (32u << 20)
int bolt3_prefill_fwd_noalloc(const bolt3_prefill_args* a, void* stream);

/* ---- utilities */
int bolt3_abi_version(void);
const char* bolt3_status_string(int status);
/* sizeof of an argument struct (0 prep, 1 consolidate, 2 attend, 3 prefill, 4 anchor, 5 rmsnorm,
 * 6 silu_mul; 0 for others), so a
 * binding can check its own layout of the structs against the compiled one */
size_t bolt3_args_size(int which);
/* Host-only: reorder indices 0..n-1 of `vals` into the order CPU torch.topk(vals, k, largest)
 * returns (first k written to out_idx). Returns 0, or 1 if a bounds check fired. */
int bolt3_topk_order_host(const float* vals, int n, int k, int largest, int32_t* out_idx);

#ifdef __cplusplus
}
#endif
#endif /* BOLT3_H_ */
