"""Algorithmic work of the Bolt-3 hot path: FLOPs of a prefill, bytes of a decode step.

Counts only useful work: masked causal halves and the extra score pass of the exact softmax are not
counted, and the bf16 hi/lo splits of fp32 operands count once. These are the numerators of the
roofline fractions bench.py reports.
"""
from __future__ import annotations

S, C, N_SINKS = 128, 128, 4


def n_consolidations(T: int) -> int:
    full = T // C
    return max(0, full - 2) if T % C == 0 else max(0, full - 1)


def proj_in_flops(D: int, H: int, HKV: int, HD: int) -> int:
    """Fused q/k/v/beta/eta projection, per token."""
    return 2 * D * (H * HD + 2 * HKV * HD + HKV + H)


def proj_out_flops(D: int, H: int, HD: int) -> int:
    """o_proj, per token."""
    return 2 * H * HD * D


def attend_flops(T: int, H: int, HD: int) -> int:
    """QK^T + PV over the visible keys + the M_res read-out, per sequence of T tokens."""
    total = 0
    for i in range(0, (T + C - 1) // C):
        tc = min(C, T - i * C)
        fixed = (N_SINKS + S) if i >= 2 else 0
        prev = C if i >= 1 else 0
        keys = tc * (fixed + prev) + tc * (tc + 1) // 2      # causal: token j sees j+1 keys
        total += 4 * HD * H * keys
        if i >= 2:
            total += 2 * HD * HD * H * tc
    return total


def consolidation_flops(HD: int) -> int:
    """One full-bank consolidation of one chain: sc, v^, cos_k, pair_cos, gram, k^M, k^T err."""
    return 7 * 2 * C * S * HD


def prefill_flops(B: int, T: int, D: int, H: int, HKV: int, HD: int) -> dict:
    tok = B * T
    parts = {
        "proj_in": tok * proj_in_flops(D, H, HKV, HD),
        "attend": B * attend_flops(T, H, HD),
        "consolidate": B * HKV * n_consolidations(T) * consolidation_flops(HD),
        "proj_out": tok * proj_out_flops(D, H, HD),
    }
    parts["total"] = sum(parts.values())
    return parts


def decode_step_bytes(n_seq: int, D: int, H: int, HKV: int, HD: int, window: float = C + (C + 1) / 2,
                      with_weights: bool = True) -> dict:
    """HBM bytes one decode step must move for n_seq sequences (one token each).

    State per sequence: attractor keys (RoPE'd) and values, their bias inputs, M_res, sinks and the
    average local window (prev chunk + half of the current one); plus the new token's k/v writes
    and consolidation amortised over C steps. Weights are read once per step for the whole batch.
    """
    per_seq = (2 * HKV * S * HD * 2            # ak_rope + av
               + HKV * S * (4 + 1)             # mass + act
               + HKV * HD * HD * 4             # M_res
               + 2 * HKV * N_SINKS * HD * 2    # sinks
               + 2 * HKV * window * HD * 2     # window keys + values
               + 3 * HKV * HD * 2 + HKV * 4    # new kr, kp, v, beta
               + (2 * HKV * C * HD * 2 * 3 + 2 * HKV * S * HD * 2 * 3 + 2 * HKV * HD * HD * 4) / C)  # consolidation
    weights = 2 * (D * (H * HD + 2 * HKV * HD + HKV + H) + H * HD * D) if with_weights else 0
    return {"state": int(n_seq * per_seq), "weights": int(weights), "total": int(n_seq * per_seq + weights)}
