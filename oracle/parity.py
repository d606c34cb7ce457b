"""Which consolidation decisions rounding may change (test infrastructure only).

A CUDA implementation and this CPU oracle compute the attractor-bank decisions of
`_consolidate_functional` (vsa_lm/config/bolt3.py:96-192) from the same inputs with different
accumulation orders. Decisions whose keys are within rounding distance of each other, or cosines
within 1e-3 of the merge thresholds (the north star's rule), may come out either way; every other
decision must be identical. `decision_ties` flags, per chain, the consolidations where such a
decision changes the outcome. The parity tests and the parity check of bench.py's CPU baseline leg
use it to tell a permitted flip from an error.
"""
from __future__ import annotations

import torch

NEAR = 1e-3      # merge decisions within this distance of 0.88 / 0.80 may flip
# Two distinct ranking keys closer than this (relative) are ordered by rounding noise: the CUDA path
# and the fp32 CPU oracle accumulate in different orders, so either may rank them either way.
TIE_REL = 1e-5


def near_threshold(rec: dict) -> torch.Tensor:
    """Chains whose merge decision has a cosine within NEAR of a threshold (flip allowed)."""
    if rec.get("kind") != "full":
        return torch.zeros(rec["score"].shape[0], dtype=torch.bool)
    nk = (rec["best_sim_k"] - 0.88).abs() < NEAR
    nv = (rec["sim_v"] - 0.80).abs() < NEAR
    return (nk | nv).any(dim=-1)


def near(a: torch.Tensor, b: torch.Tensor, rel: float) -> torch.Tensor:
    d = (a - b).abs()
    return (d > 0) & (d <= rel * torch.maximum(a.abs(), b.abs()))


def decision_ties(rec: dict, rel: float = TIE_REL) -> torch.Tensor:
    """Chains of one consolidation whose OUTCOME (the bank as a set of slots, M_res) a near-tie or a
    near-threshold cosine can change. Near-ties that only reorder slots are not flagged: the tests
    compare banks up to a permutation of slots.

    fill (bolt3.py:165-192): the m selected tokens are a set; only the pair of sorted scores straddling
    position m-1 / m decides which tokens are kept, and only when m < l_tok.
    full (bolt3.py:96-152):
      - a cosine within NEAR of 0.88 / 0.80 (the merge decision itself, north-star rule);
      - for a token that may merge (best cosine >= 0.88 - NEAR), its two best slot cosines nearly
        tied: the merge target is ambiguous;
      - eviction: win = top > bot is a prefix of length w of the sorted pairs. Swaps among winners
        only move inserted tokens between evicted slots (a permutation); the outcome changes only
        through a near-tie at the boundary: top[i] ~ bot[i] for i in {w-1, w}, or top[w-1] ~ top[w]
        (which token is inserted), or bot[w-1] ~ bot[w] (which slot is evicted), or the k_cand
        boundary of the slot ranking when k_cand < S.
    Exact ties (equal keys) are not flagged: the kernels reproduce CPU torch.topk's order of equal
    keys."""
    if rec.get("kind") != "full":
        m, l_tok = rec["m"], rec["l_tok"]
        n = rec["score"].shape[0]
        if m >= l_tok or m <= 0:
            return torch.zeros(n, dtype=torch.bool)
        sc = torch.sort(rec["score"], dim=-1, descending=True).values
        return near(sc[:, m - 1], sc[:, m], rel)
    flag = near_threshold(rec)
    s1, s2 = rec["best_sim_k"], rec["second_sim_k"]
    flag |= ((s1 >= 0.88 - NEAR) & near(s1, s2, rel)).any(dim=-1)
    top, bot, win = rec["top_vals"], rec["bot_vals"], rec["win"]
    k = top.shape[1]
    w = win.long().sum(dim=-1)
    rows = torch.arange(top.shape[0])
    for off in (-1, 0):
        i = (w + off).clamp(0, k - 1)
        ok = (w + off >= 0) & (w + off < k)
        flag |= ok & near(top[rows, i], bot[rows, i], rel)
    j0, j1 = (w - 1).clamp(0, k - 1), w.clamp(0, k - 1)
    inside = (w >= 1) & (w < k)
    flag |= inside & (near(top[rows, j0], top[rows, j1], rel) | near(bot[rows, j0], bot[rows, j1], rel))
    keep = rec["keep"]
    if k < keep.shape[1]:
        ks = torch.sort(keep, dim=-1).values
        flag |= near(ks[:, k - 1], ks[:, k], rel)
    return flag
