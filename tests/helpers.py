"""Shared helpers for the parity tests: seeded modules on the GPU and their CPU-oracle twins."""
from __future__ import annotations

import torch

from oracle import Store, oracle_cfg
from vsa_lm_b200 import Bolt3Attn
from vsa_lm_b200.workloads import layer_cfg, make_input, make_params

# Output tolerance of the north star: rtol 2e-2 in bf16. Elements near zero are held to an absolute
# bound of 2e-2 times the output's RMS instead.
RTOL = 2e-2
ATOL_RMS = 2e-2
# fp32 state tolerance (M_res, mass, pm, util)
STATE_RTOL = 1e-4
NEAR = 1e-3   # merge decisions within this distance of 0.88 / 0.80 may flip


def bf16_module(cfg: dict, seed: int, device="cuda") -> Bolt3Attn:
    m = Bolt3Attn(cfg)
    m.load_state_dict(make_params(cfg, seed), strict=True)
    return m.to(device=device, dtype=torch.bfloat16).eval()


def oracle_params(m: Bolt3Attn) -> dict:
    """The module's own (bf16) parameters on the CPU, for the oracle."""
    return {k: v.detach().cpu() for k, v in m.state_dict().items()}


def oracle_cfg_of(m: Bolt3Attn, cfg: dict) -> dict:
    oc = oracle_cfg(cfg)
    oc["inv_freq"] = m.rope.inv_freq.detach().float().cpu()
    return oc


def output_close(got: torch.Tensor, ref: torch.Tensor, what: str = "output") -> dict:
    got, ref = got.float().cpu(), ref.float().cpu()
    rms = ref.pow(2).mean().sqrt().item()
    err = (got - ref).abs()
    bound = RTOL * ref.abs() + ATOL_RMS * rms
    bad = err > bound
    info = dict(max_abs=err.max().item(), rms=rms, frac_bad=bad.float().mean().item(),
                max_rel_rms=(err.max().item() / max(rms, 1e-30)))
    assert not bad.any(), f"{what}: {int(bad.sum())} elements outside rtol {RTOL} / atol {ATOL_RMS}*rms: {info}"
    return info


def near_threshold(rec: dict) -> torch.Tensor:
    """Chains whose merge decision has a cosine within NEAR of a threshold (flip allowed)."""
    if rec.get("kind") != "full":
        return torch.zeros(rec["score"].shape[0], dtype=torch.bool)
    nk = (rec["best_sim_k"] - 0.88).abs() < NEAR
    nv = (rec["sim_v"] - 0.80).abs() < NEAR
    return (nk | nv).any(dim=-1)


def near_tie_chains(rec: dict, rel: float = 1e-6) -> torch.Tensor:
    """Chains whose ranking keys (eviction candidates, slot keep values, fill scores) contain
    distinct values closer than `rel` (relative): their order is decided by rounding noise and the
    CPU reference's own result depends on its reduction order."""
    def close_pairs(v):  # v: [chains, k] sorted
        a, b = v[:, :-1], v[:, 1:]
        d = (a - b).abs()
        return ((d > 0) & (d <= rel * torch.maximum(a.abs(), b.abs()))).any(dim=-1)

    if rec.get("kind") == "full":
        top, bot = rec["top_vals"], rec["bot_vals"]
        real = top > -1e8
        flag = close_pairs(torch.where(real, top, torch.full_like(top, -1e30)))
        flag |= close_pairs(bot)
        d = (top - bot).abs()
        flag |= (real & (d > 0) & (d <= rel * bot.abs())).any(dim=-1)
        return flag
    sc = torch.sort(rec["score"], dim=-1, descending=True).values
    return close_pairs(sc)


def ambiguous(rec: dict) -> bool:
    """A consolidation whose decisions depend on rounding noise: a cosine within NEAR of a merge
    threshold, or ranking keys within 1e-6 relative of each other (first-fill variance scores of
    near-zero-mean values tie at the fp32 ulp level; their order then follows the CPU's reduction
    order, and any later exact-tie break between those slots follows that order)."""
    return bool(near_threshold(rec).any() or near_tie_chains(rec).any())


def bank_multiset(mass: torch.Tensor, pm: torch.Tensor, act: torch.Tensor):
    """Slot-order-free view of a bank: per chain, the sorted (pm, mass) of the active slots."""
    out = []
    for c in range(mass.shape[0]):
        a = act[c].bool()
        key = torch.stack([pm[c][a].double(), mass[c][a].double()], dim=-1)
        out.append(key[torch.argsort(key[:, 0] * 1e6 + key[:, 1])])
    return out


def inputs(shape: str, B: int, T: int, dup, seed: int = 1, device="cuda"):
    cfg = layer_cfg(shape)
    x = make_input(B, T, cfg["dim"], dup=dup, seed=seed)
    return cfg, x.to(torch.bfloat16).float(), x.to(device=device, dtype=torch.bfloat16)


BF16 = Store("bf16")
