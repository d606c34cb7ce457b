"""Shared helpers for the parity tests: seeded modules on the GPU and their CPU-oracle twins, the
rule for which consolidation decisions rounding may change, and the bank comparison and re-sync
used by the free-running tests."""
from __future__ import annotations

import torch

from oracle import Store, oracle_cfg
from oracle.parity import NEAR, TIE_REL, decision_ties, near_threshold  # noqa: F401
from vsa_lm_b200 import Bolt3Attn
from vsa_lm_b200.workloads import layer_cfg, make_input, make_params

# Output tolerance of the north star: rtol 2e-2 in bf16. Elements near zero are held to an absolute
# bound of 2e-2 times the RMS of their output row (see output_close).
RTOL = 2e-2
ATOL_RMS = 2e-2
# fp32 state tolerance (M_res, mass, pm, util)
STATE_RTOL = 1e-4
# A slot's utility is the token's prediction error rel_err = |v - P.av| / |v| at insertion, with the
# softmax probabilities P rounded to bf16 before the product (the reference's CUDA arithmetic). Both
# sides round the same fp32 probabilities, but a value within one fp32 ulp of a bf16 rounding
# boundary may round either way; for a token whose duplicate already sits in the bank P is
# concentrated (p ~ 1), and one such rounding moves rel_err by up to p * 2^-9 ~ 2e-3.
UTIL_ATOL = 2e-3


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
    """Elementwise rtol 2e-2, with an absolute floor of 2e-2 x the RMS of the element's own output
    row (one token's vector, the last dimension) or of the whole output, whichever is larger."""
    got, ref = got.float().cpu(), ref.float().cpu()
    rms = ref.pow(2).mean().sqrt().item()
    row_rms = ref.pow(2).mean(dim=-1, keepdim=True).sqrt()
    err = (got - ref).abs()
    bound = RTOL * ref.abs() + ATOL_RMS * row_rms.clamp_min(rms)
    bad = err > bound
    info = dict(max_abs=err.max().item(), rms=rms, frac_bad=bad.float().mean().item(),
                max_rel_rms=(err.max().item() / max(rms, 1e-30)))
    assert not bad.any(), f"{what}: {int(bad.sum())} elements outside rtol {RTOL} / atol {ATOL_RMS}*rms: {info}"
    return info


BANK_KEYS = ("ak", "av", "mass", "util", "pm", "act")


def chain_of(bank: dict, c: int) -> dict:
    """One chain's slot arrays of a bank (native or oracle layout), on the CPU in fp32."""
    out = {}
    for k in BANK_KEYS:
        t = bank[k]
        t = t.reshape(-1, *t.shape[-2:]) if k in ("ak", "av") else t.reshape(-1, t.shape[-1])
        out[k] = t[c].detach().cpu().float() if k != "act" else t[c].detach().cpu().bool()
    return out


def match_slots(nat: dict, ref: dict):
    """Match the slots of one chain's native bank to the oracle's: (perm, why). perm[j] is the
    native slot holding the oracle's slot j (None if the banks differ as sets, `why` says how).
    Matched pairs must agree within the state tolerances: act and mass exactly (mass counts merged
    tokens), pm to 1e-4 relative, util to 1e-4 relative plus UTIL_ATOL, ak / av to a bf16 rounding
    step."""
    from scipy.optimize import linear_sum_assignment

    S = ref["mass"].numel()
    an, ar = nat["act"], ref["act"]
    if int(an.sum()) != int(ar.sum()):
        return None, f"{int(an.sum())} active slots vs {int(ar.sum())}"
    idx_n, idx_r = an.nonzero().flatten(), ar.nonzero().flatten()
    perm = torch.full((S,), -1, dtype=torch.long)
    if idx_r.numel():
        pn, pr = nat["pm"][idx_n].double(), ref["pm"][idx_r].double()
        cost = (pn[:, None] - pr[None, :]).abs() / (1.0 + pr.abs()[None, :])
        cost = cost + 10.0 * (nat["mass"][idx_n][:, None] != ref["mass"][idx_r][None, :]).double()
        akn, akr = nat["ak"][idx_n].double(), ref["ak"][idx_r].double()
        cost = cost + torch.cdist(akn, akr, p=1) / (akr.abs().sum(-1)[None, :] + 1e-6)
        rows, cols = linear_sum_assignment(cost.numpy())
        perm[idx_r[torch.as_tensor(cols)]] = idx_n[torch.as_tensor(rows)]
    # inactive slots pair up in order (all hold the blank values)
    perm[(~ar).nonzero().flatten()] = (~an).nonzero().flatten()
    g = {k: nat[k][perm] for k in BANK_KEYS}
    a = ar
    if not torch.equal(g["act"], ar):
        return None, "active slots differ"
    if not torch.equal(g["mass"][a], ref["mass"][a]):
        j = int(((g["mass"] != ref["mass"]) & a).nonzero()[0])
        return None, f"mass of slot {j}: {g['mass'][j].item()} vs {ref['mass'][j].item()}"
    checks = (("pm", 1e-4, 1e-3), ("util", 1e-4, UTIL_ATOL), ("ak", 8e-3, 1e-6), ("av", 8e-3, 1e-6))
    for k, rt, at in checks:
        d = (g[k][a] - ref[k][a]).abs()
        bad = d > rt * ref[k][a].abs() + at
        if bad.any():
            return None, f"{k} differs by up to {d.max().item():.3e}"
    return perm, ""


def m_res_error(nat: torch.Tensor, ref: torch.Tensor) -> float:
    """Largest |M_nat - M_ref| of one chain relative to the chain's largest |M_ref|."""
    nat, ref = nat.detach().cpu().float(), ref.float()
    return ((nat - ref).abs().max() / ref.abs().max().clamp_min(1e-30)).item()


class FlipLedger:
    """The consolidations whose native outcome differed from the oracle's. Each must be one that
    `decision_ties` flags (a near-tie or near-threshold decision); the fraction of such chain-steps
    is bounded and every one is printed with its reason."""

    def __init__(self, name: str, bound: float = 0.02):
        self.name, self.bound = name, bound
        self.total, self.flagged, self.flips = 0, 0, []

    def step(self, rec: dict, n_chains: int) -> torch.Tensor:
        flags = decision_ties(rec)
        self.total += n_chains
        self.flagged += int(flags.sum())
        return flags

    def flip(self, step: int, chain: int, why: str, flagged: bool) -> None:
        assert flagged, (f"{self.name}: consolidation {step}, chain {chain} differs from the oracle with no "
                         f"near-tie or near-threshold decision: {why}")
        self.flips.append((step, chain, why))

    def report(self) -> None:
        frac = len(self.flips) / max(self.total, 1)
        print(f"{self.name}: {len(self.flips)} of {self.total} chain-steps differ ({frac:.2%}); "
              f"{self.flagged} flagged near-tie/near-threshold")
        for st, c, why in self.flips:
            print(f"  consolidation {st}, chain {c}: {why}")
        assert frac <= self.bound, f"{self.name}: {frac:.2%} of chain-steps differ (bound {self.bound:.0%})"


def load_chain(bank: dict, c: int, ref: dict, m_res_ref: torch.Tensor, n_filled: int, rope=None) -> None:
    """Overwrite chain c of a native bank with the oracle's state."""
    dev = bank["mass"].device
    for k in ("ak", "av"):
        bank[k][c] = ref[k].to(device=dev, dtype=torch.bfloat16)
    for k in ("mass", "util", "pm"):
        bank[k][c] = ref[k].to(dev)
    bank["act"][c] = ref["act"].to(device=dev, dtype=torch.uint8)
    bank["m_res"][c] = m_res_ref.to(dev)
    bank["n_filled"][c] = n_filled
    if rope is not None and bank.get("ak_rope") is not None:
        bank["ak_rope"][c] = rope.to(device=dev, dtype=torch.bfloat16)


def sync_bank(ledger: FlipLedger, step: int, rec: dict, bank: dict, ref_bank: dict, n_filled: int,
              m_res_tol: float, rope_fn=None) -> set:
    """Compare every chain of a native bank (and its M_res) with the oracle's after one
    consolidation, then load the oracle's state into every chain (teacher forcing: the next
    consolidation starts from exactly the oracle's pre-state, so rounding differences do not
    accumulate across steps). A chain that differs beyond the state tolerances must be flagged by
    `decision_ties`; it is counted as a flip. Returns the chains that flipped."""
    flags = ledger.step(rec, bank["mass"].shape[0])
    flipped = set()
    torch.cuda.synchronize()
    for c in range(bank["mass"].shape[0]):
        ref = chain_of(ref_bank, c)
        perm, why = match_slots(chain_of(bank, c), ref)
        m_ref = ref_bank["m_res"].reshape(-1, *ref_bank["m_res"].shape[-2:])[c]
        if perm is not None:
            err = m_res_error(bank["m_res"][c], m_ref)
            if err >= m_res_tol:
                perm, why = None, f"M_res differs by {err:.2e} of its max"
        if perm is None:
            ledger.flip(step, c, why, bool(flags[c]))
            flipped.add(c)
        load_chain(bank, c, ref, m_ref, n_filled, rope_fn(c) if rope_fn else None)
    return flipped


def inputs(shape: str, B: int, T: int, dup, seed: int = 1, device="cuda"):
    cfg = layer_cfg(shape)
    x = make_input(B, T, cfg["dim"], dup=dup, seed=seed)
    return cfg, x.to(torch.bfloat16).float(), x.to(device=device, dtype=torch.bfloat16)


def decoder_projections(m, h, pos):
    """The projections Bolt3Decoder.layer_step computes for h [b, t, D], in the oracle's layouts
    (fp32 on the CPU)."""
    return tuple(t.float().cpu() for t in m.step_projections(h, pos))


class LockstepTap:
    """Runs the Bolt-3 layers of a ModelDecoderOracle in lockstep with the native decoder.

    While active, every Bolt3Decoder.layer_step call also steps the oracle's matching layer on the
    projections the GPU computed for that call (decoder_projections), checks the layer's output
    against the oracle's, and after each consolidation checks the native bank and M_res and then
    loads the oracle's state into them (sync_bank; flips must be flagged and are counted in
    `ledger`). The oracle layer outputs are kept by (layer index, position) and serve as the model
    oracle's `attn_source`, so the oracle's own forward through the model (embedding, anchors, MLP,
    norms) uses exactly the Bolt-3 outputs checked here."""

    def __init__(self, model, oracle, ledger: FlipLedger):
        from vsa_lm_b200 import Bolt3Decoder

        self.cls, self.oracle, self.ledger = Bolt3Decoder, oracle, ledger
        self.index = {id(blk.vsa): i for i, blk in enumerate(model.blocks) if hasattr(blk, "vsa")}
        self.outs = {}
        oracle.attn_source = self

    def __enter__(self):
        orig = self.orig = self.cls.layer_step
        tap = self

        def layer_step(ly, st, h, pos_start, m_res, partial_fp32=False):
            from oracle import rope_at

            li = tap.index[id(ly)]
            proj = decoder_projections(ly, h, pos_start)
            L = tap.oracle.layers[li]
            n_rec = len(L.record)
            out = orig(ly, st, h, pos_start, m_res, partial_fp32)
            ref = L.step(h.float().cpu(), pos_start, proj=proj)
            output_close(out.float().cpu(), ref, f"layer {li} attention at position {pos_start}")
            tap.outs[(li, pos_start)] = ref
            if len(L.record) > n_rec:
                HD = ly.HD
                bank = dict(st.bank)
                bank["m_res"] = m_res.view(-1, HD, HD)
                ref_bank = dict(L.sc, m_res=L.m_res.view(-1, HD, HD))
                rope = lambda c: rope_at(L.sc["ak"][c], L.sc["pm"][c], L.cfg["inv_freq"], BF16)
                sync_bank(tap.ledger, len(L.record) - 1, L.record[-1], bank, ref_bank, L.n_filled, STATE_RTOL, rope)
            return out

        self.cls.layer_step = staticmethod(layer_step)
        return self

    def __exit__(self, *exc):
        self.cls.layer_step = staticmethod(self.orig)

    def __call__(self, layer: int, pos: int):
        return self.outs[(layer, pos)]


BF16 = Store("bf16")
