"""Bolt-3 dual-field attention, restated on the CPU as a parity oracle (test infrastructure only).

Every function cites the lines of the reference `vsa_lm/config/bolt3.py` (and `vsa_lm/surgery.py`)
whose arithmetic it restates. The oracle computes in fp32 throughout. A `Store` object decides the
precision of *stored* activations: `Store("fp32")` reproduces the reference run in fp32 on the CPU
(the configs[0] case, pinned bit-for-bit-ish against the reference's own outputs), `Store("bf16")`
rounds exactly the tensors that the reference keeps in the model dtype `dt` when the model is bf16
(projections, RoPE'd keys, attractor keys/values, softmax probabilities before P@V, the attention
output) while every product and sum stays fp32. The CUDA kernels follow the same convention
(bf16 operands, exact bf16 products, fp32 accumulation), so `Store("bf16")` is the oracle they are
compared with.

Tie order of `torch.topk` on the CPU is implementation defined; the oracle calls `torch.topk` exactly
where the reference does (bolt3.py:133-134, 183), so it reproduces the reference's order.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

__all__ = [
    "N_SINKS", "SIM_K", "SIM_V", "GAMMA_U", "Store", "llama_inv_freq", "rms_norm", "rope_at",
    "gamma_delta", "project", "blank_bank", "consolidate", "attend", "forward", "LayerDecoderOracle",
    "n_consolidations", "oracle_cfg",
]

N_SINKS = 4                                   # bolt3.py:30
SIM_K, SIM_V, GAMMA_U = 0.88, 0.80, 0.995     # bolt3.py:31


class Store:
    """Precision of stored activations: identity for fp32, round-to-nearest-even bf16 otherwise."""

    def __init__(self, mode: str = "fp32"):
        if mode not in ("fp32", "bf16"):
            raise ValueError(mode)
        self.mode = mode
        self.bf16 = mode == "bf16"

    def __call__(self, t: torch.Tensor) -> torch.Tensor:
        return t.to(torch.bfloat16).float() if self.bf16 else t.float()


def llama_inv_freq(head_dim: int, theta: float, rope_scaling: dict | None = None) -> torch.Tensor:
    """RoPE inverse frequencies incl. llama3 scaling (surgery.py:56-72)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    if rope_scaling and rope_scaling.get("rope_type") == "llama3":
        old_ctx = float(rope_scaling["original_max_position_embeddings"])
        factor = float(rope_scaling["factor"])
        low, high = float(rope_scaling["low_freq_factor"]), float(rope_scaling["high_freq_factor"])
        wavelen = 2.0 * math.pi / inv
        scaled = torch.where(wavelen > old_ctx / low, inv / factor, inv)
        smooth = (old_ctx / wavelen - low) / (high - low)
        blended = (1.0 - smooth) * scaled / factor + smooth * scaled
        medium = ~(wavelen < old_ctx / high) & ~(wavelen > old_ctx / low)
        inv = torch.where(medium, blended, scaled)
    return inv


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float, store: Store) -> torch.Tensor:
    """LlamaRMSNorm (surgery.py:43-53): fp32 inside, cast back to the stored dtype."""
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return store(y * weight.float())


def rope_at(x: torch.Tensor, pos: torch.Tensor, inv_freq: torch.Tensor, store: Store) -> torch.Tensor:
    """Rotate-half RoPE of stored values `x[..., n, HD]` at fp32 positions `pos[..., n]`.

    Integer positions: LlamaRoPE.forward (surgery.py:86-93). Fractional attractor positions:
    _apply_rope_pos (bolt3.py:17-20). cos/sin are cast to the stored dtype and, for bf16, each
    product and the sum round to bf16 as the reference's bf16 tensor arithmetic does.
    """
    freqs = pos.float().unsqueeze(-1) * inv_freq.float()
    emb = torch.cat((freqs, freqs), dim=-1)
    c, s = store(emb.cos()), store(emb.sin())
    h = x.shape[-1] // 2
    rot = torch.cat((-x[..., h:], x[..., :h]), dim=-1)
    return store(store(x * c) + store(rot * s))


def gamma_delta(log_gamma: torch.Tensor) -> torch.Tensor:
    """Per-KV-head M_res decay (bolt3.py:56-57); follows the parameter's dtype like the reference."""
    return (0.999 * torch.sigmoid(log_gamma)).clamp(1e-3, 0.999).float()


def _lin(xf: torch.Tensor, params: dict, name: str, store: Store) -> torch.Tensor:
    y = xf @ params[name + ".weight"].float().t()
    bias = params.get(name + ".bias")
    if bias is not None:
        y = y + bias.float()
    return store(y)


def project(params: dict, cfg: dict, x: torch.Tensor, store: Store):
    """q/k/v projections + optional per-head RMSNorm (head_qkv, bolt3.py:59-66) and the beta/eta
    gates (bolt3.py:198-199). Returns q_raw [b,H,T,HD], k_raw/v [b,HKV,T,HD], beta [b,HKV,T],
    eta [b,H,T], all as stored values in fp32 tensors."""
    b, T, _ = x.shape
    H, HKV, HD = cfg["H"], cfg["HKV"], cfg["HD"]
    xf = store(x.float())
    q = _lin(xf, params, "q_proj", store).view(b, T, H, HD)
    k = _lin(xf, params, "k_proj", store).view(b, T, HKV, HD)
    v = _lin(xf, params, "v_proj", store).view(b, T, HKV, HD)
    if cfg.get("qk_norm"):
        q = rms_norm(q, params["q_norm.weight"], cfg["eps"], store)
        k = rms_norm(k, params["k_norm.weight"], cfg["eps"], store)
    beta = store(torch.sigmoid(_lin(xf, params, "beta_proj", store)))
    eta = store(torch.tanh(_lin(xf, params, "eta_proj", store)))
    return (q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
            beta.transpose(1, 2), eta.transpose(1, 2))


def blank_bank(bh: int, S: int, HD: int) -> dict:
    """Initial attractor bank and M_res (bolt3.py:83-92)."""
    return dict(
        ak=torch.zeros(bh, S, HD), av=torch.zeros(bh, S, HD),
        mass=torch.ones(bh, S), util=torch.zeros(bh, S), pm=torch.zeros(bh, S),
        act=torch.zeros(bh, S, dtype=torch.bool), m_res=torch.zeros(bh, HD, HD), n_filled=0,
    )


def consolidate(bank: dict | None, kr: torch.Tensor, kp: torch.Tensor, v: torch.Tensor,
                pos: torch.Tensor, beta: torch.Tensor, *, kappa: torch.Tensor, gam: torch.Tensor,
                inv_freq: torch.Tensor, b: int, hkv: int, S: int, store: Store,
                record: list | None = None) -> dict:
    """One `_consolidate_functional` call (bolt3.py:68-192) on all b*hkv chains at once.

    kr/kp/v: [bh, l, HD] stored values; pos: [l] fp32 token positions; beta: [bh, l].
    kappa, gam: [hkv] fp32. Returns the new bank (a fresh dict). If `record` is a list, the
    per-chain decisions of this call are appended to it (for flip accounting).
    """
    bh, l_tok, hd = kr.shape
    scale = hd ** -0.5
    if bank is None:
        bank = blank_bank(bh, S, hd)
    ak, av, mass, pm, act, m_res = bank["ak"], bank["av"], bank["mass"], bank["pm"], bank["act"], bank["m_res"]
    n_filled = bank["n_filled"]
    p_f = pos.float().view(1, l_tok).expand(bh, l_tok)
    util = bank["util"] * GAMMA_U                                           # :94
    v32 = v.float()
    kr_n = F.normalize(kr.float(), dim=-1)
    rec = {"n_filled": n_filled, "l_tok": l_tok}

    def predict(mass_bias, masked):
        # attractor read-out prediction of each token's value (:97-103 / :169-174)
        k_read = rope_at(ak.view(b, hkv, S, hd), pm.view(b, hkv, S), inv_freq, store).view(bh, S, hd)
        sc = torch.bmm(kp.float(), k_read.transpose(-1, -2)) * scale + mass_bias
        if masked:
            sc = sc.masked_fill(~act.unsqueeze(1), -1e9)
        v_hat = torch.bmm(store(F.softmax(sc, dim=-1)), av)
        return (v32 - v_hat).norm(dim=-1) / (v32.norm(dim=-1) + 1e-6)

    if n_filled >= S:
        # ---- full bank: predict, match, merge (:96-123)
        kap = kappa.float().repeat(b).view(bh, 1, 1)
        rel_err = predict(kap * torch.log(mass.clamp_min(1.0)).unsqueeze(1), masked=False)
        cos_k = torch.bmm(kr_n, F.normalize(ak.float(), dim=-1).transpose(-1, -2))
        best_sim_k, best_slot = cos_k.max(dim=-1)
        matched_av = torch.gather(av, 1, best_slot.unsqueeze(-1).expand(-1, -1, hd))
        sim_v = F.cosine_similarity(v32, matched_av, dim=-1)
        score_j = rel_err * (1.0 - best_sim_k.clamp(0.0, 1.0))
        merge = (best_sim_k >= SIM_K) & (sim_v >= SIM_V)

        onehot = F.one_hot(best_slot, num_classes=S).float() * merge.float().unsqueeze(-1)
        cnt = onehot.sum(dim=1)
        k_sum = torch.bmm(onehot.transpose(1, 2), kr.float())
        v_sum = torch.bmm(onehot.transpose(1, 2), v32)
        p_sum = torch.bmm(onehot.transpose(1, 2), p_f.unsqueeze(-1)).squeeze(-1)
        hit = cnt > 0
        new_m = mass + cnt
        ak = torch.where(hit.unsqueeze(-1), store((mass.unsqueeze(-1) * ak + k_sum) / new_m.unsqueeze(-1)), ak)
        av = torch.where(hit.unsqueeze(-1), store((mass.unsqueeze(-1) * av + v_sum) / new_m.unsqueeze(-1)), av)
        pm = torch.where(hit, (mass * pm + p_sum) / new_m, pm)
        mass = torch.where(hit, new_m, mass)

        # ---- diversity eviction: sorted greedy match of novel tokens against weak slots (:125-152)
        ak_n = F.normalize(ak.float(), dim=-1)
        eye = torch.eye(S, dtype=torch.bool).unsqueeze(0)
        pair_cos = torch.bmm(ak_n, ak_n.transpose(-1, -2)).masked_fill(eye, -1.0)
        keep = util * (1.0 - pair_cos.max(dim=-1).values.clamp(0.0, 0.98))
        cand = torch.where(~merge, score_j, torch.full_like(score_j, -1e9))
        k_cand = min(l_tok, S)
        top_vals, top_toks = torch.topk(cand, k=k_cand, dim=-1, largest=True)
        bot_vals, bot_slots = torch.topk(keep, k=k_cand, dim=-1, largest=False)
        win = (top_vals > bot_vals) & (top_vals > -1e8)
        ins = torch.zeros_like(merge).scatter(1, top_toks, win)
        w3 = win.unsqueeze(-1)
        gidx = top_toks.unsqueeze(-1).expand(-1, -1, hd)
        sidx = bot_slots.unsqueeze(-1).expand(-1, -1, hd)
        ak = ak.scatter(1, sidx, torch.where(w3, torch.gather(kr.float(), 1, gidx), torch.gather(ak, 1, sidx)))
        av = av.scatter(1, sidx, torch.where(w3, torch.gather(v32, 1, gidx), torch.gather(av, 1, sidx)))
        pm = pm.scatter(1, bot_slots, torch.where(win, torch.gather(p_f, 1, top_toks), torch.gather(pm, 1, bot_slots)))
        mass = mass.scatter(1, bot_slots, torch.where(win, torch.ones_like(bot_vals), torch.gather(mass, 1, bot_slots)))
        util = util.scatter(1, bot_slots, torch.where(win, torch.gather(rel_err, 1, top_toks), torch.gather(util, 1, bot_slots)))

        # ---- Gershgorin-normalised one-shot delta rule into M_res (:154-162)
        w_ev = beta.float() * (~merge & ~ins).float()
        gram = torch.bmm(kr_n, kr_n.transpose(-1, -2)).abs()
        gersh = torch.bmm(gram, w_ev.unsqueeze(-1)).squeeze(-1).clamp_min(1.0)
        err = (v32 - torch.bmm(kr_n, m_res)) * (w_ev / gersh).unsqueeze(-1)
        m_res = gam.float().repeat(b).view(bh, 1, 1) * m_res + torch.bmm(kr_n.transpose(1, 2), err)
        # runner-up cosine of each token: a near-tie with best_sim_k makes the merge target ambiguous
        second_sim_k = cos_k.topk(2, dim=-1).values[..., 1] if S > 1 else best_sim_k
        rec.update(kind="full", rel_err=rel_err, best_sim_k=best_sim_k, second_sim_k=second_sim_k,
                   best_slot=best_slot, sim_v=sim_v, merge=merge, score=score_j, keep=keep,
                   top_vals=top_vals, top_toks=top_toks, bot_vals=bot_vals, bot_slots=bot_slots, win=win,
                   ins=ins)
        if record is not None:
            record.append(rec)
        return dict(ak=ak, av=av, mass=mass, util=util, pm=pm, act=act, m_res=m_res, n_filled=n_filled)

    # ---- fill path: the best m tokens take the next empty slots, the rest are dropped (:165-192)
    m = min(S - n_filled, l_tok)
    if n_filled > 0:
        rel_err = predict(torch.log(mass.clamp_min(1.0)).unsqueeze(1), masked=True)
        cos_k = torch.bmm(kr_n, F.normalize(ak.float(), dim=-1).transpose(-1, -2))
        cos_k = cos_k.masked_fill(~act.unsqueeze(1), 0.0)
        score_j = rel_err * (1.0 - cos_k.max(dim=-1).values.clamp(0.0, 1.0))
        init_u = rel_err
    else:
        score_j = F.normalize(v32, dim=-1).var(dim=-1)
        init_u = torch.full((bh, l_tok), 0.15)
    top_toks = torch.topk(score_j, k=m, dim=-1, largest=True).indices
    slots = torch.arange(n_filled, n_filled + m).unsqueeze(0).expand(bh, -1)
    gidx = top_toks.unsqueeze(-1).expand(-1, -1, hd)
    ak = ak.scatter(1, slots.unsqueeze(-1).expand(-1, -1, hd), torch.gather(kr.float(), 1, gidx))
    av = av.scatter(1, slots.unsqueeze(-1).expand(-1, -1, hd), torch.gather(v32, 1, gidx))
    pm = pm.scatter(1, slots, torch.gather(p_f, 1, top_toks))
    mass = mass.scatter(1, slots, torch.ones(bh, m))
    util = util.scatter(1, slots, torch.gather(init_u, 1, top_toks))
    act = act.scatter(1, slots, torch.ones(bh, m, dtype=torch.bool))
    rec.update(kind="fill", score=score_j, top_toks=top_toks, m=m)
    if record is not None:
        record.append(rec)
    return dict(ak=ak, av=av, mass=mass, util=util, pm=pm, act=act, m_res=m_res, n_filled=n_filled + m)


def attend(q_p, q_r, eta, loc_k, loc_v, n_before, sinks, bank, *, kappa, gam, inv_freq, res_w, eps,
           G: int, store: Store, causal: bool = True):
    """Three-field softmax attention of one query block plus the M_res read-out epilogue.

    Forward chunk body (bolt3.py:219-256) and the decoder step (bolt3.py:365-402) share this.
    q_p/q_r: [b,H,t,HD]; eta: [b,H,t]; loc_k/loc_v: [b,HKV,L,HD] RoPE'd window keys / values, of
    which the first `n_before` precede the query block (query i sees keys j <= n_before + i);
    sinks: (sink_k, sink_v) or None; bank: attractor bank dict or None. Returns y [b,H,t,HD]
    as stored values.
    """
    b, H, t, hd = q_p.shape
    hkv = H // G
    scale = hd ** -0.5
    rep = lambda z: z.repeat_interleave(G, dim=1)                       # repeat_kv (surgery.py:96-100)
    s_loc = torch.matmul(q_p, rep(loc_k).transpose(-1, -2)) * scale
    if causal:
        qi = torch.arange(t)[:, None]
        kj = torch.arange(loc_k.shape[2])[None, :]
        s_loc = s_loc.masked_fill(~(kj <= n_before + qi).view(1, 1, t, -1), float("-inf"))
    sp, vp = [], []
    if sinks is not None:
        sp.append(torch.matmul(q_p, rep(sinks[0]).transpose(-1, -2)) * scale)
        vp.append(rep(sinks[1]))
    if bank is not None:
        S = bank["ak"].shape[1]
        ak_eff = rope_at(bank["ak"].view(b, hkv, S, hd), bank["pm"].view(b, hkv, S), inv_freq, store)
        s_att = torch.matmul(q_p, rep(ak_eff).transpose(-1, -2)) * scale
        bias = kappa.float().view(1, hkv, 1, 1) * torch.log(bank["mass"].view(b, hkv, 1, S).clamp_min(1.0))
        s_att = (s_att + rep(bias)).masked_fill(~rep(bank["act"].view(b, hkv, 1, S)), float("-inf"))
        sp.append(s_att)
        vp.append(rep(bank["av"].view(b, hkv, S, hd)))
    sp.append(s_loc)
    vp.append(rep(loc_v))
    p = store(F.softmax(torch.cat(sp, dim=-1), dim=-1))
    y = store(torch.matmul(p, torch.cat(vp, dim=2)))
    if bank is not None:
        q_n = F.normalize(q_r.view(b, hkv, G, t, hd), dim=-1)
        ym = torch.einsum("bhgtc,bhcd->bhgtd", q_n, bank["m_res"].view(b, hkv, hd, hd))
        ym = ym * ((1.0 - gam).view(1, hkv, 1, 1, 1) / (hd ** 0.5))
        ym_n = rms_norm(ym.reshape(b, H, t, hd), res_w, eps, Store("fp32"))
        y = store(y + store(eta.unsqueeze(-1) * ym_n))
    return y


def n_consolidations(T: int, C: int) -> int:
    """Number of consolidations Bolt3Attn.forward performs (bolt3.py:262: full and not last chunk)."""
    full = T // C
    return max(0, full - 2) if T % C == 0 else max(0, full - 1)


def forward(params: dict, cfg: dict, x: torch.Tensor, store: Store, *, S: int = 128, C: int = 128,
            record: list | None = None, snapshots: list | None = None, return_y_heads: bool = False,
            proj: tuple | None = None):
    """Bolt3Attn.forward (bolt3.py:194-276): chunked three-field attention + o_proj.

    x: [b, T, D]. Returns [b, T, D] (stored values). `record` collects the per-consolidation
    decisions; `snapshots` collects the bank after each consolidation. `proj` (optional) replaces
    the projections with given stored values (q_raw, k_raw, v, beta, eta) in project()'s layouts,
    so that the rest of the algorithm can be checked on exactly the inputs another implementation
    computed.
    """
    b, T, _ = x.shape
    H, HKV, HD = cfg["H"], cfg["HKV"], cfg["HD"]
    G = H // HKV
    inv_freq = cfg["inv_freq"]
    q_r, k_r, v, beta, eta = project(params, cfg, x, store) if proj is None else [t.float() for t in proj]
    pos = torch.arange(T, dtype=torch.float32)
    q_p = rope_at(q_r, pos, inv_freq, store)
    k_p = rope_at(k_r, pos, inv_freq, store)
    gam = gamma_delta(params["log_gamma"])
    kappa = params["kappa"].float()
    common = dict(kappa=kappa, gam=gam, inv_freq=inv_freq, res_w=params["res_norm.weight"],
                  eps=cfg["eps"], G=G, store=store)
    sinks = bank = prev = None
    ys = []
    for s in range(0, T, C):
        e = min(T, s + C)
        if prev is not None:
            loc_k = torch.cat([prev[1], k_p[:, :, s:e]], dim=2)
            loc_v = torch.cat([prev[2], v[:, :, s:e]], dim=2)
            n_before = prev[1].shape[2]
        else:
            loc_k, loc_v, n_before = k_p[:, :, s:e], v[:, :, s:e], 0
        ys.append(attend(q_p[:, :, s:e], q_r[:, :, s:e], eta[:, :, s:e], loc_k, loc_v, n_before,
                         sinks, bank, **common))
        if e - s == C and e < T:                                         # :262
            if prev is not None:
                p_kr, p_kp, p_v, p_pos, p_b = prev
                if sinks is None:                                        # :265-268
                    ns = min(N_SINKS, p_kp.shape[2])
                    sinks = (p_kp[:, :, :ns], p_v[:, :, :ns])
                    p_kr, p_kp, p_v, p_pos, p_b = p_kr[:, :, ns:], p_kp[:, :, ns:], p_v[:, :, ns:], p_pos[ns:], p_b[:, :, ns:]
                l = p_kr.shape[2]
                bank = consolidate(bank, p_kr.reshape(b * HKV, l, HD), p_kp.reshape(b * HKV, l, HD),
                                   p_v.reshape(b * HKV, l, HD), p_pos, p_b.reshape(b * HKV, l),
                                   kappa=kappa, gam=gam, inv_freq=inv_freq, b=b, hkv=HKV, S=S,
                                   store=store, record=record)
                if snapshots is not None:
                    snapshots.append({k: (t.clone() if torch.is_tensor(t) else t) for k, t in bank.items()})
            prev = (k_r[:, :, s:e], k_p[:, :, s:e], v[:, :, s:e], pos[s:e], beta[:, :, s:e])
    y = torch.cat(ys, dim=2)                                               # [b,H,T,HD]
    out = store(y.transpose(1, 2).reshape(b, T, H * HD) @ params["o_proj.weight"].float().t())
    return (out, y) if return_y_heads else out


class LayerDecoderOracle:
    """Bolt3Decoder.step for one Bolt-3 layer (bolt3.py:343-425), state in the reference's format.

    `step(h, pos_start)` takes the normed hidden states h [b, t, D] of the new tokens and returns the
    attention branch output o_proj(y) [b, t, D]; consolidation runs whenever the current chunk
    reaches C tokens (bolt3.py:406-425, the last chunk included).
    """

    def __init__(self, params: dict, cfg: dict, b: int, store: Store, *, S: int = 128, C: int = 128):
        self.p, self.cfg, self.b, self.store, self.S, self.C = params, cfg, b, store, S, C
        HD, HKV = cfg["HD"], cfg["HKV"]
        self.m_res = torch.zeros(b, HKV, HD, HD)                           # states[li] (bolt3.py:309)
        self.sc = {k: None for k in ("ak", "av", "mass", "util", "pm", "act", "sink_k", "sink_v",
                                     "prev_kr", "prev_kp", "prev_v", "prev_pos", "prev_b",
                                     "cur_kr", "cur_kp", "cur_v", "cur_pos", "cur_b")}
        self.n_filled = 0
        self.record: list = []

    def bank(self):
        if self.sc["ak"] is None:
            return None
        return dict(ak=self.sc["ak"], av=self.sc["av"], mass=self.sc["mass"], util=self.sc["util"],
                    pm=self.sc["pm"], act=self.sc["act"],
                    m_res=self.m_res.view(-1, self.cfg["HD"], self.cfg["HD"]), n_filled=self.n_filled)

    def step(self, h: torch.Tensor, pos_start: int, proj: tuple | None = None) -> torch.Tensor:
        """`proj` (optional): the step's projections as stored values, as in forward()."""
        p, cfg, st, sc = self.p, self.cfg, self.store, self.sc
        b, t, _ = h.shape
        H, HKV, HD = cfg["H"], cfg["HKV"], cfg["HD"]
        G = H // HKV
        inv_freq = cfg["inv_freq"]
        q_r, k_r, v, beta, eta = project(p, cfg, h, st) if proj is None else [t_.float() for t_ in proj]
        pos = torch.arange(pos_start, pos_start + t, dtype=torch.float32)
        q_p, k_p = rope_at(q_r, pos, inv_freq, st), rope_at(k_r, pos, inv_freq, st)
        gam = gamma_delta(p["log_gamma"])
        kappa = p["kappa"].float()
        len_before = 0 if sc["cur_kp"] is None else sc["cur_kp"].shape[2]
        new = dict(cur_kr=k_r, cur_kp=k_p, cur_v=v, cur_pos=pos, cur_b=beta)
        for k, val in new.items():                                          # :356-363
            sc[k] = val if sc[k] is None else torch.cat([sc[k], val], dim=-1 if k == "cur_pos" else 2)
        if sc["prev_kp"] is not None:
            loc_k = torch.cat([sc["prev_kp"], sc["cur_kp"]], dim=2)
            loc_v = torch.cat([sc["prev_v"], sc["cur_v"]], dim=2)
            n_before = sc["prev_kp"].shape[2] + len_before
        else:
            loc_k, loc_v, n_before = sc["cur_kp"], sc["cur_v"], len_before
        sinks = None if sc["sink_k"] is None else (sc["sink_k"], sc["sink_v"])
        bank = self.bank()
        y = attend(q_p, q_r, eta, loc_k, loc_v, n_before, sinks, bank, kappa=kappa, gam=gam,
                   inv_freq=inv_freq, res_w=p["res_norm.weight"], eps=cfg["eps"], G=G, store=st,
                   causal=t > 1)
        out = st(y.transpose(1, 2).reshape(b, t, H * HD) @ p["o_proj.weight"].float().t())
        if sc["cur_kp"].shape[2] >= self.C:                                  # :406-425
            if sc["prev_kp"] is not None:
                p_kr, p_kp, p_v, p_pos, p_b = sc["prev_kr"], sc["prev_kp"], sc["prev_v"], sc["prev_pos"], sc["prev_b"]
                if sc["sink_k"] is None:
                    ns = min(N_SINKS, p_kp.shape[2])
                    sc["sink_k"], sc["sink_v"] = p_kp[:, :, :ns].clone(), p_v[:, :, :ns].clone()
                    p_kr, p_kp, p_v, p_pos, p_b = p_kr[:, :, ns:], p_kp[:, :, ns:], p_v[:, :, ns:], p_pos[ns:], p_b[:, :, ns:]
                l = p_kr.shape[2]
                nb = consolidate(bank, p_kr.reshape(b * HKV, l, HD), p_kp.reshape(b * HKV, l, HD),
                                 p_v.reshape(b * HKV, l, HD), p_pos, p_b.reshape(b * HKV, l),
                                 kappa=kappa, gam=gam, inv_freq=inv_freq, b=b, hkv=HKV, S=self.S,
                                 store=st, record=self.record)
                for k in ("ak", "av", "mass", "util", "pm", "act"):
                    sc[k] = nb[k]
                self.m_res = nb["m_res"].view(b, HKV, HD, HD)
                self.n_filled = nb["n_filled"]
            for k in ("kr", "kp", "v", "pos", "b"):
                sc["prev_" + k], sc["cur_" + k] = sc["cur_" + k], None
        return out


def oracle_cfg(cfg: dict) -> dict:
    """Dimensions and constants the oracle reads, from a reference-style cfg dict (bolt3.py:26-42)."""
    D, H, HKV = int(cfg["dim"]), int(cfg["num_heads"]), int(cfg["num_kv_heads"])
    HD = int(cfg.get("head_dim") or D // H)
    return dict(D=D, H=H, HKV=HKV, HD=HD, eps=float(cfg["eps"]), qk_norm=bool(cfg.get("qk_norm", False)),
                inv_freq=llama_inv_freq(HD, float(cfg["rope_theta"]), cfg.get("rope_scaling")))
