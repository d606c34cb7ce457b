"""Decoder steps that push the pending chunk past C tokens (vsa_lm/config/bolt3.py:355-363, 406-425).

The reference lets the current chunk grow by a whole step: a step of t tokens on top of a pending
chunk of c tokens leaves a chunk of c + t > C tokens, which becomes the previous chunk at once (it
has reached C) and is consolidated whole, as one `_consolidate_functional` call of c + t tokens, at
the next chunk boundary. This happens when a prompt is fed in C-token slices from a position that is
not a multiple of C: continue_generate or memorize after an unaligned prompt or answer.

The native kernels hold windows of two chunks of at most C tokens each and consolidate chunks of C,
so such an oversize chunk takes this path for as long as it is part of the window: the step that
creates it and every step until it is consolidated. The projections and prep (RMSNorm, RoPE, gates)
stay native; the window attention and the consolidation of the oversize chunk restate the
reference's algorithm in fp32 torch arithmetic on the GPU, with the storage roundings of the native
path (bf16 keys, values and probabilities; fp32 scores, bank statistics and M_res). Chunks of exactly
C tokens are consolidated by the native kernel as usual, and the state returns to the native window
ring at the first boundary after the oversize chunk is consolidated.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import kernels as K

SIM_K, SIM_V, GAMMA_U = 0.88, 0.80, 0.995      # merge thresholds and utility decay (bolt3.py:31)
N_SINKS = 4


def _bf(t: torch.Tensor) -> torch.Tensor:
    """Round to bf16 and back (the storage precision of keys, values and probabilities)."""
    return t.to(torch.bfloat16).float()


def rope_slots(ak: torch.Tensor, pm: torch.Tensor, inv_freq: torch.Tensor) -> torch.Tensor:
    """RoPE of bf16 attractor keys ak [..., S, HD] at fractional positions pm [..., S] (bolt3.py:12-20):
    cos and sin rounded to bf16, each product and the sum rounded to bf16. Returns bf16."""
    ang = pm.float().unsqueeze(-1) * inv_freq.float()
    ang = torch.cat((ang, ang), dim=-1)
    h = ak.shape[-1] // 2
    akb = ak.to(torch.bfloat16)
    rot = torch.cat((-akb[..., h:], akb[..., :h]), dim=-1)
    return akb * ang.cos().to(torch.bfloat16) + rot * ang.sin().to(torch.bfloat16)


@torch.no_grad()
def attend(ly, st, consts: dict, q_rope: torch.Tensor, q_raw: torch.Tensor, eta: torch.Tensor,
           keys: torch.Tensor, vals: torch.Tensor, n_before: int, m_res: torch.Tensor, b: int, t: int) -> torch.Tensor:
    """The step's three-field attention and M_res read-out (bolt3.py:365-402) for a window of any
    length. q_rope / q_raw: [b*H, t, HD] bf16 and eta [b*H, t] fp32 as bolt3_prep writes them; keys /
    vals: the window's RoPE'd keys and values [b*HKV, L, HD] bf16, of which the first n_before precede
    the step (query i sees window key j iff j <= n_before + i). Returns y [b, t, H, HD] bf16."""
    H, HKV, HD, G = ly.H, ly.HKV, ly.HD, ly.G
    L = keys.shape[1]
    scale = HD ** -0.5
    dev = keys.device
    with torch.autocast("cuda", enabled=False):
        qp = q_rope.float().view(b, HKV, G * t, HD)        # rows (g, i) of each KV head's query heads
        s_parts, v_parts = [], []
        if st.sinks_set:
            sk = st.sink_k.float().view(b, HKV, N_SINKS, HD)
            s_parts.append(torch.matmul(qp, sk.transpose(-1, -2)) * scale)
            v_parts.append(st.sink_v.float().view(b, HKV, N_SINKS, HD))
        if st.has_bank:
            bank, S = st.bank, ly.S
            s_att = torch.matmul(qp, bank["ak_rope"].float().view(b, HKV, S, HD).transpose(-1, -2)) * scale
            bias = consts["kappa"].view(1, HKV, 1, 1) * torch.log(bank["mass"].view(b, HKV, 1, S).clamp_min(1.0))
            act = bank["act"].view(b, HKV, 1, S).bool()
            s_parts.append((s_att + bias).masked_fill(~act, float("-inf")))
            v_parts.append(bank["av"].float().view(b, HKV, S, HD))
        s_loc = torch.matmul(qp, keys.float().view(b, HKV, L, HD).transpose(-1, -2)) * scale
        qi = torch.arange(G * t, device=dev) % t
        kj = torch.arange(L, device=dev)
        s_loc = s_loc.masked_fill(~(kj[None, :] <= n_before + qi[:, None]).view(1, 1, G * t, L), float("-inf"))
        s_parts.append(s_loc)
        v_parts.append(vals.float().view(b, HKV, L, HD))
        p = _bf(torch.softmax(torch.cat(s_parts, dim=-1), dim=-1))
        y = _bf(torch.matmul(p, torch.cat(v_parts, dim=2)))
        if st.has_bank:
            qn = F.normalize(q_raw.float().view(b, HKV, G * t, HD), dim=-1)
            ym = torch.matmul(qn, m_res.view(b, HKV, HD, HD)) * consts["coef"].view(1, HKV, 1, 1)
            ym = ym * torch.rsqrt(ym.pow(2).mean(-1, keepdim=True) + ly.eps) * consts["res_w"]
            y = _bf(y + _bf(eta.view(b, HKV, G * t, 1) * ym))
    return y.view(b, HKV, G, t, HD).permute(0, 3, 1, 2, 4).to(torch.bfloat16).contiguous().view(b, t, H, HD)


@torch.no_grad()
def consolidate(ly, st, consts: dict, m_res: torch.Tensor, kr: torch.Tensor, kp: torch.Tensor, v: torch.Tensor,
                pos: torch.Tensor, beta: torch.Tensor) -> None:
    """One `_consolidate_functional` call (bolt3.py:68-192) of l tokens on every chain of the state's
    bank, in place: kr / kp / v [b*HKV, l, HD] bf16, pos [l] fp32 positions, beta [b*HKV, l] fp32;
    m_res [b, HKV, HD, HD] fp32 (the caller's states[li]). Updates ak, av, mass, util, pm, act, the
    RoPE'd keys the attention reads and n_filled."""
    bank, S = st.bank, ly.S
    n, l_tok, HD = kr.shape
    b, HKV = st.B, ly.HKV
    dev = kr.device
    scale = HD ** -0.5
    inv_freq = consts["inv_freq"]
    with torch.autocast("cuda", enabled=False):
        if st.has_bank:                                                    # :83-92 (blank) or the bank
            ak, av = bank["ak"].float(), bank["av"].float()
            mass, util, pm = bank["mass"].clone(), bank["util"].clone(), bank["pm"].clone()
            act = bank["act"].bool()
            n_filled = st.n_filled
            M = m_res.view(n, HD, HD).clone()
        else:
            ak, av = torch.zeros(n, S, HD, device=dev), torch.zeros(n, S, HD, device=dev)
            mass, util, pm = torch.ones(n, S, device=dev), torch.zeros(n, S, device=dev), torch.zeros(n, S, device=dev)
            act = torch.zeros(n, S, dtype=torch.bool, device=dev)
            n_filled = 0
            M = torch.zeros(n, HD, HD, device=dev)
        p_f = pos.float().view(1, l_tok).expand(n, l_tok)
        util = util * GAMMA_U                                              # :94
        krf, kpf, v32 = kr.float(), kp.float(), v.float()
        kr_n = F.normalize(krf, dim=-1)

        def predict(mass_bias, masked):                                    # :97-103 / :169-174
            k_read = rope_slots(ak, pm, inv_freq).float()
            sc = torch.bmm(kpf, k_read.transpose(-1, -2)) * scale + mass_bias
            if masked:
                sc = sc.masked_fill(~act.unsqueeze(1), -1e9)
            v_hat = torch.bmm(_bf(torch.softmax(sc, dim=-1)), av)
            return (v32 - v_hat).norm(dim=-1) / (v32.norm(dim=-1) + 1e-6)

        if n_filled >= S:
            # full bank: prediction, cosine match, merge (:96-123)
            kap = consts["kappa"].repeat(b).view(n, 1, 1)
            rel_err = predict(kap * torch.log(mass.clamp_min(1.0)).unsqueeze(1), masked=False)
            cos_k = torch.bmm(kr_n, F.normalize(ak, dim=-1).transpose(-1, -2))
            best_sim_k, best_slot = cos_k.max(dim=-1)
            matched_av = torch.gather(av, 1, best_slot.unsqueeze(-1).expand(-1, -1, HD))
            sim_v = F.cosine_similarity(v32, matched_av, dim=-1)
            score_j = rel_err * (1.0 - best_sim_k.clamp(0.0, 1.0))
            merge = (best_sim_k >= SIM_K) & (sim_v >= SIM_V)
            onehot = F.one_hot(best_slot, num_classes=S).float() * merge.float().unsqueeze(-1)
            cnt = onehot.sum(dim=1)
            k_sum = torch.bmm(onehot.transpose(1, 2), krf)
            v_sum = torch.bmm(onehot.transpose(1, 2), v32)
            p_sum = torch.bmm(onehot.transpose(1, 2), p_f.unsqueeze(-1)).squeeze(-1)
            hit = cnt > 0
            new_m = mass + cnt
            ak = torch.where(hit.unsqueeze(-1), _bf((mass.unsqueeze(-1) * ak + k_sum) / new_m.unsqueeze(-1)), ak)
            av = torch.where(hit.unsqueeze(-1), _bf((mass.unsqueeze(-1) * av + v_sum) / new_m.unsqueeze(-1)), av)
            pm = torch.where(hit, (mass * pm + p_sum) / new_m, pm)
            mass = torch.where(hit, new_m, mass)
            # diversity eviction: novel tokens against the weakest slots, sorted greedy match (:125-152)
            ak_n = F.normalize(ak, dim=-1)
            eye = torch.eye(S, dtype=torch.bool, device=dev).unsqueeze(0)
            pair_cos = torch.bmm(ak_n, ak_n.transpose(-1, -2)).masked_fill(eye, -1.0)
            keep = util * (1.0 - pair_cos.max(dim=-1).values.clamp(0.0, 0.98))
            cand = torch.where(~merge, score_j, torch.full_like(score_j, -1e9))
            k_cand = min(l_tok, S)
            top_vals, top_toks = torch.topk(cand, k=k_cand, dim=-1, largest=True)
            bot_vals, bot_slots = torch.topk(keep, k=k_cand, dim=-1, largest=False)
            win = (top_vals > bot_vals) & (top_vals > -1e8)
            ins = torch.zeros_like(merge).scatter(1, top_toks, win)
            w3 = win.unsqueeze(-1)
            gidx = top_toks.unsqueeze(-1).expand(-1, -1, HD)
            sidx = bot_slots.unsqueeze(-1).expand(-1, -1, HD)
            ak = ak.scatter(1, sidx, torch.where(w3, torch.gather(krf, 1, gidx), torch.gather(ak, 1, sidx)))
            av = av.scatter(1, sidx, torch.where(w3, torch.gather(v32, 1, gidx), torch.gather(av, 1, sidx)))
            pm = pm.scatter(1, bot_slots, torch.where(win, torch.gather(p_f, 1, top_toks), torch.gather(pm, 1, bot_slots)))
            mass = mass.scatter(1, bot_slots, torch.where(win, torch.ones_like(bot_vals), torch.gather(mass, 1, bot_slots)))
            util = util.scatter(1, bot_slots, torch.where(win, torch.gather(rel_err, 1, top_toks),
                                                          torch.gather(util, 1, bot_slots)))
            # Gershgorin-normalised one-shot delta rule into M_res (:154-162)
            w_ev = beta.float() * (~merge & ~ins).float()
            gram = torch.bmm(kr_n, kr_n.transpose(-1, -2)).abs()
            gersh = torch.bmm(gram, w_ev.unsqueeze(-1)).squeeze(-1).clamp_min(1.0)
            err = (v32 - torch.bmm(kr_n, M)) * (w_ev / gersh).unsqueeze(-1)
            M = consts["gamma"].repeat(b).view(n, 1, 1) * M + torch.bmm(kr_n.transpose(1, 2), err)
        else:
            # fill path: the best m tokens take the next empty slots, the rest are dropped (:165-192)
            m = min(S - n_filled, l_tok)
            if n_filled > 0:
                rel_err = predict(torch.log(mass.clamp_min(1.0)).unsqueeze(1), masked=True)
                cos_k = torch.bmm(kr_n, F.normalize(ak, dim=-1).transpose(-1, -2)).masked_fill(~act.unsqueeze(1), 0.0)
                score_j = rel_err * (1.0 - cos_k.max(dim=-1).values.clamp(0.0, 1.0))
                init_u = rel_err
            else:
                score_j = F.normalize(v32, dim=-1).var(dim=-1)
                init_u = torch.full((n, l_tok), 0.15, device=dev)
            top_toks = torch.topk(score_j, k=m, dim=-1, largest=True).indices
            slots = torch.arange(n_filled, n_filled + m, device=dev).unsqueeze(0).expand(n, -1)
            gidx = top_toks.unsqueeze(-1).expand(-1, -1, HD)
            ak = ak.scatter(1, slots.unsqueeze(-1).expand(-1, -1, HD), torch.gather(krf, 1, gidx))
            av = av.scatter(1, slots.unsqueeze(-1).expand(-1, -1, HD), torch.gather(v32, 1, gidx))
            pm = pm.scatter(1, slots, torch.gather(p_f, 1, top_toks))
            mass = mass.scatter(1, slots, torch.ones(n, m, device=dev))
            util = util.scatter(1, slots, torch.gather(init_u, 1, top_toks))
            act = act.scatter(1, slots, torch.ones(n, m, dtype=torch.bool, device=dev))
            n_filled += m
        bank["ak"].copy_(ak)
        bank["av"].copy_(av)
        bank["mass"].copy_(mass)
        bank["util"].copy_(util)
        bank["pm"].copy_(pm)
        bank["act"].copy_(act.to(torch.uint8))
        bank["ak_rope"].copy_(rope_slots(bank["ak"], bank["pm"], inv_freq))
        bank["n_filled"].fill_(n_filled)
        m_res.view(n, HD, HD).copy_(M)
    st.n_filled = n_filled


@torch.no_grad()
@K.traced("oversize.layer_step")
def layer_step(ly, st, h: torch.Tensor, pos_start: int, m_res: torch.Tensor, partial_fp32: bool,
               consolidate_ring) -> torch.Tensor:
    """A Bolt-3 decoder step whose window holds, or whose step makes, a chunk of more than C tokens.
    `consolidate_ring(ly, st, m_res, consts)` consolidates a previous chunk of C tokens held in the
    window ring with the native kernel (and sets the sinks the first time)."""
    b, t, D = h.shape
    H, HKV, HD, C = ly.H, ly.HKV, ly.HD, ly.C
    n = b * HKV
    dev = h.device
    if st.cur_len == 0:
        st.slot_pos[st.cur_slot] = pos_start
    elif pos_start != st.slot_pos[st.cur_slot] + st.cur_len:
        raise NotImplementedError("native decoder needs contiguous positions within a chunk")
    f = ly.fused(dev)
    c = f.consts
    st._consts = c
    proj = F.linear(h.reshape(b * t, D).to(torch.bfloat16), f.w_in, f.b_in)
    bf = dict(dtype=torch.bfloat16, device=dev)
    q_raw, q_rope = torch.empty(b * H, t, HD, **bf), torch.empty(b * H, t, HD, **bf)
    eta = torch.empty(b * H, t, dtype=torch.float32, device=dev)
    c0, cl = st.cur_slot * C, st.cur_len
    big = cl + t > C
    common = dict(B=b, T=t, H=H, HKV=HKV, HD=HD, inv_freq=c["inv_freq"], eps=ly.eps, q_norm_w=c["qn"],
                  k_norm_w=c["kn"], pos0=pos_start, cols=f.cols, parts=3, q_raw=q_raw, q_rope=q_rope, eta=eta,
                  q_head_stride=t)
    if big:
        # the new rows go to buffers of their own; the current chunk becomes ring rows + these rows
        nk = [torch.empty(n, t, HD, **bf) for _ in range(3)]
        nb = torch.empty(n, t, dtype=torch.float32, device=dev)
        K.prep(proj, k_raw=nk[0], k_rope=nk[1], v=nk[2], beta=nb, k_head_stride=t, k_t_off=0, **common)
        cur = dict(kr=torch.cat([st.ring_kr[:, c0:c0 + cl], nk[0]], 1), kp=torch.cat([st.ring_kp[:, c0:c0 + cl], nk[1]], 1),
                   v=torch.cat([st.ring_v[:, c0:c0 + cl], nk[2]], 1), beta=torch.cat([st.ring_b[:, c0:c0 + cl], nb], 1))
    else:
        K.prep(proj, k_raw=st.ring_kr, k_rope=st.ring_kp, v=st.ring_v, beta=st.ring_b, k_head_stride=2 * C,
               k_t_off=c0 + cl, **common)
        cur = dict(kr=st.ring_kr[:, c0:c0 + cl + t], kp=st.ring_kp[:, c0:c0 + cl + t],
                   v=st.ring_v[:, c0:c0 + cl + t], beta=st.ring_b[:, c0:c0 + cl + t])
    if st.big_prev is not None:
        prev_kp, prev_v = st.big_prev["kp"], st.big_prev["v"]
    elif st.prev_slot >= 0:
        p0 = st.prev_slot * C
        prev_kp, prev_v = st.ring_kp[:, p0:p0 + C], st.ring_v[:, p0:p0 + C]
    else:
        prev_kp = prev_v = None
    n_prev = 0 if prev_kp is None else prev_kp.shape[1]
    keys = cur["kp"] if prev_kp is None else torch.cat([prev_kp, cur["kp"]], 1)
    vals = cur["v"] if prev_v is None else torch.cat([prev_v, cur["v"]], 1)
    y = attend(ly, st, c, q_rope, q_raw, eta, keys, vals, n_prev + cl, m_res, b, t)
    if partial_fp32:
        out = torch.mm(y.view(b * t, H * HD), f.w_out.t(), out_dtype=torch.float32).view(b, t, -1)
    else:
        out = F.linear(y.view(b, t, H * HD), f.w_out)
    new_len = cl + t
    if new_len < C:
        st.cur_len = new_len
        return out
    # the current chunk is complete: consolidate the previous one, then the current one is previous
    st.status.check(block=True)
    if st.big_prev is not None:
        bp = st.big_prev
        kr_, kp_, v_, b_, p0 = bp["kr"], bp["kp"], bp["v"], bp["beta"], bp["pos0"]
        if not st.sinks_set:                                               # :413-416
            st.sink_k.copy_(kp_[:, :N_SINKS])
            st.sink_v.copy_(v_[:, :N_SINKS])
            st.sinks_set = True
            kr_, kp_, v_, b_, p0 = kr_[:, N_SINKS:], kp_[:, N_SINKS:], v_[:, N_SINKS:], b_[:, N_SINKS:], p0 + N_SINKS
        pos = torch.arange(p0, p0 + kr_.shape[1], dtype=torch.float32, device=dev)
        consolidate(ly, st, c, m_res, kr_, kp_, v_, pos, b_)
        st.big_prev = None
    elif st.prev_slot >= 0:
        consolidate_ring(ly, st, m_res, c)
    if new_len > C:
        st.big_prev = dict(kr=cur["kr"].contiguous(), kp=cur["kp"].contiguous(), v=cur["v"].contiguous(),
                           beta=cur["beta"].contiguous(), pos0=st.slot_pos[st.cur_slot])
        st.prev_slot, st.cur_slot, st.cur_len = -1, 0, 0
    else:
        st.prev_slot, st.cur_slot, st.cur_len = st.cur_slot, 1 - st.cur_slot, 0
    st.status.arm(f"Bolt-3 decode chunk ending at position {pos_start + t}")
    return out
