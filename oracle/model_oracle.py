"""Model-level decode oracle for a hybrid Bolt-3 language model (test infrastructure only).

Restates, on the CPU in fp32 with `Store` deciding the stored precision, what the reference's
`Bolt3Decoder` does for a whole model:
- `step` (vsa_lm/config/bolt3.py:335-447): embedding; per block x += attention(norm1(x)) and
  x += mlp(norm2(x)) (vsa_lm/config/standard.py:360-363); final norm. Bolt-3 blocks use
  `LayerDecoderOracle`; softmax anchors append RoPE'd keys/values to a cache and attend causally
  within the new block (bolt3.py:426-445); the MLP is SwiGLU (vsa_lm/surgery.py:202-211).
- `memorize` / `forget` (bolt3.py:528-557): traces of the change a document made to M_res, and
  their decayed subtraction.
Parameters come as a state_dict with the reference's key layout (`embed_tokens.weight`,
`blocks.{i}.norm1.weight`, `blocks.{i}.vsa.*` or `blocks.{i}.attn.*`, `blocks.{i}.mlp.*`,
`norm.weight`, `lm_head.weight`).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .bolt3_oracle import LayerDecoderOracle, Store, gamma_delta, rms_norm, rope_at


def _sub(params: dict, prefix: str) -> dict:
    n = len(prefix)
    return {k[n:]: v for k, v in params.items() if k.startswith(prefix)}


class ModelDecoderOracle:
    """Decoder state and step of a hybrid model: `layer_types[i]` is "vsa" (Bolt-3) or "softmax"."""

    def __init__(self, params: dict, layer_cfg: dict, layer_types: list[str], b: int, store: Store,
                 eps: float, C: int = 128):
        self.p, self.cfg, self.types, self.b, self.store, self.eps, self.C = params, layer_cfg, layer_types, b, store, eps, C
        # optional callable (layer index, position) -> the Bolt-3 layer's projections as stored values
        # (LayerDecoderOracle.step's `proj`): checks the rest of the model on exactly the projections
        # another implementation computed
        self.proj_source = None
        # optional callable (layer index, position) -> a Bolt-3 layer's attention-branch output for
        # the step, used instead of stepping that layer here (its state is then advanced elsewhere)
        self.attn_source = None
        self.layers = []
        for i, t in enumerate(layer_types):
            if t == "vsa":
                self.layers.append(LayerDecoderOracle(_sub(params, f"blocks.{i}.vsa."), layer_cfg, b, store, C=C))
            else:
                self.layers.append({"k": None, "v": None})

    def _lin(self, x, w):
        return self.store(x @ w.float().t())

    def _anchor(self, i: int, h: torch.Tensor, pos_start: int) -> torch.Tensor:
        p, cfg, st = _sub(self.p, f"blocks.{i}.attn."), self.cfg, self.store
        b, t, _ = h.shape
        H, HKV, HD = cfg["H"], cfg["HKV"], cfg["HD"]
        q = self._lin(h, p["q_proj.weight"]).view(b, t, H, HD)
        k = self._lin(h, p["k_proj.weight"]).view(b, t, HKV, HD)
        v = self._lin(h, p["v_proj.weight"]).view(b, t, HKV, HD)
        if "q_norm.weight" in p:
            q, k = rms_norm(q, p["q_norm.weight"], cfg["eps"], st), rms_norm(k, p["k_norm.weight"], cfg["eps"], st)
        q, k, v = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
        pos = torch.arange(pos_start, pos_start + t, dtype=torch.float32)
        q, k = rope_at(q, pos, cfg["inv_freq"], st), rope_at(k, pos, cfg["inv_freq"], st)
        cache = self.layers[i]
        cache["k"] = k if cache["k"] is None else torch.cat([cache["k"], k], dim=2)
        cache["v"] = v if cache["v"] is None else torch.cat([cache["v"], v], dim=2)
        n = cache["k"].shape[2]
        G = H // HKV
        kk, vv = cache["k"].repeat_interleave(G, dim=1), cache["v"].repeat_interleave(G, dim=1)
        s = q @ kk.transpose(-1, -2) / HD ** 0.5
        if t > 1:
            qi = torch.arange(t)[:, None]
            kj = torch.arange(n)[None, :]
            s = s.masked_fill(~(kj <= n - t + qi), float("-inf"))
        y = st(torch.softmax(s, dim=-1) @ vv)
        return self._lin(y.transpose(1, 2).reshape(b, t, H * HD), p["o_proj.weight"])

    def step(self, tokens: torch.Tensor, pos_start: int) -> torch.Tensor:
        """Final normed hidden states [b, t, D] of the new tokens (stored values)."""
        st, p = self.store, self.p
        x = st(p["embed_tokens.weight"].float()[tokens])
        for i, t in enumerate(self.types):
            h = rms_norm(x, p[f"blocks.{i}.norm1.weight"], self.eps, st)
            if t == "vsa" and self.attn_source is not None:
                a = self.attn_source(i, pos_start)
            elif t == "vsa":
                proj = self.proj_source(i, pos_start) if self.proj_source is not None else None
                a = self.layers[i].step(h, pos_start, proj=proj)
            else:
                a = self._anchor(i, h, pos_start)
            x = st(x + a)
            h2 = rms_norm(x, p[f"blocks.{i}.norm2.weight"], self.eps, st)
            g = self._lin(h2, p[f"blocks.{i}.mlp.gate_proj.weight"])
            u = self._lin(h2, p[f"blocks.{i}.mlp.up_proj.weight"])
            x = st(x + self._lin(st(st(F.silu(g)) * u), p[f"blocks.{i}.mlp.down_proj.weight"]))
        return rms_norm(x, p["norm.weight"], self.eps, st)

    def logits(self, h_last: torch.Tensor) -> torch.Tensor:
        return h_last @ self.p["lm_head.weight"].float().t()

    def feed(self, ids: torch.Tensor, pos: int):
        """C-token slices of a prompt from `pos`; (last hidden states, next position)."""
        h = None
        for s in range(0, ids.shape[1], self.C):
            piece = ids[:, s:s + self.C]
            h = self.step(piece, pos)
            pos += piece.shape[1]
        return h, pos

    def m_res(self, i: int) -> torch.Tensor:
        return self.layers[i].m_res

    def memorize(self, ids: torch.Tensor, pos: int):
        """Feed a document; per Bolt-3 layer the trace (end position, M_after - gamma^(n // C) M_before)
        (bolt3.py:528-545). Returns (next position, traces)."""
        before = {i: self.layers[i].m_res.clone() for i, t in enumerate(self.types) if t == "vsa"}
        _, pos = self.feed(ids, pos)
        traces = []
        for i, t in enumerate(self.types):
            if t != "vsa":
                traces.append(None)
                continue
            gam = gamma_delta(self.p[f"blocks.{i}.vsa.log_gamma"]).view(1, -1, 1, 1)
            traces.append((pos, self.layers[i].m_res - gam ** (ids.shape[1] // self.C) * before[i]))
        return pos, traces

    def forget(self, traces, next_pos: int) -> None:
        """M_res -= gamma^max(0, (next_pos - end) // C) * delta per traced layer (bolt3.py:547-557)."""
        for i, tr in enumerate(traces):
            if tr is None:
                continue
            end, delta = tr
            gam = gamma_delta(self.p[f"blocks.{i}.vsa.log_gamma"]).view(1, -1, 1, 1)
            self.layers[i].m_res = self.layers[i].m_res - gam ** max(0, (next_pos - end) // self.C) * delta
