"""Minimal hybrid language-model shell for Bolt-3 configurations.

Mirrors the parts of the reference's `UniversalVSALM` / `UniversalBlock` (vsa_lm/config/standard.py:
341-404) that a Bolt-3 model uses: token embedding, blocks of (RMSNorm, Bolt-3 or softmax attention,
RMSNorm, SwiGLU MLP), final norm and LM head, with the same attribute names (`embed_tokens`,
`blocks[i].norm1/.vsa/.attn/.norm2/.mlp`, `norm`, `lm_head`, `config`) so `Bolt3Decoder` drives
either model. Layer placement follows compute_layer_types (vsa_lm/config/inspector.py:42-58).
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from .bolt3 import Bolt3Attn, LlamaRMSNorm, LlamaRoPE


def compute_layer_types(num_layers: int, hybrid_every: int) -> list[str]:
    """Every hybrid_every-th layer is a softmax anchor, the rest are Bolt-3 (inspector.py:55-58)."""
    return ["softmax" if (hybrid_every > 0 and (li + 1) % hybrid_every == 0) else "vsa" for li in range(num_layers)]


class LlamaMLP(nn.Module):
    """SwiGLU MLP (vsa_lm/surgery.py:202-211)."""

    def __init__(self, cfg: dict):
        super().__init__()
        D, I = cfg["dim"], cfg["intermediate"]
        self.gate_proj = nn.Linear(D, I, bias=False)
        self.up_proj = nn.Linear(D, I, bias=False)
        self.down_proj = nn.Linear(I, D, bias=False)

    def _gate_up_weight(self) -> torch.Tensor:
        """One [2I, D] weight whose halves are the gate and up parameters' own storage: the first call
        moves the two parameters into it (no second copy of the weights), later calls return it as long
        as the parameters still live there (a weight load copies into them in place; a replaced
        parameter or a device move makes it again)."""
        g, u = self.gate_proj.weight, self.up_proj.weight
        w = getattr(self, "_gu", None)
        if w is None or w.data_ptr() != g.data_ptr() or w[g.shape[0]:].data_ptr() != u.data_ptr() \
                or w.dtype != g.dtype or w.device != g.device:
            with torch.no_grad():
                w = torch.cat([g, u], 0)
                self.gate_proj.weight.data = w[:g.shape[0]]
                self.up_proj.weight.data = w[g.shape[0]:]
            self._gu = w
        return w

    def act(self, x):
        """silu(gate_proj(x)) * up_proj(x): for bf16 CUDA inputs outside autograd the two projections
        are one GEMM and the elementwise step one kernel (csrc/silu_mul.cu), with torch's roundings."""
        g = self.gate_proj.weight
        if (x.is_cuda and g.is_cuda and g.dtype == torch.bfloat16 and g.shape[0] % 8 == 0
                and not (torch.is_grad_enabled() and (x.requires_grad or g.requires_grad))):
            from . import kernels as K

            return K.silu_mul(F.linear(x.to(g.dtype), self._gate_up_weight()))
        return F.silu(self.gate_proj(x)) * self.up_proj(x)

    def forward(self, x):
        return self.down_proj(self.act(x))


class SoftmaxAttn(nn.Module):
    """Causal GQA softmax anchor layer (the plain form of standard.py:55-123)."""

    def __init__(self, cfg: dict):
        super().__init__()
        D, H, HKV = cfg["dim"], cfg["num_heads"], cfg["num_kv_heads"]
        HD = cfg.get("head_dim") or D // H
        self.H, self.HKV, self.HD, self.G = H, HKV, HD, H // HKV
        bias = bool(cfg.get("qkv_bias", False))
        self.q_proj = nn.Linear(D, H * HD, bias=bias)
        self.k_proj = nn.Linear(D, HKV * HD, bias=bias)
        self.v_proj = nn.Linear(D, HKV * HD, bias=bias)
        self.o_proj = nn.Linear(H * HD, D, bias=False)
        if cfg.get("qk_norm", False):
            self.q_norm, self.k_norm = LlamaRMSNorm(HD, cfg["eps"]), LlamaRMSNorm(HD, cfg["eps"])
        else:
            self.q_norm = self.k_norm = None
        self.rope = LlamaRoPE(HD, cfg["rope_theta"], cfg.get("rope_scaling"))

    def head_qkv(self, x):
        B, T, _ = x.shape
        q = self.q_proj(x).view(B, T, self.H, self.HD)
        k = self.k_proj(x).view(B, T, self.HKV, self.HD)
        v = self.v_proj(x).view(B, T, self.HKV, self.HD)
        if self.q_norm is not None:
            q, k = self.q_norm(q), self.k_norm(k)
        return q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)

    def forward(self, x):
        B, T, _ = x.shape
        q, k, v = self.head_qkv(x)
        q, k = self.rope(q), self.rope(k)
        y = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=self.G > 1)
        return self.o_proj(y.transpose(1, 2).reshape(B, T, self.H * self.HD))


class Block(nn.Module):
    def __init__(self, cfg: dict, attn_type: str, max_T: int):
        super().__init__()
        self.norm1 = LlamaRMSNorm(cfg["dim"], cfg["eps"])
        if attn_type == "vsa":
            self.vsa = Bolt3Attn(cfg, max_T=max_T, S=int(cfg.get("bolt3_S", 128)), C=int(cfg.get("bolt3_C", 128)))
        else:
            self.attn = SoftmaxAttn(cfg)
        self.norm2 = LlamaRMSNorm(cfg["dim"], cfg["eps"])
        self.mlp = LlamaMLP(cfg)

    def forward(self, x):
        attn = self.vsa if hasattr(self, "vsa") else self.attn
        x = x + attn(self.norm1(x))
        return x + self.mlp(self.norm2(x))


class Bolt3LM(nn.Module):
    """Hybrid LM with Bolt-3 layers and softmax anchors (UniversalVSALM with is_bolt3=True)."""

    def __init__(self, vocab_size: int, dim: int, num_layers: int, num_heads: int, num_kv_heads: int,
                 intermediate: int, max_T: int = 2048, hybrid_every: int = 4, rope_theta: float = 1e4,
                 rope_scaling: dict | None = None, eps: float = 1e-5, head_dim: int | None = None,
                 qk_norm: bool = False, tie_word_embeddings: bool = True, **extra):
        super().__init__()
        head_dim = head_dim or dim // num_heads
        layer_types = extra.pop("layer_types", None) or compute_layer_types(num_layers, hybrid_every)
        self.config = dict(vocab_size=vocab_size, dim=dim, num_layers=num_layers, num_heads=num_heads,
                           num_kv_heads=num_kv_heads, intermediate=intermediate, max_T=max_T,
                           hybrid_every=hybrid_every, rope_theta=rope_theta, rope_scaling=rope_scaling,
                           eps=eps, head_dim=head_dim, qk_norm=qk_norm, layer_types=layer_types,
                           is_bolt3=True, bolt3_S=128, bolt3_C=128, **extra)
        self.embed_tokens = nn.Embedding(vocab_size, dim)
        self.blocks = nn.ModuleList([Block(self.config, lt, max_T) for lt in layer_types])
        self.norm = LlamaRMSNorm(dim, eps)
        self.lm_head = nn.Linear(dim, vocab_size, bias=False)
        if tie_word_embeddings:
            self.lm_head.weight = self.embed_tokens.weight

    def forward(self, input_ids):
        x = self.embed_tokens(input_ids)
        for blk in self.blocks:
            x = blk(x)
        return self.norm(x)
