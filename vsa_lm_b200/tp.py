"""Tensor parallelism of a Bolt-3 layer by KV head.

Every Bolt-3 field (sinks, local window, attractor bank, M_res) belongs to one (sequence, KV head)
chain and nothing mixes chains (vsa_lm/config/bolt3.py:73-80 flattens the batch to b*HKV chains).
A rank therefore owns a contiguous block of KV heads, the G query heads of each (query head h
reads KV head h // G, as repeat_kv does), the matching rows of the q/k/v/beta/eta projections, the
matching columns of o_proj and the per-KV-head constants (kappa, log_gamma). Its forward yields a
partial o_proj sum; one all-reduce over the group completes the layer. This is the only
collective: the attention itself has no exchange step. The partial sums stay in fp32 (o_proj's
bf16 GEMM writes them unrounded) and are rounded to bf16 once, after the all-reduce, as the
unsharded layer rounds its single GEMM.
"""
from __future__ import annotations


import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from .bolt3 import Bolt3Attn, Bolt3Decoder, Bolt3LayerState
from .model import LlamaMLP, SoftmaxAttn


def kv_head_range(HKV: int, rank: int, world: int) -> tuple[int, int]:
    """KV heads [k0, k1) of `rank` when HKV heads are split evenly over `world` ranks."""
    if world <= 0 or HKV % world:
        raise ValueError(f"{HKV} KV heads do not split evenly over {world} ranks")
    n = HKV // world
    return rank * n, (rank + 1) * n


@torch.no_grad()
def shard_by_kv_head(layer: Bolt3Attn, rank: int, world: int) -> Bolt3Attn:
    """A Bolt3Attn holding this rank's KV heads of `layer` (same dtype and device). Its forward
    returns the rank's partial o_proj output: the sum over ranks is the full layer's output."""
    k0, k1 = kv_head_range(layer.HKV, rank, world)
    G, HD = layer.G, layer.HD
    q0, q1 = k0 * G, k1 * G
    D = layer.q_proj.weight.shape[1]
    cfg = dict(dim=D, num_heads=q1 - q0, num_kv_heads=k1 - k0, head_dim=HD, eps=layer.eps,
               rope_theta=1.0, qkv_bias=layer.q_proj.bias is not None, qk_norm=layer.q_norm is not None)
    ref = layer.q_proj.weight
    local = Bolt3Attn(cfg, S=layer.S, C=layer.C).to(dtype=ref.dtype, device=ref.device)
    local.rope.inv_freq.copy_(layer.rope.inv_freq)           # the frequencies, whatever their scaling
    rows = lambda lin, a, b: (lin.weight[a:b], None if lin.bias is None else lin.bias[a:b])

    def put(dst, src):
        w, b = src
        dst.weight.copy_(w)
        if b is not None:
            dst.bias.copy_(b)

    put(local.q_proj, rows(layer.q_proj, q0 * HD, q1 * HD))
    put(local.k_proj, rows(layer.k_proj, k0 * HD, k1 * HD))
    put(local.v_proj, rows(layer.v_proj, k0 * HD, k1 * HD))
    put(local.beta_proj, rows(layer.beta_proj, k0, k1))
    put(local.eta_proj, rows(layer.eta_proj, q0, q1))
    local.o_proj.weight.copy_(layer.o_proj.weight[:, q0 * HD:q1 * HD])
    local.kappa.copy_(layer.kappa[k0:k1])
    local.log_gamma.copy_(layer.log_gamma[k0:k1])
    local.res_norm.weight.copy_(layer.res_norm.weight)
    if layer.q_norm is not None:
        local.q_norm.weight.copy_(layer.q_norm.weight)
        local.k_norm.weight.copy_(layer.k_norm.weight)
    local.sim_k, local.sim_v, local.gamma_u = layer.sim_k, layer.sim_v, layer.gamma_u
    return local


class Bolt3AttnTP(torch.nn.Module):
    """A Bolt-3 layer split by KV head over a process group: the rank's shard runs the native
    forward (or decode step) and the partial outputs meet in one all-reduce (NCCL over NVLink on a
    GPU group). Drop-in for Bolt3Attn.forward on every rank of the group."""

    def __init__(self, layer: Bolt3Attn, group=None):
        super().__init__()
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.local = shard_by_kv_head(layer, self.rank, self.world)

    def reduce(self, partial: torch.Tensor, dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
        """Sum the fp32 partial outputs of all ranks, then round once."""
        if self.world > 1:
            dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=self.group)
        return partial.to(dtype)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.reduce(self.local._native_forward(x, partial_fp32=True), x.dtype)

    def new_decode_state(self, B: int, device) -> tuple[Bolt3LayerState, torch.Tensor]:
        """This rank's decoder state and M_res ([B, HKV/world, HD, HD] fp32)."""
        ly = self.local
        return Bolt3LayerState(ly, B, device), torch.zeros(B, ly.HKV, ly.HD, ly.HD, device=device)

    def decode_step(self, st: Bolt3LayerState, h: torch.Tensor, pos_start: int, m_res: torch.Tensor) -> torch.Tensor:
        """Bolt3Decoder.layer_step on this rank's KV heads, then the all-reduce of o_proj."""
        return self.reduce(Bolt3Decoder.layer_step(self.local, st, h, pos_start, m_res, partial_fp32=True))


# ---- the whole hybrid model split by KV head, with the MLP split by column

def _linear_rows(lin: nn.Linear, a: int, b: int) -> nn.Linear:
    """Output features [a, b) of `lin` (a column-parallel piece: its outputs are complete)."""
    w = lin.weight
    out = nn.Linear(w.shape[1], b - a, bias=lin.bias is not None, device=w.device, dtype=w.dtype)
    with torch.no_grad():
        out.weight.copy_(w[a:b])
        if lin.bias is not None:
            out.bias.copy_(lin.bias[a:b])
    return out


def _linear_cols(lin: nn.Linear, a: int, b: int) -> nn.Linear:
    """Input features [a, b) of a bias-free `lin` (a row-parallel piece: its outputs are partial sums)."""
    if lin.bias is not None:
        raise NotImplementedError("a row-parallel split of a linear layer with a bias is not supported")
    w = lin.weight
    out = nn.Linear(b - a, w.shape[0], bias=False, device=w.device, dtype=w.dtype)
    with torch.no_grad():
        out.weight.copy_(w[:, a:b])
    return out


@torch.no_grad()
def shard_softmax_attn(attn: SoftmaxAttn, rank: int, world: int) -> SoftmaxAttn:
    """A softmax anchor layer holding this rank's KV heads, their G query heads and the matching
    o_proj columns (standard.py:55-123 split the way shard_by_kv_head splits a Bolt-3 layer). The
    per-head norms and the RoPE frequencies are the layer's own."""
    k0, k1 = kv_head_range(attn.HKV, rank, world)
    G, HD = attn.G, attn.HD
    q0, q1 = k0 * G, k1 * G
    w = attn.q_proj.weight
    eps = attn.q_norm.eps if attn.q_norm is not None else 1e-5
    cfg = dict(dim=w.shape[1], num_heads=q1 - q0, num_kv_heads=k1 - k0, head_dim=HD, eps=eps, rope_theta=1.0,
               qkv_bias=attn.q_proj.bias is not None, qk_norm=attn.q_norm is not None)
    with torch.device(w.device):
        local = SoftmaxAttn(cfg).to(w.dtype)
    local.q_proj = _linear_rows(attn.q_proj, q0 * HD, q1 * HD)
    local.k_proj = _linear_rows(attn.k_proj, k0 * HD, k1 * HD)
    local.v_proj = _linear_rows(attn.v_proj, k0 * HD, k1 * HD)
    local.o_proj = _linear_cols(attn.o_proj, q0 * HD, q1 * HD)
    if attn.q_norm is not None:
        local.q_norm.weight.copy_(attn.q_norm.weight)
        local.k_norm.weight.copy_(attn.k_norm.weight)
    local.rope.inv_freq = attn.rope.inv_freq.clone()
    return local


@torch.no_grad()
def shard_mlp(mlp: LlamaMLP, rank: int, world: int) -> LlamaMLP:
    """This rank's block of the SwiGLU intermediate features: rows of gate/up, columns of down."""
    D, n = mlp.gate_proj.weight.shape[1], mlp.gate_proj.weight.shape[0]
    if n % world:
        raise ValueError(f"{n} intermediate features do not split evenly over {world} ranks")
    i0, i1 = rank * n // world, (rank + 1) * n // world
    with torch.device("meta"):
        local = LlamaMLP(dict(dim=D, intermediate=i1 - i0))
    local.gate_proj = _linear_rows(mlp.gate_proj, i0, i1)
    local.up_proj = _linear_rows(mlp.up_proj, i0, i1)
    local.down_proj = _linear_cols(mlp.down_proj, i0, i1)
    return local


def _mm_fp32(x: torch.Tensor, lin: nn.Linear) -> torch.Tensor:
    """x @ lin.weight^T with the products summed and returned in fp32, unrounded."""
    w = lin.weight
    x2 = x.reshape(-1, x.shape[-1])
    if x2.is_cuda:
        out = torch.mm(x2.to(w.dtype), w.t(), out_dtype=torch.float32)
    else:   # the CPU has no mixed-output GEMM: the same products and fp32 sums from fp32 operands
        out = torch.mm(x2.to(w.dtype).float(), w.float().t())
    return out.view(*x.shape[:-1], -1)


def mlp_partial(mlp: LlamaMLP, x: torch.Tensor) -> torch.Tensor:
    """A column shard's share of the SwiGLU MLP: its intermediate features are complete, down_proj
    gives an fp32 partial sum."""
    return _mm_fp32(mlp.act(x), mlp.down_proj)


def anchor_partial(attn: SoftmaxAttn, x: torch.Tensor) -> torch.Tensor:
    """A KV-head shard's share of a softmax anchor over a whole sequence (causal; RoPE from 0):
    the attention of its heads is complete, o_proj gives an fp32 partial sum."""
    B, T, _ = x.shape
    q, k, v = attn.head_qkv(x)
    q, k = attn.rope(q), attn.rope(k)
    y = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=attn.G > 1)
    return _mm_fp32(y.transpose(1, 2).reshape(B, T, attn.H * attn.HD), attn.o_proj)


class _TPBlock(nn.Module):
    def __init__(self, blk, rank: int, world: int):
        super().__init__()
        self.norm1, self.norm2 = blk.norm1, blk.norm2
        if hasattr(blk, "vsa"):
            self.vsa = shard_by_kv_head(blk.vsa, rank, world)
        else:
            self.attn = shard_softmax_attn(blk.attn, rank, world)
        self.mlp = shard_mlp(blk.mlp, rank, world)


class Bolt3LMTP(nn.Module):
    """The hybrid model (Bolt3LM) split over a process group: every attention layer, Bolt-3 or softmax
    anchor, by KV head (its query heads, projection rows and o_proj columns), and every SwiGLU MLP
    by intermediate feature (gate/up rows, down_proj columns). Each attention and each MLP ends in
    one all-reduce of fp32 partial sums (NCCL over NVLink on a GPU group), rounded to bf16 once as
    the unsharded bf16 GEMM rounds its output. The embedding, the norms and the LM head are
    replicated. The attribute names follow Bolt3LM, so Bolt3Decoder.blank_state builds this rank's
    (KV-head) state and Bolt3DecoderTP steps it. Without an initialised process group it is the
    whole model on one rank (no collective)."""

    def __init__(self, model, group=None):
        super().__init__()
        on = dist.is_available() and dist.is_initialized()
        self.group = group
        self.rank = dist.get_rank(group) if on else 0
        self.world = dist.get_world_size(group) if on else 1
        self.config = dict(model.config)
        self.embed_tokens, self.norm, self.lm_head = model.embed_tokens, model.norm, model.lm_head
        self.blocks = nn.ModuleList([_TPBlock(b, self.rank, self.world) for b in model.blocks])

    def reduce(self, partial: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
        """Sum the fp32 partials of all ranks in place, then round once."""
        if self.world > 1:
            dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=self.group)
        return partial.to(dtype)

    @torch.no_grad()
    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        """Whole-sequence forward (Bolt3LM.forward): final normed hidden states [B, T, D]."""
        x = self.embed_tokens(input_ids)
        for blk in self.blocks:
            h = blk.norm1(x)
            part = blk.vsa._native_forward(h, partial_fp32=True) if hasattr(blk, "vsa") else anchor_partial(blk.attn, h)
            x = x + self.reduce(part, x.dtype)
            x = x + self.reduce(mlp_partial(blk.mlp, blk.norm2(x)), x.dtype)
        return self.norm(x)


class Bolt3DecoderTP(Bolt3Decoder):
    """Bolt3Decoder over a Bolt3LMTP: every rank keeps the decode state of its KV heads (Bolt-3
    banks, M_res, windows and the anchors' KV caches) and runs the same steps; the partial outputs
    of each attention and each MLP meet in an all-reduce. Every rank sees the same logits, so greedy
    decoding agrees without communication; sampled tokens are drawn on rank 0 and broadcast."""

    def __init__(self, model: Bolt3LMTP, **kwargs):
        if not isinstance(model, Bolt3LMTP):
            raise TypeError("Bolt3DecoderTP drives a Bolt3LMTP")
        super().__init__(model, **kwargs)

    def _blocks(self, tokens: torch.Tensor, pos_start: int, states, kv_caches, dev_pos=None) -> torch.Tensor:
        m = self.model
        blocks = m.blocks
        with torch.autocast("cuda", torch.bfloat16, enabled=tokens.is_cuda):
            x = m.embed_tokens(tokens)
            h = blocks[0].norm1(x)
            for li, blk in enumerate(blocks):
                if hasattr(blk, "vsa"):
                    if dev_pos is None:
                        part = self.layer_step(blk.vsa, kv_caches[li], h, pos_start, states[li], partial_fp32=True)
                    else:
                        part = self._layer_launch(blk.vsa, kv_caches[li], h, pos_start, states[li],
                                                  partial_fp32=True, dev_pos=dev_pos)
                else:
                    part = self._anchor_attention(blk.attn, kv_caches[li], h, pos_start, partial_fp32=True,
                                                  dev_pos=dev_pos)
                x, h2 = blk.norm2.add_forward(x, m.reduce(part, x.dtype))
                nxt = blocks[li + 1].norm1 if li + 1 < len(blocks) else m.norm
                x, h = nxt.add_forward(x, m.reduce(mlp_partial(blk.mlp, h2), x.dtype))
            return h

    def graphs_supported(self, device) -> bool:
        """CUDA graphs capture NCCL collectives; a gloo group's all-reduces run on the host."""
        m = self.model
        if m.world > 1 and dist.get_backend(m.group) != "nccl":
            return False
        return super().graphs_supported(device)

    def _sample(self, logits, temperature: float, top_k: int = 40, top_p: float = 0.95):
        nxt = Bolt3Decoder._sample(logits, temperature, top_k=top_k, top_p=top_p)
        if temperature > 0 and self.model.world > 1:
            dist.broadcast(nxt, src=dist.get_global_rank(self.model.group, 0) if self.model.group else 0,
                           group=self.model.group)
        return nxt
