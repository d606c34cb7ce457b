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

from .bolt3 import Bolt3Attn, Bolt3Decoder, Bolt3LayerState


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
