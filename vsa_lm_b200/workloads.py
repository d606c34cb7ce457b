"""Seeded synthetic workloads for the Bolt-3 hot path.

No public dataset is involved: every input is a seeded synthetic tensor whose shapes and value
distributions follow the five benchmark configurations of the project (configs[0..4]). Parameters
are drawn from an explicit torch.Generator in a fixed order, so the same seed gives the same weights
for the reference module, the CPU oracle and the CUDA drop-in (the dict keys are the reference's
`Bolt3Attn` state_dict keys, vsa_lm/config/bolt3.py:33-54).

Deviation from the reference initialisation (documented on purpose): the reference zero-initialises
`beta_proj.weight` and `eta_proj.weight` (bolt3.py:47,50), which would make eta identically 0 and
hide the M_res read-out. Here they are drawn N(0, 0.02); `kappa`, `log_gamma`, the q/k norm weights
are perturbed around their init values so that per-head parameters are exercised.
"""
from __future__ import annotations

import math

import torch

# Layer shapes. `eps` / `theta` follow the donor families named by each config (Qwen3-4B: eps 1e-6,
# theta 1e6, qk_norm; Llama-3-8B: eps 1e-5, theta 5e5). configs[0] names no theta: 1e4 is used.
SHAPES = {
    "tiny": dict(dim=256, num_heads=4, num_kv_heads=2, head_dim=64, rope_theta=1e4, eps=1e-5, qk_norm=False),
    "config0": dict(dim=960, num_heads=15, num_kv_heads=5, head_dim=64, rope_theta=1e4, eps=1e-5, qk_norm=False),
    "qwen3_4b": dict(dim=2560, num_heads=32, num_kv_heads=8, head_dim=128, rope_theta=1e6, eps=1e-6, qk_norm=True),
    "llama3_8b": dict(dim=4096, num_heads=32, num_kv_heads=8, head_dim=128, rope_theta=5e5, eps=1e-5, qk_norm=False),
}

# Workloads (batch, sequence, near-duplicate fraction) of the benchmark configurations.
WORKLOADS = {
    "config0": dict(shape="config0", B=1, T=1024, dup="chunks"),
    "config1": dict(shape="qwen3_4b", B=8, T=8192, dup=0.3),
    "config2": dict(shape="qwen3_4b", B=256, T=4096, dup=0.3, decode_steps=512),
    "config4": dict(shape="llama3_8b", B=1, T=131072, dup=0.2),
}


def layer_cfg(shape: str | dict, **over) -> dict:
    """Reference-style cfg dict for `Bolt3Attn(cfg)` (keys read at bolt3.py:26-42)."""
    cfg = dict(SHAPES[shape]) if isinstance(shape, str) else dict(shape)
    cfg.update(over)
    return cfg


def make_params(cfg: dict, seed: int = 0, qkv_bias: bool | None = None) -> dict:
    """Seeded parameters with the reference's state_dict keys (fp32, CPU)."""
    g = torch.Generator().manual_seed(seed)
    D, H, HKV = int(cfg["dim"]), int(cfg["num_heads"]), int(cfg["num_kv_heads"])
    HD = int(cfg.get("head_dim") or D // H)
    bias = bool(cfg.get("qkv_bias", False)) if qkv_bias is None else qkv_bias

    def lin_w(n_out, n_in):
        bound = 1.0 / math.sqrt(n_in)
        return (torch.rand(n_out, n_in, generator=g) * 2 - 1) * bound

    p = {}
    p["q_proj.weight"] = lin_w(H * HD, D)
    if bias:
        p["q_proj.bias"] = (torch.rand(H * HD, generator=g) * 2 - 1) / math.sqrt(D)
    p["k_proj.weight"] = lin_w(HKV * HD, D)
    if bias:
        p["k_proj.bias"] = (torch.rand(HKV * HD, generator=g) * 2 - 1) / math.sqrt(D)
    p["v_proj.weight"] = lin_w(HKV * HD, D)
    if bias:
        p["v_proj.bias"] = (torch.rand(HKV * HD, generator=g) * 2 - 1) / math.sqrt(D)
    p["o_proj.weight"] = lin_w(D, H * HD)
    if cfg.get("qk_norm", False):
        p["q_norm.weight"] = 1.0 + 0.05 * torch.randn(HD, generator=g)
        p["k_norm.weight"] = 1.0 + 0.05 * torch.randn(HD, generator=g)
    p["kappa"] = 1.0 + 0.1 * torch.randn(HKV, generator=g)
    p["log_gamma"] = 3.5 + 0.5 * torch.randn(HKV, generator=g)
    p["beta_proj.weight"] = 0.02 * torch.randn(HKV, D, generator=g)
    p["beta_proj.bias"] = torch.full((HKV,), -1.0)
    p["eta_proj.weight"] = 0.02 * torch.randn(H, D, generator=g)
    p["eta_proj.bias"] = torch.zeros(H)
    p["res_norm.weight"] = torch.full((HD,), 0.05)
    return p


def make_input(B: int, T: int, D: int, dup=0.0, seed: int = 1, C: int = 128,
               device="cpu", dtype=torch.float32) -> torch.Tensor:
    """Hidden states x ~ N(0, 1) with near-duplicate tokens that drive the merge path.

    dup = "chunks": every 4th chunk (3, 7, ...) repeats the chunk two before it plus N(0, 0.05^2)
    noise. dup = f (float): a fraction f of the tokens at t >= 2C are copies of a token
    src <= t - C plus N(0, 0.05^2) noise, src uniform (configs[1], [2], [4]).
    """
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(B, T, D, generator=g, device=device, dtype=torch.float32)
    if dup == "chunks":
        for c in range(3, (T + C - 1) // C, 4):
            s, e = c * C, min(T, (c + 1) * C)
            src = (c - 2) * C
            x[:, s:e] = x[:, src:src + (e - s)] + 0.05 * torch.randn(B, e - s, D, generator=g, device=device)
    elif dup and T > 2 * C:
        t = torch.arange(2 * C, T, device=device)
        pick = torch.rand(B, t.numel(), generator=g, device=device) < float(dup)
        src = (torch.rand(B, t.numel(), generator=g, device=device) * (t - C + 1).float()).long()
        src = torch.minimum(src, t - C)
        noise = 0.05 * torch.randn(B, t.numel(), D, generator=g, device=device)
        for bi in range(B):
            tt = t[pick[bi]]
            # read sources from the clean copy so that chains of copies stay near their origin
            x[bi, tt] = x[bi, src[bi, pick[bi]]] + noise[bi, pick[bi]]
    return x.to(dtype)


# Hybrid model shapes for the decoder-level tests (Bolt3LM keyword arguments). "tiny_lm" has two
# Bolt-3 layers and one softmax anchor (hybrid_every = 3).
MODEL_SHAPES = {
    "tiny_lm": dict(vocab_size=512, dim=256, num_layers=3, num_heads=4, num_kv_heads=2, head_dim=64,
                    intermediate=512, hybrid_every=3, rope_theta=1e4, eps=1e-5, qk_norm=False,
                    tie_word_embeddings=False),
    # head_dim 128 with qk_norm (the one-token streaming attention kernel), three Bolt-3 layers and an anchor
    "small_lm": dict(vocab_size=1024, dim=512, num_layers=4, num_heads=8, num_kv_heads=2, head_dim=128,
                     intermediate=1024, hybrid_every=4, rope_theta=1e6, eps=1e-6, qk_norm=True,
                     tie_word_embeddings=True),
    # the Qwen3-4B architecture as a hybrid (27 Bolt-3 layers, 9 softmax anchors)
    "qwen3_4b_lm": dict(vocab_size=151936, dim=2560, num_layers=36, num_heads=32, num_kv_heads=8, head_dim=128,
                        intermediate=9728, hybrid_every=4, rope_theta=1e6, eps=1e-6, qk_norm=True,
                        tie_word_embeddings=True, max_T=4096),
}


def model_layer_types(mcfg: dict) -> list[str]:
    """Bolt-3 ("vsa") or softmax anchor per layer: every hybrid_every-th layer is an anchor
    (vsa_lm/config/inspector.py:55-58)."""
    he = int(mcfg["hybrid_every"])
    return ["softmax" if he > 0 and (li + 1) % he == 0 else "vsa" for li in range(int(mcfg["num_layers"]))]


def make_model_params(mcfg: dict, seed: int = 0) -> dict:
    """Seeded parameters of a whole hybrid model with the reference's state_dict keys
    (vsa_lm/config/standard.py:366-399): every Bolt-3 layer from make_params, anchors and MLPs
    uniform in +-1/sqrt(fan_in), norms near 1, embedding N(0, 1)."""
    g = torch.Generator().manual_seed(seed)
    D, V, I = int(mcfg["dim"]), int(mcfg["vocab_size"]), int(mcfg["intermediate"])
    H, HKV = int(mcfg["num_heads"]), int(mcfg["num_kv_heads"])
    HD = int(mcfg.get("head_dim") or D // H)

    def lin(n_out, n_in):
        return (torch.rand(n_out, n_in, generator=g) * 2 - 1) / math.sqrt(n_in)

    def norm(n):
        return 1.0 + 0.05 * torch.randn(n, generator=g)

    lcfg = dict(dim=D, num_heads=H, num_kv_heads=HKV, head_dim=HD, rope_theta=mcfg["rope_theta"],
                eps=mcfg["eps"], qk_norm=mcfg.get("qk_norm", False))
    p = {"embed_tokens.weight": torch.randn(V, D, generator=g)}
    for li, t in enumerate(model_layer_types(mcfg)):
        pre = f"blocks.{li}."
        p[pre + "norm1.weight"] = norm(D)
        if t == "vsa":
            for k, v in make_params(lcfg, seed * 1000 + li).items():
                p[pre + "vsa." + k] = v
        else:
            p[pre + "attn.q_proj.weight"] = lin(H * HD, D)
            p[pre + "attn.k_proj.weight"] = lin(HKV * HD, D)
            p[pre + "attn.v_proj.weight"] = lin(HKV * HD, D)
            p[pre + "attn.o_proj.weight"] = lin(D, H * HD)
            if mcfg.get("qk_norm", False):
                p[pre + "attn.q_norm.weight"] = norm(HD)
                p[pre + "attn.k_norm.weight"] = norm(HD)
        p[pre + "norm2.weight"] = norm(D)
        p[pre + "mlp.gate_proj.weight"] = lin(I, D)
        p[pre + "mlp.up_proj.weight"] = lin(I, D)
        p[pre + "mlp.down_proj.weight"] = lin(D, I)
    p["norm.weight"] = norm(D)
    p["lm_head.weight"] = p["embed_tokens.weight"] if mcfg.get("tie_word_embeddings", True) else lin(V, D)
    return p


@torch.no_grad()
def init_model_on_device(model: torch.nn.Module, seed: int = 0) -> None:
    """Seeded random weights for a whole hybrid model, drawn on the model's device (a model of
    billions of parameters would take minutes to build through make_model_params on the CPU). The
    laws are make_model_params's: linear weights uniform in +-1/sqrt(fan_in), the embedding N(0, 1),
    norms 1 + 0.05 N(0, 1), and the Bolt-3 layers' own parameters as in make_params (kappa, log_gamma,
    the beta / eta gates, res_norm)."""
    dev = next(model.parameters()).device
    g = torch.Generator(device=dev).manual_seed(seed)
    for name, p in model.named_parameters():
        leaf = name.rsplit(".", 1)[-1] if "." in name else name
        mod = name.rsplit(".", 2)[-2] if name.count(".") >= 1 else ""
        if name == "embed_tokens.weight":
            p.normal_(0.0, 1.0, generator=g)
        elif leaf == "kappa":
            p.normal_(0.0, 0.1, generator=g).add_(1.0)
        elif leaf == "log_gamma":
            p.normal_(0.0, 0.5, generator=g).add_(3.5)
        elif mod in ("beta_proj", "eta_proj"):
            if leaf == "weight":
                p.normal_(0.0, 0.02, generator=g)
            else:
                p.fill_(-1.0 if mod == "beta_proj" else 0.0)
        elif mod == "res_norm":
            p.fill_(0.05)
        elif p.dim() == 1:   # norm weights
            p.normal_(0.0, 0.05, generator=g).add_(1.0)
        elif p.dim() == 2:   # linear weights [out, in]
            bound = 1.0 / math.sqrt(p.shape[1])
            p.uniform_(-bound, bound, generator=g)
        else:
            raise ValueError(f"no initialisation law for {name} {tuple(p.shape)}")
