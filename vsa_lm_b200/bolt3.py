"""Drop-in `Bolt3Attn` / `Bolt3Decoder` backed by the sm_100a kernels of libbolt3.so.

Same constructor signatures, attributes, parameter names (state_dict keys), methods and decoder
state lists as the reference `vsa_lm/config/bolt3.py`, so a model built by the reference's
converter loads unchanged (`load_state_dict` of `blocks.{i}.vsa.*`). The attention math runs only
in CUDA kernels; calling it on CPU tensors raises instead of falling back.

Precision contract (the reference's CUDA behaviour under bf16 autocast, bolt3.py:339): activations
are stored in bf16, every product and sum is accumulated in fp32, the attractor statistics and
M_res are fp32. Results are compared with the fp32 CPU oracle restating the reference
(tests/, oracle/).
"""
from __future__ import annotations

import math

import types

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import kernels as K

N_SINKS = 4


# --------------------------------------------------------------------------------------------
# helper modules with the reference's parameter layout (vsa_lm/surgery.py:43-93)

class LlamaRMSNorm(nn.Module):
    """RMSNorm with an fp32 interior (surgery.py:43-53)."""

    def __init__(self, dim: int, eps: float = 1e-5):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        dt = x.dtype
        xf = x.float()
        xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)
        return (xf * self.weight.float()).to(dt)


def llama_inv_freq(head_dim: int, theta: float, rope_scaling: dict | None, device=None) -> torch.Tensor:
    """RoPE inverse frequencies with optional llama3 scaling (surgery.py:56-72)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64, device=device).float() / head_dim))
    if rope_scaling and rope_scaling.get("rope_type") == "llama3":
        old_ctx = float(rope_scaling["original_max_position_embeddings"])
        factor = float(rope_scaling["factor"])
        low, high = float(rope_scaling["low_freq_factor"]), float(rope_scaling["high_freq_factor"])
        wavelen = 2.0 * math.pi / inv
        inv_a = torch.where(wavelen > old_ctx / low, inv / factor, inv)
        smooth = (old_ctx / wavelen - low) / (high - low)
        smoothed = (1.0 - smooth) * inv_a / factor + smooth * inv_a
        medium = ~(wavelen < old_ctx / high) & ~(wavelen > old_ctx / low)
        inv = torch.where(medium, smoothed, inv_a)
    return inv


class LlamaRoPE(nn.Module):
    """Rotate-half RoPE with a non-persistent inv_freq buffer (surgery.py:80-93)."""

    def __init__(self, head_dim: int, theta: float, rope_scaling: dict | None):
        super().__init__()
        self.register_buffer("inv_freq", llama_inv_freq(head_dim, theta, rope_scaling, torch.device("cpu")),
                             persistent=False)

    def forward(self, x: torch.Tensor, pos_start: int = 0) -> torch.Tensor:
        T = x.shape[2]
        t = torch.arange(pos_start, pos_start + T, device=x.device, dtype=torch.float32)
        freqs = t[:, None] * self.inv_freq.to(x.device)
        emb = torch.cat((freqs, freqs), dim=-1)
        cos, sin = emb.cos().to(x.dtype)[None, None], emb.sin().to(x.dtype)[None, None]
        h = x.shape[-1] // 2
        return x * cos + torch.cat((-x[..., h:], x[..., :h]), dim=-1) * sin


# --------------------------------------------------------------------------------------------

class _NativeForward(torch.autograd.Function):
    """Forward-only autograd node: the Bolt-3 backward is not implemented natively."""

    @staticmethod
    def forward(ctx, x, mod, *params):
        return mod._native_forward(x)

    @staticmethod
    def backward(ctx, *grads):
        raise NotImplementedError("Bolt3Attn (B200 native) implements the forward pass only; "
                                  "training needs the reference module")


class _Fused:
    """bf16 copies of the projection weights, rebuilt when a parameter changes."""

    def __init__(self):
        self.key = None
        self.w_in = self.b_in = self.w_out = None
        self.consts = None


class Bolt3Attn(nn.Module):
    """Bolt-3 dual-field attention (reference: vsa_lm/config/bolt3.py:23-276)."""

    def __init__(self, cfg: dict, max_T: int = 2048, S: int = 128, C: int = 128):
        super().__init__()
        D, H, HKV = int(cfg["dim"]), int(cfg["num_heads"]), int(cfg["num_kv_heads"])
        HD = int(cfg.get("head_dim") or (D // H))
        qkv_bias = bool(cfg.get("qkv_bias", False))
        if S != K.S_SLOTS or C != K.CHUNK:
            raise NotImplementedError(f"native Bolt-3 kernels support S = C = 128 (got S={S}, C={C})")
        if HD not in (64, 128) or H % HKV or H // HKV > 16:
            raise NotImplementedError(f"native Bolt-3 kernels support head_dim 64/128 and G <= 16 (HD={HD})")
        self.H, self.HKV, self.HD, self.G = H, HKV, HD, H // HKV
        self.S, self.C, self.n_sinks = S, C, N_SINKS
        self.sim_k, self.sim_v, self.gamma_u = 0.88, 0.80, 0.995
        self.eps = float(cfg["eps"])

        self.q_proj = nn.Linear(D, H * HD, bias=qkv_bias)
        self.k_proj = nn.Linear(D, HKV * HD, bias=qkv_bias)
        self.v_proj = nn.Linear(D, HKV * HD, bias=qkv_bias)
        self.o_proj = nn.Linear(H * HD, D, bias=False)
        if cfg.get("qk_norm", False):
            self.q_norm = LlamaRMSNorm(HD, cfg["eps"])
            self.k_norm = LlamaRMSNorm(HD, cfg["eps"])
        else:
            self.q_norm, self.k_norm = None, None
        self.rope = LlamaRoPE(HD, cfg["rope_theta"], cfg.get("rope_scaling"))

        self.kappa = nn.Parameter(torch.ones(HKV))
        self.log_gamma = nn.Parameter(torch.full((HKV,), 3.5))
        self.beta_proj = nn.Linear(D, HKV, bias=True)
        nn.init.zeros_(self.beta_proj.weight)
        nn.init.constant_(self.beta_proj.bias, -1.0)
        self.eta_proj = nn.Linear(D, H, bias=True)
        nn.init.zeros_(self.eta_proj.weight)
        nn.init.zeros_(self.eta_proj.bias)
        self.res_norm = LlamaRMSNorm(HD, cfg["eps"])
        with torch.no_grad():
            self.res_norm.weight.fill_(0.05)
        self._fused = _Fused()

    # ---- reference API (bolt3.py:56-66)
    def gamma_delta(self) -> torch.Tensor:
        return (0.999 * torch.sigmoid(self.log_gamma)).clamp(1e-3, 0.999).float()

    def head_qkv(self, x: torch.Tensor):
        b, t, _ = x.shape
        q = self.q_proj(x).view(b, t, self.H, self.HD)
        k = self.k_proj(x).view(b, t, self.HKV, self.HD)
        v = self.v_proj(x).view(b, t, self.HKV, self.HD)
        if self.q_norm is not None:
            q, k = self.q_norm(q), self.k_norm(k)
        return q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)

    # ---- fused weights and per-head constants, cached on the device
    def _params_key(self, device):
        ps = [self.q_proj.weight, self.k_proj.weight, self.v_proj.weight, self.o_proj.weight,
              self.beta_proj.weight, self.beta_proj.bias, self.eta_proj.weight, self.eta_proj.bias,
              self.kappa, self.log_gamma, self.res_norm.weight]
        for opt in (self.q_proj.bias, self.k_proj.bias, self.v_proj.bias,
                    getattr(self.q_norm, "weight", None), getattr(self.k_norm, "weight", None)):
            if opt is not None:
                ps.append(opt)
        return (str(device),) + tuple((p.data_ptr(), p._version) for p in ps)

    def fused(self, device):
        """(W_in [N, D] bf16, b_in [N] bf16 or None, W_out bf16, consts) for `device`, where the
        fused input projection has columns [q | k | v | beta | eta] (the bolt3_prep layout)."""
        device = torch.device(device)
        if device.type == "cuda" and device.index is None:   # "cuda" and "cuda:<current>" share one entry
            device = torch.device("cuda", torch.cuda.current_device())
        key = self._params_key(device)
        f = self._fused
        if f.key == key:
            return f
        with torch.no_grad():
            bf = dict(dtype=torch.bfloat16, device=device)
            ws = [self.q_proj.weight, self.k_proj.weight, self.v_proj.weight, self.beta_proj.weight,
                  self.eta_proj.weight]
            # One fused input projection with row blocks [k | v | beta | pad | q | eta | pad]: the first
            # n_kv rows (the k/v/beta GEMM the consolidation scan waits on) and the rest (q/eta) are
            # also usable as two separate GEMMs. Blocks start on multiples of 8 rows, so every
            # section of a projection row is 16-byte aligned.
            H, HKV, HD = self.H, self.HKV, self.HD
            r8 = lambda n: (n + 7) // 8 * 8
            n_kv = r8(2 * HKV * HD + HKV)
            n_all = n_kv + r8(H * HD + H)
            bias = lambda b, n: b.detach().to(**bf) if b is not None else torch.zeros(n, **bf)
            blocks_w = [self.k_proj.weight, self.v_proj.weight, self.beta_proj.weight]
            blocks_b = [bias(self.k_proj.bias, HKV * HD), bias(self.v_proj.bias, HKV * HD), bias(self.beta_proj.bias, HKV)]
            D = self.q_proj.weight.shape[1]
            w = torch.zeros(n_all, D, **bf)
            bvec = torch.zeros(n_all, **bf)
            r = 0
            for wt, bt in zip(blocks_w, blocks_b):
                w[r:r + wt.shape[0]] = wt.detach().to(**bf)
                bvec[r:r + wt.shape[0]] = bt
                r += wt.shape[0]
            w[n_kv:n_kv + H * HD] = self.q_proj.weight.detach().to(**bf)
            bvec[n_kv:n_kv + H * HD] = bias(self.q_proj.bias, H * HD)
            w[n_kv + H * HD:n_kv + H * HD + H] = self.eta_proj.weight.detach().to(**bf)
            bvec[n_kv + H * HD:n_kv + H * HD + H] = bias(self.eta_proj.bias, H)
            f.w_in, f.b_in = w, bvec
            f.n_kv = n_kv
            f.cols = dict(k_col=0, v_col=HKV * HD, beta_col=2 * HKV * HD, q_col=n_kv, eta_col=n_kv + H * HD)
            f.cols_kv = dict(k_col=0, v_col=HKV * HD, beta_col=2 * HKV * HD)
            f.cols_q = dict(q_col=0, eta_col=H * HD)
            f.w_out = self.o_proj.weight.detach().to(**bf).contiguous()
            gam = self.gamma_delta().detach()
            f.consts = dict(
                gamma=gam.to(device).contiguous(),
                coef=((1.0 - gam) / (self.HD ** 0.5)).float().to(device).contiguous(),
                kappa=self.kappa.detach().float().to(device).contiguous(),
                res_w=self.res_norm.weight.detach().float().to(device).contiguous(),
                inv_freq=self.rope.inv_freq.float().to(device).contiguous(),
                qn=None if self.q_norm is None else self.q_norm.weight.detach().float().to(device).contiguous(),
                kn=None if self.k_norm is None else self.k_norm.weight.detach().float().to(device).contiguous(),
            )
        f.key = key
        return f

    def project(self, x2d: torch.Tensor, f, part: str = "all") -> torch.Tensor:
        """Input projection GEMM (cuBLAS via torch): [n_tok, D] -> [n_tok, N] bf16. part = "all"
        (columns per f.cols), "kv" (f.cols_kv) or "q" (f.cols_q)."""
        if part == "kv":
            return F.linear(x2d, f.w_in[:f.n_kv], f.b_in[:f.n_kv])
        if part == "q":
            return F.linear(x2d, f.w_in[f.n_kv:], f.b_in[f.n_kv:])
        return F.linear(x2d, f.w_in, f.b_in)

    # ---- forward (bolt3.py:194-276)
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if torch.is_grad_enabled() and (x.requires_grad or any(p.requires_grad for p in self.parameters())):
            return _NativeForward.apply(x, self, *[p for p in self.parameters() if p.requires_grad])
        return self._native_forward(x)

    @torch.no_grad()
    def _native_forward(self, x: torch.Tensor, partial_fp32: bool = False) -> torch.Tensor:
        """The forward on CUDA. partial_fp32: return o_proj's output in fp32, unrounded (a tensor-
        parallel shard's partial sum, rounded once after the all-reduce)."""
        if not x.is_cuda:
            raise RuntimeError("Bolt3Attn (B200 native) runs on CUDA tensors only; no CPU path exists")
        b, T, D = x.shape
        H, HKV, HD = self.H, self.HKV, self.HD
        dev = x.device
        f = self.fused(dev)
        c = f.consts
        x2 = x.reshape(b * T, D).to(torch.bfloat16)
        bf = dict(dtype=torch.bfloat16, device=dev)
        q_raw = torch.empty(b * H, T, HD, **bf)
        q_rope = torch.empty_like(q_raw)
        k_raw = torch.empty(b * HKV, T, HD, **bf)
        k_rope = torch.empty_like(k_raw)
        v = torch.empty_like(k_raw)
        beta = torch.empty(b * HKV, T, dtype=torch.float32, device=dev)
        eta = torch.empty(b * H, T, dtype=torch.float32, device=dev)
        q_l2 = torch.empty(b * H, T, dtype=torch.float32, device=dev)
        common = dict(B=b, T=T, H=H, HKV=HKV, HD=HD, inv_freq=c["inv_freq"], eps=self.eps, q_norm_w=c["qn"],
                      k_norm_w=c["kn"], pos0=0)
        # k/v/beta first: the consolidation scan waits only on them
        K.prep(self.project(x2, f, "kv"), cols=f.cols_kv, parts=2, k_raw=k_raw, k_rope=k_rope, v=v, beta=beta,
               k_head_stride=T, k_t_off=0, **common)
        ws = torch.empty(max(1, K.prefill_workspace_bytes(b * HKV, T, HD)), dtype=torch.uint8, device=dev)
        bank = K.new_bank(b * HKV, HD, dev)
        y = torch.empty(b, T, H, HD, **bf)

        def prep_q():
            K.prep(self.project(x2, f, "q"), cols=f.cols_q, parts=1, q_raw=q_raw, q_rope=q_rope, eta=eta,
                   q_head_stride=T, q_t_off=0, q_l2=q_l2, **common)

        self._scan_and_attend(b, T, q_rope=q_rope, q_raw=q_raw, eta=eta, k_raw=k_raw, k_rope=k_rope, v=v,
                              beta=beta, q_l2=q_l2, ws=ws, bank=bank, y=y, consts=c, before_attend=prep_q)
        if partial_fp32:
            return torch.mm(y.view(b * T, H * HD), f.w_out.t(), out_dtype=torch.float32).view(b, T, -1)
        out = F.linear(y.view(b, T, H * HD), f.w_out)
        return out.to(x.dtype)

    # scan steps per segment when the consolidation scan overlaps the attention
    # Scan segment lengths, front-loaded: the attention of bank-reading chunks cannot start before the
    # q projection is done anyway, while every relaunch costs a bank reload and the slowest chain.
    SCAN_SEGMENTS = (32, 12, 8, 6, 4)
    # Past the table (long sequences) the segments double up to this length: each relaunch costs a
    # bank reload and a launch gap, while a long segment only delays the attention of its own chunks.
    SCAN_SEGMENT_MAX = 64

    def _scan_segments(self, n_cons: int):
        """(first step, steps) of each scan launch: the table, then doubling lengths up to
        SCAN_SEGMENT_MAX."""
        out, s0, i = [], 0, 0
        nt = len(self.SCAN_SEGMENTS)
        while s0 < n_cons:
            n = self.SCAN_SEGMENTS[i] if i < nt else min(self.SCAN_SEGMENT_MAX, self.SCAN_SEGMENTS[-1] << (i - nt + 1))
            n = min(n, n_cons - s0)
            out.append((s0, n))
            s0 += n
            i += 1
        return out

    def _aux_stream(self, device) -> torch.cuda.Stream:
        cache = self.__dict__.setdefault("_streams", {})
        key = str(device)
        if key not in cache:
            # highest priority: each scan segment is on the critical path, and the block scheduler
            # then hands it SMs as soon as attention CTAs retire instead of after the whole grid
            cache[key] = torch.cuda.Stream(device=device, priority=-8)
        return cache[key]

    def _scan_and_attend(self, b, T, *, q_rope, q_raw, eta, k_raw, k_rope, v, beta, q_l2, ws, bank, y, consts,
                         before_attend=None):
        """Phases B and C of the forward (bolt3.py:210-273), overlapped on two streams.

        The consolidation scan is sequential per chain and fills only b*HKV SMs, so it runs on a
        side stream in segments (SCAN_SEGMENTS) while the main stream runs the attention of
        every chunk whose snapshot (consolidation r - 2) is already written."""
        H, HKV, HD, G = self.H, self.HKV, self.HD, self.G
        c = consts
        n_chunks = (T + self.C - 1) // self.C
        n_cons = K.n_consolidations(T)
        att = dict(n_chains=b * HKV, hkv=HKV, G=G, HD=HD, T=T, q_rope=q_rope, q_raw=q_raw, eta=eta,
                   k_rope=k_rope, v=v, n_cons=n_cons, kappa=c["kappa"], coef=c["coef"], res_w=c["res_w"],
                   eps=self.eps, y=y, q_l2=q_l2)
        if n_cons == 0:
            if before_attend is not None:
                before_attend()
            K.attend_prefill(snaps=None, **att)
            return
        snaps = K.snapshot_views(ws, b * HKV, n_cons, HD)
        main = torch.cuda.current_stream(q_rope.device)
        aux = self._aux_stream(q_rope.device)
        ready = torch.cuda.Event()
        ready.record(main)
        aux.wait_event(ready)
        done = []
        with torch.cuda.stream(aux):
            for s0, n in self._scan_segments(n_cons):
                K.consolidate(n_chains=b * HKV, hkv=HKV, HD=HD, bank=bank, init_blank=s0 == 0, kr=k_raw, kp=k_rope,
                              v=v, beta=beta, chain_tokens=T, token0=s0 * self.C, step_tokens=self.C,
                              skip0=N_SINKS if s0 == 0 else 0, chunk_len=self.C, pos0=0, n_steps=n,
                              kappa=c["kappa"], gamma=c["gamma"], inv_freq=c["inv_freq"], snaps=snaps, snap0=s0)
                ev = torch.cuda.Event()
                ev.record(aux)
                done.append((s0 + n, ev))
        if before_attend is not None:   # the q projection runs while the scan starts
            before_attend()
        # chunks 0 and 1 read no bank
        K.attend_prefill(snaps=snaps, blk_begin=0, blk_count=min(2, n_chunks), **att)
        blk = 2
        for end, ev in done:
            main.wait_event(ev)
            last = n_chunks if end == n_cons else end + 2
            if last > blk:
                K.attend_prefill(snaps=snaps, blk_begin=blk, blk_count=last - blk, **att)
                blk = last

    # ---- one consolidation on reference-format tensors (bolt3.py:68-192), natively
    @torch.no_grad()
    def _consolidate_functional(self, ak, av, mass, util, pm, act, m_res, k_raw, k_rope, v_old, pos_old,
                                beta_old, inv_freq, diag_eye, gam, n_filled: int = 0):
        b, hkv, l_tok, hd = k_raw.shape
        bh = b * hkv
        dev = k_raw.device
        if not k_raw.is_cuda:
            raise RuntimeError("native _consolidate_functional needs CUDA tensors")
        if l_tok > self.C:
            raise NotImplementedError(f"native consolidation handles chunks of <= {self.C} tokens (got {l_tok})")
        f = self.fused(dev)
        dt = k_raw.dtype
        bank = K.new_bank(bh, hd, dev)
        blank = ak is None
        if not blank:
            bank["ak"].copy_(ak.reshape(bh, self.S, hd))
            bank["av"].copy_(av.reshape(bh, self.S, hd))
            bank["mass"].copy_(mass.reshape(bh, self.S))
            bank["util"].copy_(util.reshape(bh, self.S))
            bank["pm"].copy_(pm.reshape(bh, self.S))
            bank["act"].copy_(act.reshape(bh, self.S))
            bank["m_res"].copy_(m_res.reshape(bh, hd, hd))
            bank["n_filled"].fill_(int(n_filled))
        kr = k_raw.reshape(bh, l_tok, hd).to(torch.bfloat16).contiguous()
        kp = k_rope.reshape(bh, l_tok, hd).to(torch.bfloat16).contiguous()
        vv = v_old.reshape(bh, l_tok, hd).to(torch.bfloat16).contiguous()
        bb = beta_old.reshape(bh, l_tok).float().contiguous()
        pos0 = int(pos_old.reshape(-1)[0].item())
        K.consolidate(n_chains=bh, hkv=hkv, HD=hd, bank=bank, init_blank=blank, kr=kr, kp=kp, v=vv, beta=bb,
                      chain_tokens=l_tok, token0=0, step_tokens=l_tok, skip0=0, chunk_len=l_tok, pos0=pos0,
                      n_steps=1, kappa=f.consts["kappa"], gamma=gam.float().contiguous(),
                      inv_freq=f.consts["inv_freq"])
        nf = 0 if blank else int(n_filled)
        nf = nf if nf >= self.S else nf + min(self.S - nf, l_tok)
        return (bank["ak"].to(dt), bank["av"].to(dt), bank["mass"], bank["util"], bank["pm"],
                bank["act"].bool(), bank["m_res"], nf)


# --------------------------------------------------------------------------------------------
# decoder

class Bolt3LayerState:
    """Device-resident decode state of one Bolt-3 layer for B sequences.

    The local window is a two-slot ring of chunk buffers ([chains][2][C][HD]); the reference keeps
    python lists and re-concatenates them every token (bolt3.py:355-363). `m_res` is the tensor the
    caller holds in states[li] ([B, HKV, HD, HD] fp32), updated in place.
    """

    def __init__(self, ly: Bolt3Attn, B: int, device):
        self.B, self.HKV, self.HD, self.C = B, ly.HKV, ly.HD, ly.C
        n = B * ly.HKV
        bf = dict(dtype=torch.bfloat16, device=device)
        self.ring_kr = torch.empty(n, 2 * self.C, self.HD, **bf)
        self.ring_kp = torch.empty_like(self.ring_kr)
        self.ring_v = torch.empty_like(self.ring_kr)
        self.ring_b = torch.empty(n, 2 * self.C, dtype=torch.float32, device=device)
        self.sink_k = torch.empty(n, N_SINKS, self.HD, **bf)
        self.sink_v = torch.empty_like(self.sink_k)
        self.bank = K.new_bank(n, self.HD, device)
        self.slot_pos = [0, 0]
        self.cur_slot, self.cur_len = 0, 0
        self.prev_slot = -1
        self.sinks_set = False
        self.n_filled = 0
        self._plans = {}   # per step size: buffers and prebuilt launch arguments (Bolt3Decoder)

    @property
    def has_bank(self) -> bool:
        return self.n_filled > 0


class Bolt3Decoder:
    """Constant-memory decoder (reference: vsa_lm/config/bolt3.py:279-557) with native Bolt-3 layers.

    Softmax anchor layers use a static KV cache and SDPA as in the reference (bolt3.py:426-445).
    """

    def __init__(self, model, wrap_positions: bool = False, max_cache_pos: int = 65536, **kwargs):
        self.model = model.eval()
        self.max_T = model.config["max_T"]
        self.max_cache_pos = max_cache_pos
        self.C = int(model.config.get("bolt3_C", 128))

    @staticmethod
    def state_bytes(model):
        flat, per_tok = 0, 0
        for blk in model.blocks:
            if hasattr(blk, "vsa"):
                ly = blk.vsa
                flat += ly.HKV * ly.HD * ly.HD * 4 + 2 * ly.S * ly.HKV * ly.HD * 2 + 4 * ly.C * ly.HKV * ly.HD * 2
            else:
                s = blk.attn
                per_tok += 2 * s.HKV * s.HD * 2
        return flat, per_tok

    @staticmethod
    def blank_state(model, batch_size: int, device, max_kv_len: int = 4096, state_dtype=torch.float32, **kwargs):
        states, kv_caches = [None] * len(model.blocks), [None] * len(model.blocks)
        for li, blk in enumerate(model.blocks):
            if hasattr(blk, "vsa"):
                ly = blk.vsa
                states[li] = torch.zeros(batch_size, ly.HKV, ly.HD, ly.HD, device=device, dtype=torch.float32)
                kv_caches[li] = Bolt3LayerState(ly, batch_size, device)
            else:
                s = blk.attn
                kv_caches[li] = StaticKV(batch_size, s.HKV, max_kv_len, s.HD, device, dt=torch.bfloat16)
        return states, kv_caches

    # ---- decode state in the reference's format (bolt3.py:302-319 creates it, :343-425 fills it):
    # per Bolt-3 layer a dict with the bank (ak/av [b*HKV, S, HD], mass/util/pm fp32 [b*HKV, S], act
    # bool, n_filled), the sinks [b, HKV, 4, HD], and the previous / current chunk windows
    # {prev,cur}_{kr,kp,v} [b, HKV, len, HD], _pos [1, 1, len] fp32, _b [b, HKV, len]; states[li] is
    # M_res [b, HKV, HD, HD] fp32 in both formats.
    _REF_KEYS = ("ak", "av", "mass", "util", "pm", "act", "sink_k", "sink_v", "prev_kr", "prev_kp", "prev_v",
                 "prev_pos", "prev_b", "cur_kr", "cur_kp", "cur_v", "cur_pos", "cur_b")

    @staticmethod
    def state_to_reference(model, states, kv_caches):
        """(states, kv_caches) with every Bolt3LayerState replaced by the reference's dict (copies)."""
        out = []
        for li, blk in enumerate(model.blocks):
            st = kv_caches[li]
            out.append(Bolt3Decoder._layer_to_dict(st) if hasattr(blk, "vsa") else st)
        return states, out

    @staticmethod
    def state_from_reference(model, states, kv_caches, device):
        """Native (states, kv_caches) from the reference's format; states[li] tensors are moved to
        `device` as fp32 and then updated in place by the native steps."""
        out_states, out_caches = list(states), []
        for li, blk in enumerate(model.blocks):
            d = kv_caches[li]
            if hasattr(blk, "vsa"):
                out_states[li] = states[li].to(device=device, dtype=torch.float32).contiguous()
                out_caches.append(Bolt3Decoder._layer_from_dict(blk.vsa, d, out_states[li].shape[0], device))
            else:
                out_caches.append(d)
        return out_states, out_caches

    @staticmethod
    def _layer_to_dict(st: "Bolt3LayerState") -> dict:
        B, HKV, HD, C = st.B, st.HKV, st.HD, st.C
        d = {k: None for k in Bolt3Decoder._REF_KEYS}
        if st.has_bank:
            bank = st.bank
            for k in ("ak", "av", "mass", "util", "pm"):
                d[k] = bank[k].clone()
            d["act"] = bank["act"].bool()
            d["n_filled"] = int(st.n_filled)
        if st.sinks_set:
            d["sink_k"] = st.sink_k.view(B, HKV, N_SINKS, HD).clone()
            d["sink_v"] = st.sink_v.view(B, HKV, N_SINKS, HD).clone()

        def window(tag, slot, n):
            s0 = slot * C
            d[tag + "_kr"] = st.ring_kr[:, s0:s0 + n].reshape(B, HKV, n, HD).clone()
            d[tag + "_kp"] = st.ring_kp[:, s0:s0 + n].reshape(B, HKV, n, HD).clone()
            d[tag + "_v"] = st.ring_v[:, s0:s0 + n].reshape(B, HKV, n, HD).clone()
            d[tag + "_b"] = st.ring_b[:, s0:s0 + n].reshape(B, HKV, n).to(torch.bfloat16)
            p0 = st.slot_pos[slot]
            d[tag + "_pos"] = torch.arange(p0, p0 + n, dtype=torch.float32, device=st.ring_kr.device).view(1, 1, n)

        if st.prev_slot >= 0:
            window("prev", st.prev_slot, C)
        if st.cur_len > 0:
            window("cur", st.cur_slot, st.cur_len)
        return d

    @staticmethod
    def _layer_from_dict(ly: Bolt3Attn, d: dict, B: int, device) -> "Bolt3LayerState":
        st = Bolt3LayerState(ly, B, device)
        HKV, HD, C, S = ly.HKV, ly.HD, ly.C, ly.S
        n = B * HKV
        dev = dict(device=device)
        if d.get("ak") is not None:
            bank = st.bank
            bank["ak"].copy_(d["ak"].reshape(n, S, HD))
            bank["av"].copy_(d["av"].reshape(n, S, HD))
            for k in ("mass", "util", "pm"):
                bank[k].copy_(d[k].reshape(n, S))
            bank["act"].copy_(d["act"].reshape(n, S).to(torch.uint8))
            # RoPE of the attractor keys at their mean positions in the storage dtype (bolt3.py:15-18):
            # x * bf16(cos) + rotate_half(x) * bf16(sin), each product and the sum rounded to bf16
            ak = bank["ak"]
            ang = bank["pm"].unsqueeze(-1) * ly.fused(device).consts["inv_freq"].view(1, 1, -1)
            ang = torch.cat((ang, ang), dim=-1)
            h = HD // 2
            rot = torch.cat((-ak[..., h:], ak[..., :h]), dim=-1)
            bank["ak_rope"].copy_(ak * ang.cos().to(torch.bfloat16) + rot * ang.sin().to(torch.bfloat16))
            st.n_filled = int(d.get("n_filled", 0))
            bank["n_filled"].fill_(st.n_filled)
        if d.get("sink_k") is not None:
            if d["sink_k"].shape[2] != N_SINKS:
                raise NotImplementedError("native decoder state holds exactly 4 sinks")
            st.sink_k.copy_(d["sink_k"].reshape(n, N_SINKS, HD))
            st.sink_v.copy_(d["sink_v"].reshape(n, N_SINKS, HD))
            st.sinks_set = True

        def fill(tag, slot):
            L = d[tag + "_kp"].shape[2]
            s0 = slot * C
            st.ring_kr[:, s0:s0 + L].copy_(d[tag + "_kr"].reshape(n, L, HD))
            st.ring_kp[:, s0:s0 + L].copy_(d[tag + "_kp"].reshape(n, L, HD))
            st.ring_v[:, s0:s0 + L].copy_(d[tag + "_v"].reshape(n, L, HD))
            st.ring_b[:, s0:s0 + L].copy_(d[tag + "_b"].reshape(n, L).float())
            st.slot_pos[slot] = int(d[tag + "_pos"].reshape(-1)[0].item())
            return L

        if d.get("prev_kp") is not None:
            if fill("prev", 0) != C:
                raise NotImplementedError("native decoder state holds a previous chunk of exactly C tokens")
            st.prev_slot, st.cur_slot = 0, 1
        if d.get("cur_kp") is not None:
            st.cur_len = fill("cur", st.cur_slot)
            if st.cur_len >= C:
                raise NotImplementedError("a pending chunk of C tokens is consolidated by the step that fills it")
        return st

    @staticmethod
    def _sample(logits, temperature: float, top_k: int = 40, top_p: float = 0.95):
        if temperature <= 1e-5:
            return logits.argmax(-1, keepdim=True)
        probs = F.softmax(logits.float() / temperature, dim=-1)
        if top_p < 1.0:
            sp, si = torch.sort(probs, descending=True, dim=-1)
            cp = torch.cumsum(sp, dim=-1)
            sp[cp - sp > top_p] = 0.0
            sp.div_(sp.sum(dim=-1, keepdim=True).clamp_min(1e-12))
            return si.gather(-1, torch.multinomial(sp, 1))
        tv, ti = torch.topk(logits.float() / temperature, min(top_k, logits.size(-1)), dim=-1)
        return ti.gather(-1, torch.multinomial(F.softmax(tv, -1), 1))

    # ---- one Bolt-3 layer (bolt3.py:343-425)
    PLAN_MAX_TOKENS = 16   # steps of up to this many tokens keep their buffers and arguments

    @staticmethod
    def _step_plan(ly: Bolt3Attn, st: Bolt3LayerState, b: int, t: int, f, dev):
        """Buffers and prebuilt bolt3_prep / bolt3_attend arguments of a t-token step."""
        H, HKV, HD, C, G = ly.H, ly.HKV, ly.HD, ly.C, ly.G
        c = f.consts
        bf = dict(dtype=torch.bfloat16, device=dev)
        # the plan keeps its own references to the tensors its launch arguments point at: fused()
        # replaces them when the weights change, and the plan is then rebuilt at the next chunk start
        plan = types.SimpleNamespace(f=f, key=f.key, w_in=f.w_in, b_in=f.b_in, w_out=f.w_out, consts=c, cols=f.cols)
        plan.q_raw = torch.empty(b * H, t, HD, **bf)
        plan.q_rope = torch.empty_like(plan.q_raw)
        plan.eta = torch.empty(b * H, t, dtype=torch.float32, device=dev)
        plan.q_l2 = torch.empty(b * H, t, dtype=torch.float32, device=dev)
        plan.y = torch.empty(b, t, H, HD, **bf)
        plan.ring_kp, plan.ring_v = st.ring_kp.data_ptr(), st.ring_v.data_ptr()
        plan.ring_row = HD * st.ring_kp.element_size()
        cols = f.cols
        ptr = lambda x: None if x is None else x.data_ptr()
        prep = dict(
            proj=None, ld=f.w_in.shape[0], B=b, T=t, H=H, HKV=HKV, HD=HD,
            q_norm_w=ptr(c["qn"]), k_norm_w=ptr(c["kn"]), eps=ly.eps, inv_freq=c["inv_freq"].data_ptr(), pos0=0,
            q_raw=plan.q_raw.data_ptr(), q_rope=plan.q_rope.data_ptr(), q_head_stride=t, q_t_off=0,
            eta=plan.eta.data_ptr(), eta_head_stride=t, eta_t_off=0, k_raw=st.ring_kr.data_ptr(),
            k_rope=st.ring_kp.data_ptr(), v=st.ring_v.data_ptr(), k_head_stride=2 * C, k_t_off=0,
            beta=st.ring_b.data_ptr(), beta_head_stride=2 * C, beta_t_off=0, q_l2=plan.q_l2.data_ptr(), parts=3,
            q_col=cols["q_col"], k_col=cols["k_col"], v_col=cols["v_col"], beta_col=cols["beta_col"],
            eta_col=cols["eta_col"])
        bk = st.bank
        attend = dict(
            n_chains=b * HKV, hkv=HKV, G=G, HD=HD, q_rope=plan.q_rope.data_ptr(), q_raw=plan.q_raw.data_ptr(),
            eta=plan.eta.data_ptr(), Tq=t, prefill=0, seg0_chain_tokens=2 * C, seg1_chain_tokens=2 * C,
            sink_k=st.sink_k.data_ptr(), sink_v=st.sink_v.data_ptr(), sink_chain_tokens=N_SINKS,
            bank_ak_rope=bk["ak_rope"].data_ptr(), bank_av=bk["av"].data_ptr(), bank_mass=bk["mass"].data_ptr(),
            bank_act=bk["act"].data_ptr(), bank_cap=1, kappa=c["kappa"].data_ptr(), coef=c["coef"].data_ptr(),
            res_w=c["res_w"].data_ptr(), eps=ly.eps, y=plan.y.data_ptr(), y_tokens=t, q_l2=plan.q_l2.data_ptr())
        plan.args = K.DecodeStepArgs(prep, attend)
        return plan

    @staticmethod
    def layer_step(ly: Bolt3Attn, st: Bolt3LayerState, h: torch.Tensor, pos_start: int,
                   m_res: torch.Tensor, partial_fp32: bool = False) -> torch.Tensor:
        """Attention branch of one Bolt-3 layer for t new tokens: returns o_proj(y) [b, t, D] bf16
        (fp32 and unrounded with partial_fp32: a tensor-parallel shard's partial sum)."""
        b, t, D = h.shape
        H, HKV, HD, C, G = ly.H, ly.HKV, ly.HD, ly.C, ly.G
        if st.cur_len + t > C:
            raise NotImplementedError(
                f"a step of {t} tokens on top of {st.cur_len} pending ones exceeds one chunk ({C}); "
                "the native decoder keeps at most one chunk pending")
        if st.cur_len == 0:
            st.slot_pos[st.cur_slot] = pos_start
        elif pos_start != st.slot_pos[st.cur_slot] + st.cur_len:
            raise NotImplementedError("native decoder needs contiguous positions within a chunk")
        if not (m_res.is_cuda and m_res.dtype == torch.float32 and m_res.is_contiguous()):
            raise ValueError("m_res must be a contiguous fp32 CUDA tensor [B, HKV, HD, HD]")
        dev = h.device
        # the step's buffers and launch arguments, rebuilt when the layer's weights change (checked
        # whenever a chunk starts) or the step size does
        plan = st._plans.get(t)
        if plan is None or st.cur_len == 0:
            f = ly.fused(dev)
            if plan is None or plan.key != f.key:
                plan = Bolt3Decoder._step_plan(ly, st, b, t, f, dev)
                # only decode-sized steps keep their plan: a prompt chunk's buffers are large and
                # the per-call set-up is small next to its work
                if t <= Bolt3Decoder.PLAN_MAX_TOKENS:
                    st._plans[t] = plan
        proj = F.linear(h.reshape(b * t, D).to(torch.bfloat16), plan.w_in, plan.b_in)
        plan.args.launch_prep(proj, pos_start, st.cur_slot * C + st.cur_len)
        has_prev = st.prev_slot >= 0
        p0 = st.prev_slot * C if has_prev else 0
        c0 = st.cur_slot * C
        rk, rv, row = plan.ring_kp, plan.ring_v, plan.ring_row
        plan.args.launch_attend(
            seg0_k=rk + p0 * row, seg0_v=rv + p0 * row, seg0_len=C if has_prev else 0,
            seg1_k=rk + c0 * row, seg1_v=rv + c0 * row, seg1_len=st.cur_len + t, len_before=st.cur_len,
            has_sinks=st.sinks_set, has_bank=st.has_bank, bank_m=m_res.data_ptr())
        y = plan.y
        if partial_fp32:
            out = torch.mm(y.view(b * t, H * HD), plan.w_out.t(), out_dtype=torch.float32).view(b, t, -1)
        else:
            out = F.linear(y.view(b, t, H * HD), plan.w_out)
        c = plan.consts
        st.cur_len += t
        if st.cur_len >= C:                                                   # bolt3.py:406-425
            if has_prev:
                skip = 0
                if not st.sinks_set:
                    st.sink_k.copy_(st.ring_kp[:, p0:p0 + N_SINKS])
                    st.sink_v.copy_(st.ring_v[:, p0:p0 + N_SINKS])
                    st.sinks_set = True
                    skip = N_SINKS
                bank = dict(st.bank)
                bank["m_res"] = m_res.view(b * HKV, HD, HD)
                K.consolidate(n_chains=b * HKV, hkv=HKV, HD=HD, bank=bank, init_blank=not st.has_bank,
                              kr=st.ring_kr, kp=st.ring_kp, v=st.ring_v, beta=st.ring_b, chain_tokens=2 * C,
                              token0=p0, step_tokens=C, skip0=skip, chunk_len=C,
                              pos0=st.slot_pos[st.prev_slot] - p0, n_steps=1, kappa=c["kappa"],
                              gamma=c["gamma"], inv_freq=c["inv_freq"])
                nf = st.n_filled
                st.n_filled = nf if nf >= ly.S else nf + min(ly.S - nf, C - skip)
            st.prev_slot, st.cur_slot, st.cur_len = st.cur_slot, 1 - st.cur_slot, 0
        return out

    @torch.no_grad()
    def step(self, tokens: torch.Tensor, pos_start: int, states, kv_caches, record=None):
        m = self.model
        b, t_s = tokens.shape
        with torch.autocast("cuda", torch.bfloat16, enabled=tokens.is_cuda):
            x = m.embed_tokens(tokens)
            for li, blk in enumerate(m.blocks):
                h = blk.norm1(x)
                if hasattr(blk, "vsa"):
                    x = x + self.layer_step(blk.vsa, kv_caches[li], h, pos_start, states[li]).to(x.dtype)
                else:
                    ly = blk.attn
                    q, k, v = ly.head_qkv(h)
                    q, k = ly.rope(q, pos_start=pos_start), ly.rope(k, pos_start=pos_start)
                    n_prev = kv_caches[li].n
                    pk, pv = kv_caches[li].append(k, v)
                    mask = None
                    if t_s > 1:
                        qi = torch.arange(t_s, device=tokens.device)[:, None]
                        kj = torch.arange(n_prev + t_s, device=tokens.device)[None, :]
                        mask = (kj <= (n_prev + qi)).view(1, 1, t_s, n_prev + t_s)
                    y = F.scaled_dot_product_attention(q, pk.to(q.dtype), pv.to(q.dtype), attn_mask=mask,
                                                       enable_gqa=(ly.G > 1))
                    x = x + ly.o_proj(y.transpose(1, 2).reshape(b, t_s, ly.H * ly.HD))
                x = x + blk.mlp(blk.norm2(x))
            return m.norm(x), states, kv_caches

    @torch.no_grad()
    def prefill(self, ids: torch.Tensor, max_kv_len: int = 4096):
        b, t = ids.shape
        states, kv = self.blank_state(self.model, b, ids.device, max_kv_len=max(max_kv_len, t + 1024))
        h = None
        for s in range(0, t, self.C):
            e = min(t, s + self.C)
            h, states, kv = self.step(ids[:, s:e], s, states, kv)
        return h, states, kv

    @torch.no_grad()
    def generate_batch(self, ids: torch.Tensor, max_new_tokens: int, temperature: float = 0.6, top_k: int = 40,
                       top_p: float = 0.95, eos_ids: set[int] | None = None,
                       close_think_ids: list[int] | None = None):
        B, T = ids.shape
        h, states, kv = self.prefill(ids, max_kv_len=T + max_new_tokens + 64)
        logits = self.model.lm_head(h[:, -1, :])
        eos = torch.tensor(sorted(eos_ids or ()), device=ids.device, dtype=torch.long)
        done = torch.zeros(B, dtype=torch.bool, device=ids.device)
        lengths = torch.full((B,), max_new_tokens, dtype=torch.long, device=ids.device)
        out, pos = [], T
        for i in range(max_new_tokens):
            nxt = self._sample(logits, temperature, top_k=top_k, top_p=top_p)
            out.append(nxt)
            if eos.numel():
                hit = torch.isin(nxt[:, 0], eos) & ~done
                lengths[hit] = i + 1
                done |= hit
                if i % 16 == 15 and bool(done.all()):
                    break
            h, states, kv = self.step(nxt, pos, states, kv)
            logits = self.model.lm_head(h[:, -1, :])
            pos += 1
        return torch.cat(out, dim=1), lengths


class StaticKV:
    """Growing KV cache of a softmax anchor layer (reference: vsa_lm/decode.py:88-106)."""

    def __init__(self, B: int, HKV: int, Tmax: int, HD: int, dev, dt=torch.bfloat16):
        self.k = torch.empty(B, HKV, Tmax, HD, device=dev, dtype=dt)
        self.v = torch.empty_like(self.k)
        self.n = 0

    def append(self, k_new: torch.Tensor, v_new: torch.Tensor):
        L = k_new.shape[2]
        if self.n + L > self.k.shape[2]:
            new_max = max(self.n + L + 1024, self.k.shape[2] * 2)
            nk = torch.empty(self.k.shape[0], self.k.shape[1], new_max, self.k.shape[3], device=self.k.device,
                             dtype=self.k.dtype)
            nv = torch.empty_like(nk)
            nk[:, :, :self.n] = self.k[:, :, :self.n]
            nv[:, :, :self.n] = self.v[:, :, :self.n]
            self.k, self.v = nk, nv
        self.k[:, :, self.n:self.n + L] = k_new
        self.v[:, :, self.n:self.n + L] = v_new
        self.n += L
        return self.k[:, :, :self.n], self.v[:, :, :self.n]
