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
from . import oversize

N_SINKS = 4


# --------------------------------------------------------------------------------------------
# helper modules with the reference's parameter layout (vsa_lm/surgery.py:43-93)

class LlamaRMSNorm(nn.Module):
    """RMSNorm computed in fp32 and cast back to the input dtype; parameter `weight` as in the
    reference (surgery.py:43-53), so checkpoints load. bf16 CUDA inputs (outside autograd) take the
    one-kernel bolt3_rmsnorm."""

    def __init__(self, dim: int, eps: float = 1e-5):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def _kernel_ok(self, x: torch.Tensor) -> bool:
        return (x.is_cuda and x.dtype == torch.bfloat16 and x.shape[-1] % 8 == 0 and x.shape[-1] <= 4096
                and not (torch.is_grad_enabled() and (x.requires_grad or self.weight.requires_grad)))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self._kernel_ok(x):
            return K.rmsnorm(x, self.weight, self.eps)       # one kernel (csrc/rmsnorm.cu)
        out = F.rms_norm(x.float(), (x.shape[-1],), self.weight.float(), self.eps)
        return out.to(x.dtype)

    def add_forward(self, x: torch.Tensor, d: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """The residual update and the norm of its result, (x + d, norm(x + d)): one kernel for bf16
        CUDA tensors (the sum rounded to bf16 as torch's bf16 addition rounds it)."""
        if self._kernel_ok(x) and d.dtype == x.dtype and d.shape == x.shape:
            return K.add_rmsnorm(x, d, self.weight, self.eps)
        x = x + d
        return x, self(x)


def llama_inv_freq(head_dim: int, theta: float, rope_scaling: dict | None, device=None) -> torch.Tensor:
    """RoPE inverse frequencies with optional llama3 scaling. The values must equal the reference's
    bit for bit (surgery.py:56-72), so the arithmetic follows it step by step."""
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
    """Rotate-half RoPE at integer positions pos_start + t, with cos/sin rounded to the input dtype
    and the products and sums in that dtype (the reference's arithmetic, surgery.py:80-93). The
    `inv_freq` buffer is non-persistent, as in the reference."""

    def __init__(self, head_dim: int, theta: float, rope_scaling: dict | None):
        super().__init__()
        self.register_buffer("inv_freq", llama_inv_freq(head_dim, theta, rope_scaling, torch.device("cpu")),
                             persistent=False)

    def forward(self, x: torch.Tensor, pos_start: int = 0) -> torch.Tensor:
        pos = torch.arange(x.shape[2], device=x.device, dtype=torch.float32) + float(pos_start)
        return self.forward_at(x, pos)

    def forward_at(self, x: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        """RoPE at the fp32 positions `pos` [T] held on the device (the same arithmetic as forward)."""
        ang = torch.outer(pos, self.inv_freq.to(device=x.device, dtype=torch.float32))
        c, s = ang.cos().to(x.dtype), ang.sin().to(x.dtype)
        x1, x2 = x.chunk(2, dim=-1)
        return torch.cat((x1 * c - x2 * s, x2 * c + x1 * s), dim=-1)


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

    # ---- device status word (include/bolt3.h): one per device this module runs on
    def device_status(self, device) -> K.DeviceStatus:
        cache = self.__dict__.setdefault("_status_words", {})
        key = str(torch.device(device))
        if key not in cache:
            cache[key] = K.DeviceStatus(device)
        return cache[key]

    def check_status(self, block: bool = True) -> None:
        """Raise RuntimeError if a kernel of an earlier forward reported an error (an expired
        bounded wait or a failed bounds check). Every forward already checks the previous one's
        status without waiting; `block` waits for the last forward's kernels to finish."""
        for st in self.__dict__.get("_status_words", {}).values():
            st.check(block)

    @torch.no_grad()
    def _prepare(self, x: torch.Tensor):
        """Projections + RMSNorm/RoPE/gates of the whole input (phase A, bolt3.py:196-199), as the
        head-major buffers the scan and the attention read. Returns a namespace of the buffers and a
        callable that runs the q/eta half (so the caller can start the scan on k/v/beta first)."""
        if not x.is_cuda:
            raise RuntimeError("Bolt3Attn (B200 native) runs on CUDA tensors only; no CPU path exists")
        b, T, D = x.shape
        H, HKV, HD = self.H, self.HKV, self.HD
        dev = x.device
        f = self.fused(dev)
        c = f.consts
        x2 = x.reshape(b * T, D).to(torch.bfloat16)
        bf = dict(dtype=torch.bfloat16, device=dev)
        p = types.SimpleNamespace(b=b, T=T, f=f, consts=c)
        p.q_raw = torch.empty(b * H, T, HD, **bf)
        p.q_rope = torch.empty_like(p.q_raw)
        p.k_raw = torch.empty(b * HKV, T, HD, **bf)
        p.k_rope = torch.empty_like(p.k_raw)
        p.v = torch.empty_like(p.k_raw)
        p.beta = torch.empty(b * HKV, T, dtype=torch.float32, device=dev)
        p.eta = torch.empty(b * H, T, dtype=torch.float32, device=dev)
        p.q_l2 = torch.empty(b * H, T, dtype=torch.float32, device=dev)
        common = dict(B=b, T=T, H=H, HKV=HKV, HD=HD, inv_freq=c["inv_freq"], eps=self.eps, q_norm_w=c["qn"],
                      k_norm_w=c["kn"], pos0=0)
        # k/v/beta first: the consolidation scan waits only on them
        K.prep(self.project(x2, f, "kv"), cols=f.cols_kv, parts=2, k_raw=p.k_raw, k_rope=p.k_rope, v=p.v,
               beta=p.beta, k_head_stride=T, k_t_off=0, **common)

        def prep_q():
            K.prep(self.project(x2, f, "q"), cols=f.cols_q, parts=1, q_raw=p.q_raw, q_rope=p.q_rope, eta=p.eta,
                   q_head_stride=T, q_t_off=0, q_l2=p.q_l2, **common)
        return p, prep_q

    @torch.no_grad()
    def _attention_heads(self, x: torch.Tensor) -> torch.Tensor:
        """The attention output of every head before o_proj, y [b, T, H, HD] bf16 (phases A-C of
        bolt3.py:194-274). Checks the previous call's device status without waiting, and arms this
        call's."""
        status = self.device_status(x.device)
        status.check(block=False)
        p, prep_q = self._prepare(x)
        b, T = p.b, p.T
        dev = x.device
        ws = torch.empty(max(1, K.prefill_workspace_bytes(b * self.HKV, T, self.HD)), dtype=torch.uint8, device=dev)
        bank = K.new_bank(b * self.HKV, self.HD, dev)
        y = torch.empty(b, T, self.H, self.HD, dtype=torch.bfloat16, device=dev)
        self._scan_and_attend(b, T, q_rope=p.q_rope, q_raw=p.q_raw, eta=p.eta, k_raw=p.k_raw, k_rope=p.k_rope,
                              v=p.v, beta=p.beta, q_l2=p.q_l2, ws=ws, bank=bank, y=y, consts=p.consts,
                              before_attend=prep_q, status=status)
        status.arm(f"Bolt3Attn forward of {b} x {T} tokens")
        return y

    @torch.no_grad()
    @K.traced("Bolt3Attn.forward")
    def _native_forward(self, x: torch.Tensor, partial_fp32: bool = False) -> torch.Tensor:
        """The forward on CUDA. partial_fp32: return o_proj's output in fp32, unrounded (a tensor-
        parallel shard's partial sum, rounded once after the all-reduce)."""
        y = self._attention_heads(x)
        b, T = x.shape[:2]
        f = self.fused(x.device)
        if partial_fp32:
            return torch.mm(y.view(b * T, self.H * self.HD), f.w_out.t(), out_dtype=torch.float32).view(b, T, -1)
        out = F.linear(y.view(b, T, self.H * self.HD), f.w_out)
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
                         before_attend=None, status=None):
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
                   eps=self.eps, y=y, q_l2=q_l2, status=status)
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
                              kappa=c["kappa"], gamma=c["gamma"], inv_freq=c["inv_freq"], snaps=snaps, snap0=s0,
                              status=status)
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

    @torch.no_grad()
    def step_projections(self, h: torch.Tensor, pos_start: int):
        """The projections a decode step of h [b, t, D] at positions pos_start.. computes (the fused
        input GEMM and bolt3_prep, as Bolt3Decoder.layer_step runs them), returned in the
        reference's head-major layouts: q_raw [b, H, t, HD], k_raw and v [b, HKV, t, HD] bf16,
        beta [b, HKV, t] and eta [b, H, t] fp32. For inspecting a step, e.g. to check its other
        phases on exactly these inputs."""
        b, t, D = h.shape
        H, HKV, HD = self.H, self.HKV, self.HD
        f = self.fused(h.device)
        c = f.consts
        bf = dict(dtype=torch.bfloat16, device=h.device)
        q_raw, q_rope = torch.empty(b * H, t, HD, **bf), torch.empty(b * H, t, HD, **bf)
        k_raw, k_rope, v = (torch.empty(b * HKV, t, HD, **bf) for _ in range(3))
        beta = torch.empty(b * HKV, t, dtype=torch.float32, device=h.device)
        eta = torch.empty(b * H, t, dtype=torch.float32, device=h.device)
        proj = F.linear(h.reshape(b * t, D).to(torch.bfloat16), f.w_in, f.b_in)
        K.prep(proj, B=b, T=t, H=H, HKV=HKV, HD=HD, inv_freq=c["inv_freq"], eps=self.eps, q_norm_w=c["qn"],
               k_norm_w=c["kn"], pos0=pos_start, cols=f.cols, q_raw=q_raw, q_rope=q_rope, eta=eta, k_raw=k_raw,
               k_rope=k_rope, v=v, beta=beta, q_head_stride=t, q_t_off=0, k_head_stride=t, k_t_off=0)
        return (q_raw.view(b, H, t, HD), k_raw.view(b, HKV, t, HD), v.view(b, HKV, t, HD), beta.view(b, HKV, t),
                eta.view(b, H, t))

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
                      inv_freq=f.consts["inv_freq"], status=self.device_status(dev))
        st = self.device_status(dev)
        st.arm(f"_consolidate_functional of {bh} chains")
        st.check(block=True)
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
        # zeros, not empty: a step replayed from a CUDA graph reads its window slot past the current
        # length and masks those keys, and a masked value row must still be finite (0 x NaN is NaN)
        self.ring_kr = torch.zeros(n, 2 * self.C, self.HD, **bf)
        self.ring_kp = torch.zeros_like(self.ring_kr)
        self.ring_v = torch.zeros_like(self.ring_kr)
        self.ring_b = torch.empty(n, 2 * self.C, dtype=torch.float32, device=device)
        self.sink_k = torch.empty(n, N_SINKS, self.HD, **bf)
        self.sink_v = torch.empty_like(self.sink_k)
        # the bank without an M_res of its own: M_res is the caller's states[li], which every kernel
        # call is given (a second [n, HD, HD] fp32 array here would never be read)
        self.bank = K.new_bank(n, self.HD, device, m_res=False)
        self.slot_pos = [0, 0]
        self.cur_slot, self.cur_len = 0, 0
        self.prev_slot = -1
        self.sinks_set = False
        self.n_filled = 0
        self._plans = {}   # per step size: buffers and prebuilt launch arguments (Bolt3Decoder)
        self._consts = None  # the layer constants of the last step's plan (its chunk boundary uses them)
        # a previous chunk of more than C tokens (kr, kp, v, beta, pos0), held outside the ring until
        # it is consolidated (vsa_lm_b200/oversize.py); None in the common case
        self.big_prev = None
        # device status word of this state's kernels, checked at every chunk boundary
        self.status = K.DeviceStatus(device)

    @property
    def has_bank(self) -> bool:
        return self.n_filled > 0

    @staticmethod
    def bytes_per_sequence(ly: Bolt3Attn) -> int:
        """Device bytes one sequence's state of layer `ly` occupies: the buffers __init__ allocates
        (window ring kr/kp/v/beta, sinks, bank ak/av/ak_rope/mass/util/pm/act/n_filled) plus the
        caller's M_res."""
        HKV, HD, C, S = ly.HKV, ly.HD, ly.C, ly.S
        ring = 3 * 2 * C * HD * 2 + 2 * C * 4
        sinks = 2 * N_SINKS * HD * 2
        bank = 3 * S * HD * 2 + 3 * S * 4 + S + 4
        return HKV * (ring + sinks + bank + HD * HD * 4)


class Bolt3Decoder:
    """Constant-memory decoder (reference: vsa_lm/config/bolt3.py:279-557) with native Bolt-3 layers.

    Softmax anchor layers use a static KV cache and SDPA as in the reference (bolt3.py:426-445).
    """

    def __init__(self, model, wrap_positions: bool = False, max_cache_pos: int = 65536, cuda_graphs: bool = True,
                 **kwargs):
        self.model = model.eval()
        self.max_T = model.config["max_T"]
        self.max_cache_pos = max_cache_pos
        self.C = int(model.config.get("bolt3_C", 128))
        # generation loops replay their one-token steps from CUDA graphs (the reference runs them
        # eagerly, bolt3.py:287-288: a step of a 36-layer model is hundreds of launches)
        self.use_cuda_graphs = cuda_graphs

    @staticmethod
    def state_bytes(model):
        """(bytes of fixed-size state per sequence, bytes per token of the anchor layers' KV caches),
        the same pair the reference reports (bolt3.py:290-300), counted from the buffers this
        decoder actually keeps (Bolt3LayerState.bytes_per_sequence, AnchorKV's bf16 k and v)."""
        fixed = sum(Bolt3LayerState.bytes_per_sequence(b.vsa) for b in model.blocks if hasattr(b, "vsa"))
        per_token = sum(2 * b.attn.HKV * b.attn.HD * 2 for b in model.blocks if not hasattr(b, "vsa"))
        return fixed, per_token

    @staticmethod
    def blank_state(model, batch_size: int, device, max_kv_len: int = 4096, state_dtype=torch.float32, **kwargs):
        """(states, kv_caches) for `batch_size` sequences (bolt3.py:302-319): per Bolt-3 layer an fp32
        M_res [B, HKV, HD, HD] in states and a Bolt3LayerState in kv_caches; per softmax anchor an
        AnchorKV with room for max_kv_len tokens. M_res is always fp32 (the kernels update it in place)."""
        states, kv_caches = [], []
        for blk in model.blocks:
            if hasattr(blk, "vsa"):
                ly = blk.vsa
                states.append(torch.zeros(batch_size, ly.HKV, ly.HD, ly.HD, device=device, dtype=torch.float32))
                kv_caches.append(Bolt3LayerState(ly, batch_size, device))
            else:
                a = blk.attn
                states.append(None)
                kv_caches.append(AnchorKV(batch_size, a.HKV, max_kv_len, a.HD, device, dt=torch.bfloat16))
        return states, kv_caches

    @staticmethod
    def check_status(kv_caches, block: bool = True) -> None:
        """Raise RuntimeError if a kernel of an earlier step reported an error (an expired bounded
        wait or a failed bounds check). Steps already check at every chunk boundary."""
        for st in kv_caches:
            if isinstance(st, Bolt3LayerState):
                st.status.check(block)

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

        if st.big_prev is not None:
            bp = st.big_prev
            L = bp["kp"].shape[1]
            for k in ("kr", "kp", "v"):
                d["prev_" + k] = bp[k].reshape(B, HKV, L, HD).clone()
            d["prev_b"] = bp["beta"].reshape(B, HKV, L).to(torch.bfloat16)
            d["prev_pos"] = torch.arange(bp["pos0"], bp["pos0"] + L, dtype=torch.float32,
                                         device=bp["kp"].device).view(1, 1, L)
        elif st.prev_slot >= 0:
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
            L = d["prev_kp"].shape[2]
            if L == C:
                fill("prev", 0)
                st.prev_slot, st.cur_slot = 0, 1
            else:   # a longer previous chunk stays outside the ring until it is consolidated
                st.big_prev = dict(kr=d["prev_kr"].reshape(n, L, HD).to(**dev, dtype=torch.bfloat16).contiguous(),
                                   kp=d["prev_kp"].reshape(n, L, HD).to(**dev, dtype=torch.bfloat16).contiguous(),
                                   v=d["prev_v"].reshape(n, L, HD).to(**dev, dtype=torch.bfloat16).contiguous(),
                                   beta=d["prev_b"].reshape(n, L).to(**dev, dtype=torch.float32).contiguous(),
                                   pos0=int(d["prev_pos"].reshape(-1)[0].item()))
        if d.get("cur_kp") is not None:
            st.cur_len = fill("cur", st.cur_slot)
            if st.cur_len >= C:
                raise NotImplementedError("a pending chunk of C tokens is consolidated by the step that fills it")
        return st

    @staticmethod
    def _sample(logits, temperature: float, top_k: int = 40, top_p: float = 0.95):
        """Next token of every row, [B, 1] (the reference's sampling rule, bolt3.py:321-333): greedy
        for temperature ~ 0; otherwise a draw from softmax(logits / temperature) restricted to the
        nucleus (the tokens, by descending probability, whose preceding mass is <= top_p) when
        top_p < 1, else to the top_k logits. The draw is a Gumbel-max on the device, so nothing
        waits on the host."""
        if temperature <= 1e-5:
            return logits.argmax(dim=-1, keepdim=True)
        z = logits.float() / temperature
        if top_p < 1.0:
            probs, order = torch.sort(torch.softmax(z, dim=-1), dim=-1, descending=True)
            ahead = torch.cumsum(probs, dim=-1) - probs
            cand = torch.where(ahead > top_p, torch.full_like(probs, float("-inf")), probs.log())
        else:
            vals, order = torch.topk(z, min(top_k, z.shape[-1]), dim=-1)
            cand = torch.log_softmax(vals, dim=-1)
        u = torch.rand_like(cand).clamp_(1e-20, 1.0)
        pick = torch.argmax(cand - torch.log(-torch.log(u)), dim=-1, keepdim=True)
        return order.gather(-1, pick)

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
            res_w=c["res_w"].data_ptr(), eps=ly.eps, y=plan.y.data_ptr(), y_tokens=t, q_l2=plan.q_l2.data_ptr(),
            status=st.status.word.data_ptr())
        plan.args = K.DecodeStepArgs(prep, attend)
        return plan

    @staticmethod
    @K.traced("Bolt3Decoder.layer_step")
    def layer_step(ly: Bolt3Attn, st: Bolt3LayerState, h: torch.Tensor, pos_start: int,
                   m_res: torch.Tensor, partial_fp32: bool = False) -> torch.Tensor:
        """Attention branch of one Bolt-3 layer for t new tokens: returns o_proj(y) [b, t, D] bf16
        (fp32 and unrounded with partial_fp32: a tensor-parallel shard's partial sum). A step that
        pushes the pending chunk past C tokens, and every step while such a chunk is in the window,
        runs vsa_lm_b200/oversize.py's path (bolt3.py:355-363, 406-425)."""
        if st.cur_len + h.shape[1] > ly.C or st.big_prev is not None:
            Bolt3Decoder._check_step(ly, st, h, m_res)
            return oversize.layer_step(ly, st, h, pos_start, m_res, partial_fp32, Bolt3Decoder._consolidate_ring)
        out = Bolt3Decoder._layer_launch(ly, st, h, pos_start, m_res, partial_fp32)
        Bolt3Decoder._layer_advance(ly, st, h.shape[1], pos_start, m_res)
        return out

    @staticmethod
    def _check_step(ly: Bolt3Attn, st: Bolt3LayerState, h: torch.Tensor, m_res: torch.Tensor) -> None:
        b, t, D = h.shape
        if b != st.B or h.device != m_res.device or not h.is_cuda:
            raise ValueError(f"hidden states [{b}, {t}, {D}] on {h.device} do not match a state of {st.B} sequences "
                             f"with M_res on {m_res.device}")
        if h.device.index != torch.cuda.current_device():
            raise RuntimeError(f"the step's tensors are on {h.device}; make that device current")
        if not (m_res.dtype == torch.float32 and m_res.is_contiguous()
                and tuple(m_res.shape) == (b, ly.HKV, ly.HD, ly.HD)):
            raise ValueError(f"m_res must be a contiguous fp32 CUDA tensor [{b}, {ly.HKV}, {ly.HD}, {ly.HD}]")

    @staticmethod
    def _layer_launch(ly: Bolt3Attn, st: Bolt3LayerState, h: torch.Tensor, pos_start: int, m_res: torch.Tensor,
                      partial_fp32: bool = False, dev_pos: "K.DevicePosition | None" = None) -> torch.Tensor:
        """The kernels of a Bolt-3 layer step (projection, prep, attention, o_proj), enqueued on the
        current stream; the state's host bookkeeping is _layer_advance's. With dev_pos (a step captured
        into a CUDA graph) the kernels read the step's position from the device: the launch is built
        for position dev_pos.ref and stays valid for dev_pos.span positions of the current chunk."""
        b, t, D = h.shape
        H, HKV, HD, C, G = ly.H, ly.HKV, ly.HD, ly.C, ly.G
        if st.cur_len + t > C or st.big_prev is not None:
            # the native kernels hold windows of two chunks of at most C tokens (layer_step takes
            # oversize chunks through vsa_lm_b200/oversize.py)
            raise ValueError(f"a native launch needs a window of chunks of at most {C} tokens")
        Bolt3Decoder._check_step(ly, st, h, m_res)
        if dev_pos is not None and (t != 1 or dev_pos.ref != pos_start or st.cur_len + dev_pos.span > C):
            raise ValueError("a device-position launch is a one-token step at its reference position whose span "
                             "stays within the chunk")
        if st.cur_len == 0:
            st.slot_pos[st.cur_slot] = pos_start
        elif pos_start != st.slot_pos[st.cur_slot] + st.cur_len:
            raise NotImplementedError("native decoder needs contiguous positions within a chunk")
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
        st._consts = plan.consts
        proj = F.linear(h.reshape(b * t, D).to(torch.bfloat16), plan.w_in, plan.b_in)
        plan.args.launch_prep(proj, pos_start, st.cur_slot * C + st.cur_len, dev_pos)
        has_prev = st.prev_slot >= 0
        p0 = st.prev_slot * C if has_prev else 0
        c0 = st.cur_slot * C
        rk, rv, row = plan.ring_kp, plan.ring_v, plan.ring_row
        plan.args.launch_attend(
            seg0_k=rk + p0 * row, seg0_v=rv + p0 * row, seg0_len=C if has_prev else 0,
            seg1_k=rk + c0 * row, seg1_v=rv + c0 * row, seg1_len=st.cur_len + t, len_before=st.cur_len,
            has_sinks=st.sinks_set, has_bank=st.has_bank, bank_m=m_res.data_ptr(), dev_pos=dev_pos)
        y = plan.y
        if partial_fp32:
            return torch.mm(y.view(b * t, H * HD), plan.w_out.t(), out_dtype=torch.float32).view(b, t, -1)
        return F.linear(y.view(b, t, H * HD), plan.w_out)

    @staticmethod
    def _layer_advance(ly: Bolt3Attn, st: Bolt3LayerState, t: int, pos_start: int, m_res: torch.Tensor) -> None:
        """Host side of a Bolt-3 layer step whose kernels are enqueued: the pending chunk grows by t
        tokens, and a chunk that reaches C tokens consolidates the previous one into the bank and
        M_res (bolt3.py:406-425) and becomes the previous chunk."""
        C = ly.C
        st.cur_len += t
        if st.cur_len >= C:                                                   # bolt3.py:406-425
            # errors of the previous chunk's kernels (their status copy finished long ago)
            st.status.check(block=True)
            if st.prev_slot >= 0:
                Bolt3Decoder._consolidate_ring(ly, st, m_res, st._consts)
            st.prev_slot, st.cur_slot, st.cur_len = st.cur_slot, 1 - st.cur_slot, 0
            st.status.arm(f"Bolt-3 decode chunk ending at position {pos_start + t}")

    @staticmethod
    @K.traced("Bolt3Decoder.consolidate")
    def _consolidate_ring(ly: Bolt3Attn, st: Bolt3LayerState, m_res: torch.Tensor, c: dict) -> None:
        """The native consolidation of the previous chunk (C tokens in its ring slot) into the bank
        and M_res; the first one also sets the sinks and leaves them out (bolt3.py:408-425)."""
        b, HKV, HD, C = st.B, ly.HKV, ly.HD, ly.C
        p0 = st.prev_slot * C
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
                      gamma=c["gamma"], inv_freq=c["inv_freq"], status=st.status)
        nf = st.n_filled
        st.n_filled = nf if nf >= ly.S else nf + min(ly.S - nf, C - skip)

    @staticmethod
    def _anchor_attention(ly, cache: "AnchorKV", h: torch.Tensor, pos_start: int,
                          partial_fp32: bool = False, dev_pos: "K.DevicePosition | None" = None) -> torch.Tensor:
        """A softmax anchor layer's attention branch for t new tokens (bolt3.py:426-445): RoPE at
        pos_start, the new k/v appended to the layer's cache, causal within the new block
        (partial_fp32: o_proj's output in fp32, unrounded, as a tensor-parallel shard's partial sum).
        One-token steps on the GPU run bolt3_anchor_decode (append and attention in one kernel); with
        dev_pos (a step captured into a CUDA graph) the position comes from the device and the cache's
        host count is left to the caller."""
        b, t, _ = h.shape
        q, k, v = ly.head_qkv(h)
        if t == 1 and h.is_cuda and q.dtype == torch.bfloat16 and cache.buf.dtype == torch.bfloat16:
            if dev_pos is None:
                cache.reserve(1)
            # RoPE of q and the new key inside the kernel, at pos_start (shifted with the device position)
            y = torch.empty(b, ly.H, ly.HD, dtype=torch.bfloat16, device=h.device)
            K.anchor_decode(q=q.reshape(b, ly.H, ly.HD).contiguous(), k_new=k.reshape(b, ly.HKV, ly.HD).contiguous(),
                            v_new=v.reshape(b, ly.HKV, ly.HD).contiguous(), k_cache=cache.k, v_cache=cache.v,
                            n=cache.n, y=y, scale=ly.HD ** -0.5, dev_pos=dev_pos,
                            inv_freq=_fp32_inv_freq(ly.rope, h.device), pos0=pos_start)
            if dev_pos is None:
                cache.n += 1
            y = y.view(b, 1, ly.H * ly.HD)
        else:
            if dev_pos is not None:
                raise ValueError("device-position anchor steps are one bf16 token on the GPU")
            q, k = ly.rope(q, pos_start=pos_start), ly.rope(k, pos_start=pos_start)
            n_before = cache.n
            keys, vals = cache.append(k, v)
            mask = None
            if t > 1:   # query i sees every cached key and the new keys up to itself
                mask = torch.ones(t, n_before + t, dtype=torch.bool, device=h.device).tril(diagonal=n_before)
            y = F.scaled_dot_product_attention(q, keys.to(q.dtype), vals.to(q.dtype), attn_mask=mask,
                                               enable_gqa=ly.G > 1)
            y = y.transpose(1, 2).reshape(b, t, ly.H * ly.HD)
        if partial_fp32:
            w = ly.o_proj.weight
            return torch.mm(y.reshape(b * t, -1).to(w.dtype), w.t(), out_dtype=torch.float32).view(b, t, -1)
        return ly.o_proj(y)

    @torch.no_grad()
    @K.traced("Bolt3Decoder.step")
    def step(self, tokens: torch.Tensor, pos_start: int, states, kv_caches, record=None):
        """Run t new tokens [b, t] at positions pos_start.. through every block; returns the final
        normed hidden states [b, t, D] and the (updated in place) state lists (bolt3.py:335-447)."""
        return self._blocks(tokens, pos_start, states, kv_caches), states, kv_caches

    def _blocks(self, tokens: torch.Tensor, pos_start: int, states, kv_caches,
                dev_pos: "K.DevicePosition | None" = None) -> torch.Tensor:
        """The step's computation. With dev_pos only the kernels are enqueued (a step captured into a
        CUDA graph: the position comes from the device, the host bookkeeping is _advance's)."""
        m = self.model
        blocks = m.blocks
        with torch.autocast("cuda", torch.bfloat16, enabled=tokens.is_cuda):
            x = m.embed_tokens(tokens)
            h = blocks[0].norm1(x)
            for li, blk in enumerate(blocks):
                if hasattr(blk, "vsa"):
                    if dev_pos is None:
                        attn = self.layer_step(blk.vsa, kv_caches[li], h, pos_start, states[li])
                    else:
                        attn = self._layer_launch(blk.vsa, kv_caches[li], h, pos_start, states[li], dev_pos=dev_pos)
                else:
                    attn = self._anchor_attention(blk.attn, kv_caches[li], h, pos_start, dev_pos=dev_pos)
                # each residual update and the norm that reads its result are one kernel
                x, h2 = blk.norm2.add_forward(x, attn.to(x.dtype))
                nxt = blocks[li + 1].norm1 if li + 1 < len(blocks) else m.norm
                x, h = nxt.add_forward(x, blk.mlp(h2).to(x.dtype))
            return h

    def _advance(self, t: int, pos_start: int, states, kv_caches) -> None:
        """Host bookkeeping of a step whose kernels ran without it (a CUDA-graph replay)."""
        for li, blk in enumerate(self.model.blocks):
            if hasattr(blk, "vsa"):
                self._layer_advance(blk.vsa, kv_caches[li], t, pos_start, states[li])
            else:
                kv_caches[li].n += t

    def graphs_supported(self, device) -> bool:
        """One-token steps may be replayed from CUDA graphs on this device: a CUDA model whose
        parameters and buffers (the RoPE frequencies among them) all live on that device."""
        device = torch.device(device)
        if not (self.use_cuda_graphs and device.type == "cuda"):
            return False
        idx = device.index if device.index is not None else torch.cuda.current_device()
        return all(t.device.type == "cuda" and t.device.index == idx
                   for t in list(self.model.parameters()) + list(self.model.buffers()))

    def step_graph(self, states, kv_caches) -> "DecodeGraph":
        """A runner of one-token steps on (states, kv_caches) replayed from CUDA graphs (one capture
        per chunk of C positions); results equal step()'s."""
        return DecodeGraph(self, states, kv_caches)

    def _feed(self, ids: torch.Tensor, pos: int, states, kv_caches):
        """Run a prompt through step() in C-token slices from position `pos`; returns the last
        slice's hidden states and the position after the prompt."""
        h = None
        for s0 in range(0, ids.shape[1], self.C):
            piece = ids[:, s0:s0 + self.C]
            h, states, kv_caches = self.step(piece, pos, states, kv_caches)
            pos += piece.shape[1]
        return h, pos

    @torch.no_grad()
    def prefill(self, ids: torch.Tensor, max_kv_len: int = 4096):
        """Fresh state for ids [b, t] and the prompt run through it (bolt3.py:449-457)."""
        states, kv = self.blank_state(self.model, ids.shape[0], ids.device, max_kv_len=max(max_kv_len, ids.shape[1] + 1024))
        h, _ = self._feed(ids, 0, states, kv)
        return h, states, kv

    @torch.no_grad()
    def generate_batch(self, ids: torch.Tensor, max_new_tokens: int, temperature: float = 0.6, top_k: int = 40,
                       top_p: float = 0.95, eos_ids: set[int] | None = None,
                       close_think_ids: list[int] | None = None):
        """Decode max_new_tokens for every row of ids [B, T] after prefilling it (bolt3.py:459-500).
        Returns (tokens [B, n], lengths [B]): a row's length is the step at which it produced an
        end-of-sequence id (inclusive), else max_new_tokens; decoding stops early once every row has
        finished (checked every 16 tokens). With close_think_ids, rows that have not closed their
        thinking block by step max(64, max_new_tokens - 64) are forced to emit that token sequence."""
        B, T = ids.shape
        dev = ids.device
        h, states, kv = self.prefill(ids, max_kv_len=T + max_new_tokens + 64)
        logits = self.model.lm_head(h[:, -1, :])
        eos = torch.tensor(sorted(eos_ids or ()), dtype=torch.long, device=dev)
        finished = torch.zeros(B, dtype=torch.bool, device=dev)
        lengths = torch.full((B,), max_new_tokens, dtype=torch.long, device=dev)
        forced = None
        if close_think_ids:
            forced = torch.tensor(list(close_think_ids), dtype=torch.long, device=dev)
            closer = int(close_think_ids[1]) if len(close_think_ids) > 1 else None
            cursor = torch.full((B,), -1, dtype=torch.long, device=dev)   # next forced token, -1 = none
            closed = torch.zeros(B, dtype=torch.bool, device=dev)
            trigger = max(64, max_new_tokens - 64)
        toks = []
        runner = self.step_graph(states, kv) if self.graphs_supported(dev) else None
        for i in range(max_new_tokens):
            nxt = self._sample(logits, temperature, top_k=top_k, top_p=top_p)
            if forced is not None:
                if i == trigger:
                    cursor = torch.where(~closed & ~finished & (cursor < 0), torch.zeros_like(cursor), cursor)
                active = cursor >= 0
                nxt = torch.where(active[:, None], forced[cursor.clamp(min=0)][:, None], nxt)
                cursor = torch.where(active, cursor + 1, cursor)
                done_forcing = active & (cursor >= forced.numel())
                closed = closed | done_forcing
                cursor = torch.where(done_forcing, torch.full_like(cursor, -1), cursor)
                if closer is not None:
                    closed = closed | (nxt[:, 0] == closer)
            toks.append(nxt)
            if eos.numel():
                newly = torch.isin(nxt[:, 0], eos) & ~finished
                lengths = torch.where(newly, torch.full_like(lengths, i + 1), lengths)
                finished = finished | newly
                if i % 16 == 15 and bool(finished.all()):
                    break
            if runner is not None:
                h = runner.step(nxt, T + i)
            else:
                h, states, kv = self.step(nxt, T + i, states, kv)
            logits = self.model.lm_head(h[:, -1, :])
        if runner is not None:
            runner.close()
        return torch.cat(toks, dim=1), lengths

    @torch.no_grad()
    def generate(self, prompt: torch.Tensor, max_new_tokens: int, temperature: float = 0.0, top_k: int = 40,
                 top_p: float = 0.95, eos_ids: set[int] | None = None, close_think_ids: list[int] | None = None):
        """The prompt followed by the first row's generated tokens up to its length (bolt3.py:502-506)."""
        toks, n = self.generate_batch(prompt, max_new_tokens, temperature, top_k, top_p, eos_ids, close_think_ids)
        return torch.cat([prompt, toks[:, :int(n[0])]], dim=1)

    @torch.no_grad()
    def continue_generate(self, ids: torch.Tensor, states, kv_caches, start_pos: int, max_new_tokens: int,
                          temperature: float = 0.0, top_k: int = 40, top_p: float = 0.95,
                          eos_ids: set[int] | None = None):
        """Feed ids from start_pos onto existing state, then decode up to max_new_tokens, stopping
        before the step of an end-of-sequence id of row 0 (bolt3.py:508-526). Returns (tokens,
        states, kv_caches, next position)."""
        h, pos = self._feed(ids, start_pos, states, kv_caches)
        logits = self.model.lm_head(h[:, -1, :])
        toks = []
        runner = self.step_graph(states, kv_caches) if self.graphs_supported(ids.device) else None
        for _ in range(max_new_tokens):
            nxt = self._sample(logits, temperature, top_k=top_k, top_p=top_p)
            toks.append(nxt)
            if eos_ids and int(nxt[0, 0]) in eos_ids:
                break
            if runner is not None:
                h = runner.step(nxt, pos)
            else:
                h, states, kv_caches = self.step(nxt, pos, states, kv_caches)
            logits = self.model.lm_head(h[:, -1, :])
            pos += 1
        if runner is not None:
            runner.close()
        out = torch.cat(toks, dim=1) if toks else torch.empty(ids.shape[0], 0, dtype=torch.long, device=ids.device)
        return out, states, kv_caches, pos

    @torch.no_grad()
    def memorize(self, ids: torch.Tensor, states, kv_caches, start_pos: int):
        """Feed a document from start_pos and record, per Bolt-3 layer, the change it made to M_res
        net of the decay the earlier state went through: trace = (end position, M_after -
        gamma^(n_tokens // C) * M_before) (bolt3.py:528-545). Other layers get None."""
        before = {li: states[li].clone() for li, blk in enumerate(self.model.blocks) if hasattr(blk, "vsa")}
        _, pos = self._feed(ids, start_pos, states, kv_caches)
        n_tok = ids.shape[1]
        traces = []
        for li, blk in enumerate(self.model.blocks):
            if li not in before:
                traces.append(None)
                continue
            decay = blk.vsa.gamma_delta().to(states[li].device).view(1, -1, 1, 1) ** (n_tok // blk.vsa.C)
            traces.append((pos, states[li] - decay * before[li]))
        return states, kv_caches, pos, traces

    @torch.no_grad()
    def forget(self, traces, states, next_pos: int, kv_caches=None, pre_kv_lens=None):
        """Subtract memorized traces from M_res, each decayed by the chunks consolidated since its
        end position: M -= gamma^max(0, (next_pos - end) // C) * delta (bolt3.py:547-557). The new
        states[li] are fresh fp32 tensors; later steps update them in place."""
        for li, tr in enumerate(traces):
            if tr is None or states[li] is None:
                continue
            end, delta = tr
            ly = self.model.blocks[li].vsa
            k = max(0, (next_pos - end) // ly.C)
            decay = ly.gamma_delta().to(delta.device).view(1, -1, 1, 1) ** k
            states[li] = (states[li] - decay * delta).contiguous()
        return states


def _fp32_inv_freq(rope: "LlamaRoPE", device) -> torch.Tensor:
    """The RoPE module's frequencies as a contiguous fp32 tensor on `device`, kept between calls (made
    again when the buffer is replaced or changed in place): a kernel argument, not a per-step copy."""
    t = rope.inv_freq
    key = (t.data_ptr(), t._version, t.dtype, str(torch.device(device)))
    cached = getattr(rope, "_fp32_cache", None)
    if cached is None or cached[0] != key:
        cached = (key, t.detach().to(device=device, dtype=torch.float32).contiguous())
        rope._fp32_cache = cached
    return cached[1]


class AnchorKV:
    """KV cache of one softmax anchor layer: a single buffer [2, B, HKV, capacity, HD] written in
    place. `k`, `v` (views of the buffer) and `n` (tokens held) carry the names of the reference's
    cache (vsa_lm/decode.py:88-106), so code that reads a cache, such as a cartridge writer, works
    unchanged. The capacity is max_kv_len rounded up to a multiple of 256 tokens; an append that
    does not fit doubles it (one copy of the held tokens)."""

    def __init__(self, B: int, HKV: int, Tmax: int, HD: int, dev, dt=torch.bfloat16):
        cap = max(256, -(-int(Tmax) // 256) * 256)
        self.buf = torch.empty(2, B, HKV, cap, HD, device=dev, dtype=dt)
        self.n = 0

    @property
    def k(self) -> torch.Tensor:
        return self.buf[0]

    @property
    def v(self) -> torch.Tensor:
        return self.buf[1]

    @property
    def capacity(self) -> int:
        return self.buf.shape[3]

    def reserve(self, L: int) -> None:
        """Room for L more tokens: the capacity doubles (one copy of the held tokens) until they fit."""
        if self.n + L > self.capacity:
            cap = self.capacity
            while cap < self.n + L:
                cap *= 2
            grown = torch.empty(*self.buf.shape[:3], cap, self.buf.shape[4], device=self.buf.device,
                                dtype=self.buf.dtype)
            grown[:, :, :, :self.n].copy_(self.buf[:, :, :, :self.n])
            self.buf = grown

    def append(self, k_new: torch.Tensor, v_new: torch.Tensor):
        """Write L new keys/values [B, HKV, L, HD] after the held ones; returns views of all n."""
        L = k_new.shape[2]
        self.reserve(L)
        self.buf[0, :, :, self.n:self.n + L].copy_(k_new)
        self.buf[1, :, :, self.n:self.n + L].copy_(v_new)
        self.n += L
        return self.buf[0, :, :, :self.n], self.buf[1, :, :, :self.n]


class _ChunkGraph:
    """A one-token decode step captured into a CUDA graph at the first position it serves and
    replayed for every later position of the same chunk. Every launch of such a step is the same
    within a chunk except for the token position, which the kernels read from the device
    (K.DevicePosition); a new chunk (the window slots change) takes a new capture. The host
    bookkeeping, and a chunk boundary's consolidation, run eagerly after each replay. Subclasses
    give the step's body, what it needs allocated before a capture, and its bookkeeping."""

    def __init__(self, device, C: int):
        self.device, self.C = torch.device(device), C
        self.pos = K.DevicePosition(self.device)
        self.graph, self.out = None, None
        self.lo = self.hi = -1            # positions the current graph serves
        self.next = None                  # the position the host state expects next
        self.captures = 0

    def _phase(self) -> int: ...
    def _prepare(self, span: int) -> None: ...
    def _body(self, pos: int) -> torch.Tensor: ...
    def _advance(self, pos: int) -> None: ...

    @K.traced("DecodeGraph.capture")
    def _capture(self, pos: int) -> None:
        self.graph = self.out = None      # the previous graph and its private memory are released
        span = self.C - self._phase()
        self._prepare(span)               # everything the captured launches point at exists first
        self.pos.ref, self.pos.span = pos, span
        self.pos.set(pos)
        if self.captures == 0:
            # first capture: one eager run of the same launches initialises the libraries' lazy state
            # (it rewrites exactly what the replay below writes: this step's window and cache rows)
            self._body(pos)
        # captured on a side stream that joins the current one; torch.cuda.graph() would also run a
        # garbage collection and empty the allocator cache at every capture, once per chunk here
        main = torch.cuda.current_stream()
        side = self._side = getattr(self, "_side", None) or torch.cuda.Stream(self.device)
        side.wait_stream(main)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            g.capture_begin()
            try:
                self.out = self._body(pos)
            finally:
                g.capture_end()
        main.wait_stream(side)
        self.graph, self.lo, self.hi = g, pos, pos + span
        self.captures += 1

    def close(self) -> None:
        """Release the captured graph (and its memory). A graph that holds NCCL collectives (a
        tensor-parallel decoder's) must be released before its process group is destroyed."""
        self.graph = self.out = None
        self.lo = self.hi = -1

    @K.traced("DecodeGraph.replay")
    def _replay(self, pos: int) -> torch.Tensor:
        if self.next is not None and pos != self.next:
            raise ValueError(f"decode steps must be consecutive: expected position {self.next}, got {pos}")
        if self.graph is None or not (self.lo <= pos < self.hi):
            self._capture(pos)
        self.pos.set(pos)
        self.graph.replay()
        self._advance(pos)
        self.next = pos + 1
        return self.out


def _ensure_step_plan(ly: Bolt3Attn, st: Bolt3LayerState, device) -> None:
    f = ly.fused(device)
    plan = st._plans.get(1)
    if plan is None or plan.key != f.key:
        st._plans[1] = Bolt3Decoder._step_plan(ly, st, st.B, 1, f, device)


class DecodeGraph(_ChunkGraph):
    """One-token decode steps of a Bolt3Decoder (or Bolt3DecoderTP) replayed from CUDA graphs.

    A step of the hybrid model is hundreds of kernel launches (36 layers of norms, GEMMs, the Bolt-3
    prep / attention / o_proj, the anchors' attention, the MLP), more host time than GPU time at
    decode sizes; replayed, the step costs the host one graph launch. Results equal step()'s.
    step() returns a static buffer that the next step overwrites."""

    def __init__(self, dec: "Bolt3Decoder", states, kv_caches):
        bolt = [st for st in kv_caches if isinstance(st, Bolt3LayerState)]
        anch = [c for c in kv_caches if isinstance(c, AnchorKV)]
        ref = bolt[0].ring_kp if bolt else anch[0].buf
        super().__init__(ref.device, dec.C)
        self.dec, self.states, self.kv = dec, states, kv_caches
        self.B = bolt[0].B if bolt else anch[0].buf.shape[1]
        self.tok = torch.zeros(self.B, 1, dtype=torch.long, device=self.device)

    def _phase(self) -> int:
        lens = {st.cur_len for st in self.kv if isinstance(st, Bolt3LayerState)}
        if len(lens) > 1:
            raise RuntimeError("the Bolt-3 layers of a decode state are at different chunk phases")
        return lens.pop() if lens else 0

    def _prepare(self, span: int) -> None:
        for li, blk in enumerate(self.dec.model.blocks):
            if hasattr(blk, "vsa"):
                _ensure_step_plan(blk.vsa, self.kv[li], self.device)
            else:
                self.kv[li].reserve(span)

    def _body(self, pos: int) -> torch.Tensor:
        return self.dec._blocks(self.tok, pos, self.states, self.kv, dev_pos=self.pos)

    def _advance(self, pos: int) -> None:
        self.dec._advance(1, pos, self.states, self.kv)

    @torch.no_grad()
    def step(self, tokens: torch.Tensor, pos: int) -> torch.Tensor:
        """One token per sequence ([B, 1] ids on the device) at position pos; the final normed hidden
        states [B, 1, D] (a static buffer). While a layer's window holds a chunk of more than C
        tokens (after an unaligned prompt slice) the steps run eagerly."""
        if any(isinstance(st, Bolt3LayerState) and st.big_prev is not None for st in self.kv):
            if self.next is not None and pos != self.next:
                raise ValueError(f"decode steps must be consecutive: expected position {self.next}, got {pos}")
            self.graph = self.out = None
            h, _, _ = self.dec.step(tokens, pos, self.states, self.kv)
            self.next = pos + 1
            return h
        self.tok.copy_(tokens)
        return self._replay(pos)


# the reference's name for the anchor-layer cache class (vsa_lm/decode.py:88)
StaticKV = AnchorKV
