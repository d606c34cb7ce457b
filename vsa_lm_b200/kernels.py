"""Torch-facing wrappers of the Bolt-3 C-ABI: check devices, dtypes and contiguity, pass raw pointers
and the current CUDA stream. PyTorch only provides device memory and streams here; every kernel is
in libbolt3.so. Nothing here falls back to a CPU or PyTorch implementation.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

S_SLOTS = 128
CHUNK = 128
N_SINKS = 4


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


# Kernel launches issued through this module (C-ABI calls that returned BOLT3_OK), for bench.py's
# gpu_launches count.
_launches = 0


def launch_count() -> int:
    return _launches


def _count(n: int) -> None:
    global _launches
    _launches += n


def _need(t: torch.Tensor, dtype: torch.dtype, name: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (the Bolt-3 path has no CPU implementation)")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def n_consolidations(T: int, C: int = CHUNK) -> int:
    """Consolidations Bolt3Attn.forward runs for T tokens (vsa_lm/config/bolt3.py:262)."""
    full = T // C
    return max(0, full - 2) if T % C == 0 else max(0, full - 1)


def prep(proj: torch.Tensor, *, B: int, T: int, H: int, HKV: int, HD: int, inv_freq: torch.Tensor,
         eps: float, q_norm_w: torch.Tensor | None, k_norm_w: torch.Tensor | None, pos0: int,
         cols: dict, parts: int = 3, q_raw=None, q_rope=None, eta=None, k_raw=None, k_rope=None, v=None,
         beta=None, q_head_stride: int = 0, q_t_off: int = 0, k_head_stride: int = 0, k_t_off: int = 0,
         q_l2: torch.Tensor | None = None) -> None:
    """RMSNorm/RoPE/gates from a projection output into head-major buffers (bolt3_prep). `cols` gives
    the column offsets q_col, k_col, v_col, beta_col, eta_col of the sections in `proj`; `parts`
    selects q/eta (1), k/v/beta (2) or both (3). `q_l2` (optional, laid out like eta) receives
    |q_raw| per row."""
    lib = _lib.load()
    _need(proj, torch.bfloat16, "proj")
    outs = []
    if parts & 1:
        outs += [("q_raw", q_raw, torch.bfloat16), ("q_rope", q_rope, torch.bfloat16), ("eta", eta, torch.float32)]
    if parts & 2:
        outs += [("k_raw", k_raw, torch.bfloat16), ("k_rope", k_rope, torch.bfloat16), ("v", v, torch.bfloat16),
                 ("beta", beta, torch.float32)]
    for name, t, dt in outs:
        _need(t, dt, name)
    _need(inv_freq, torch.float32, "inv_freq")
    a = _lib.PrepArgs(
        proj=proj.data_ptr(), ld=proj.stride(0), B=B, T=T, H=H, HKV=HKV, HD=HD,
        q_norm_w=_ptr(q_norm_w), k_norm_w=_ptr(k_norm_w), eps=eps, inv_freq=inv_freq.data_ptr(),
        pos0=pos0, q_raw=_ptr(q_raw), q_rope=_ptr(q_rope), q_head_stride=q_head_stride,
        q_t_off=q_t_off, eta=_ptr(eta), eta_head_stride=q_head_stride, eta_t_off=q_t_off,
        k_raw=_ptr(k_raw), k_rope=_ptr(k_rope), v=_ptr(v), k_head_stride=k_head_stride,
        k_t_off=k_t_off, beta=_ptr(beta), beta_head_stride=k_head_stride, beta_t_off=k_t_off,
        q_l2=_ptr(q_l2), parts=parts, q_col=cols.get("q_col", 0), k_col=cols.get("k_col", 0),
        v_col=cols.get("v_col", 0), beta_col=cols.get("beta_col", 0), eta_col=cols.get("eta_col", 0))
    _lib.check(lib.bolt3_prep(ctypes.byref(a), _stream()), "bolt3_prep")
    _count(1)


def consolidate(*, n_chains: int, hkv: int, HD: int, bank: dict, init_blank: bool,
                kr: torch.Tensor, kp: torch.Tensor, v: torch.Tensor, beta: torch.Tensor,
                chain_tokens: int, token0: int, step_tokens: int, skip0: int, chunk_len: int,
                pos0: int, n_steps: int, kappa: torch.Tensor, gamma: torch.Tensor,
                inv_freq: torch.Tensor, snaps: dict | None = None, snap0: int = 0,
                status: torch.Tensor | None = None) -> None:
    """Run n_steps consolidations on every chain (bolt3_consolidate). `bank` holds the state
    tensors ak, av, ak_rope (bf16 [chains,S,HD]), mass, util, pm (fp32 [chains,S]), act (uint8),
    m_res (fp32 [chains,HD,HD]) and n_filled (int32 [chains]); they are updated in place."""
    lib = _lib.load()
    snaps = snaps or {}
    a = _lib.ConsolidateArgs(
        n_chains=n_chains, hkv=hkv, HD=HD,
        ak=bank["ak"].data_ptr(), av=bank["av"].data_ptr(), ak_rope=_ptr(bank.get("ak_rope")),
        mass=bank["mass"].data_ptr(), util=bank["util"].data_ptr(), pm=bank["pm"].data_ptr(),
        act=bank["act"].data_ptr(), m_res=bank["m_res"].data_ptr(), n_filled=bank["n_filled"].data_ptr(),
        init_blank=int(init_blank), kr=kr.data_ptr(), kp=kp.data_ptr(), v=v.data_ptr(), beta=beta.data_ptr(),
        chain_tokens=chain_tokens, token0=token0, step_tokens=step_tokens, skip0=skip0,
        chunk_len=chunk_len, pos0=pos0, n_steps=n_steps, kappa=kappa.data_ptr(), gamma=gamma.data_ptr(),
        inv_freq=inv_freq.data_ptr(),
        snap_ak_rope=_ptr(snaps.get("ak_rope")), snap_av=_ptr(snaps.get("av")),
        snap_mass=_ptr(snaps.get("mass")), snap_act=_ptr(snaps.get("act")), snap_m=_ptr(snaps.get("m")),
        snap_cap=int(snaps["ak_rope"].shape[1]) if snaps else 0, snap0=snap0, status=_ptr(status))
    _lib.check(lib.bolt3_consolidate(ctypes.byref(a), _stream()), "bolt3_consolidate")
    _count(1 if a.n_steps > 0 else 0)


def attend_decode(*, n_chains: int, hkv: int, G: int, HD: int, q_rope: torch.Tensor, q_raw: torch.Tensor,
                  eta: torch.Tensor, Tq: int, seg0_k: torch.Tensor, seg0_v: torch.Tensor,
                  seg0_chain_tokens: int, seg0_len: int, seg1_k: torch.Tensor, seg1_v: torch.Tensor,
                  seg1_chain_tokens: int, seg1_len: int, len_before: int,
                  sinks: tuple | None, bank: dict | None, kappa: torch.Tensor, coef: torch.Tensor,
                  res_w: torch.Tensor, eps: float, y: torch.Tensor, q_l2: torch.Tensor | None = None) -> None:
    """Attention of Tq new tokens over sinks, the current bank and the two-chunk window."""
    lib = _lib.load()
    a = _lib.AttendArgs(
        n_chains=n_chains, hkv=hkv, G=G, HD=HD, q_rope=q_rope.data_ptr(), q_raw=q_raw.data_ptr(),
        eta=eta.data_ptr(), Tq=Tq, prefill=0,
        seg0_k=seg0_k.data_ptr(), seg0_v=seg0_v.data_ptr(), seg0_chain_tokens=seg0_chain_tokens,
        seg0_len=seg0_len, seg1_k=seg1_k.data_ptr(), seg1_v=seg1_v.data_ptr(),
        seg1_chain_tokens=seg1_chain_tokens, seg1_len=seg1_len, len_before=len_before,
        sink_k=_ptr(sinks[0]) if sinks else None, sink_v=_ptr(sinks[1]) if sinks else None,
        sink_chain_tokens=N_SINKS, has_sinks=int(sinks is not None),
        bank_ak_rope=_ptr(bank["ak_rope"]) if bank else None, bank_av=_ptr(bank["av"]) if bank else None,
        bank_mass=_ptr(bank["mass"]) if bank else None, bank_act=_ptr(bank["act"]) if bank else None,
        bank_m=_ptr(bank["m_res"]) if bank else None, bank_cap=1, has_bank=int(bank is not None),
        kappa=kappa.data_ptr(), coef=coef.data_ptr(), res_w=res_w.data_ptr(), eps=eps,
        y=y.data_ptr(), y_tokens=Tq, q_l2=_ptr(q_l2))
    _lib.check(lib.bolt3_attend(ctypes.byref(a), _stream()), "bolt3_attend")
    _count(1)


class DecodeStepArgs:
    """The decoder's per-step bolt3_prep and bolt3_attend argument blocks, built once for a (layer,
    state, step size) and launched every step with only the fields that move rewritten: the
    projection output, RoPE position and ring write offset (prep), the ring slots, window lengths and
    whether sinks and a bank exist yet (attend). The buffers the blocks point at are the caller's
    and must stay alive."""

    def __init__(self, prep_fields: dict, attend_fields: dict):
        self.lib = _lib.load()
        self.prep = _lib.PrepArgs(**prep_fields)
        self.attend = _lib.AttendArgs(**attend_fields)

    def launch_prep(self, proj: torch.Tensor, pos0: int, k_t_off: int) -> None:
        a = self.prep
        if proj.stride(0) != a.ld or not proj.is_contiguous():
            raise ValueError("proj must be a contiguous [tokens, ld] projection output")
        a.proj, a.pos0, a.k_t_off, a.beta_t_off = proj.data_ptr(), pos0, k_t_off, k_t_off
        _lib.check(self.lib.bolt3_prep(ctypes.byref(a), _stream()), "bolt3_prep")
        _count(1)

    def launch_attend(self, *, seg0_k: int, seg0_v: int, seg0_len: int, seg1_k: int, seg1_v: int,
                      seg1_len: int, len_before: int, has_sinks: bool, has_bank: bool, bank_m: int) -> None:
        a = self.attend
        a.seg0_k, a.seg0_v, a.seg0_len = seg0_k, seg0_v, seg0_len
        a.seg1_k, a.seg1_v, a.seg1_len, a.len_before = seg1_k, seg1_v, seg1_len, len_before
        a.has_sinks, a.has_bank, a.bank_m = int(has_sinks), int(has_bank), bank_m
        _lib.check(self.lib.bolt3_attend(ctypes.byref(a), _stream()), "bolt3_attend")
        _count(1)


def prefill_workspace_bytes(n_chains: int, T: int, HD: int) -> int:
    return int(_lib.load().bolt3_prefill_workspace_size(n_chains, T, HD))


def snapshot_views(ws: torch.Tensor, n_chains: int, n_cons: int, HD: int, S: int = S_SLOTS) -> dict:
    """Views of a prefill workspace as the consolidation snapshots, at the offsets
    bolt3_prefill_fwd uses: ak_rope / av images, mass, act, and the split M_res image."""
    ns = n_chains * n_cons
    off = 0
    views = {}
    for name, nbytes in (("ak_rope", ns * S * HD * 2), ("av", ns * S * HD * 2), ("mass", ns * S * 4),
                         ("act", ns * S), ("m", ns * HD * HD * 4)):
        views[name] = ws[off:off + nbytes]
        off = (off + nbytes + 255) // 256 * 256
    views["ak_rope"] = views["ak_rope"].view(torch.bfloat16).view(n_chains, n_cons, S, HD)
    views["av"] = views["av"].view(torch.bfloat16).view(n_chains, n_cons, S, HD)
    views["mass"] = views["mass"].view(torch.float32)
    views["m"] = views["m"].view(torch.float32)
    return views


def attend_prefill(*, n_chains: int, hkv: int, G: int, HD: int, T: int, q_rope, q_raw, eta, k_rope, v,
                   snaps: dict | None, n_cons: int, kappa, coef, res_w, eps: float, y: torch.Tensor,
                   blk_begin: int = 0, blk_count: int = 0, q_l2=None, status=None) -> None:
    """Attention of prefill query blocks [blk_begin, blk_begin + blk_count) (bolt3_attend, prefill
    mode): chunk r reads snapshot r - 2 of the consolidation scan."""
    lib = _lib.load()
    sn = snaps or {}
    a = _lib.AttendArgs(
        n_chains=n_chains, hkv=hkv, G=G, HD=HD, q_rope=q_rope.data_ptr(), q_raw=q_raw.data_ptr(),
        eta=eta.data_ptr(), Tq=T, prefill=1, seg0_k=k_rope.data_ptr(), seg0_v=v.data_ptr(),
        seg0_chain_tokens=T, seg1_k=k_rope.data_ptr(), seg1_v=v.data_ptr(), seg1_chain_tokens=T,
        bank_ak_rope=_ptr(sn.get("ak_rope")), bank_av=_ptr(sn.get("av")), bank_mass=_ptr(sn.get("mass")),
        bank_act=_ptr(sn.get("act")), bank_m=_ptr(sn.get("m")), bank_cap=n_cons,
        kappa=kappa.data_ptr(), coef=coef.data_ptr(), res_w=res_w.data_ptr(), eps=eps,
        y=y.data_ptr(), y_tokens=T, status=_ptr(status), q_l2=_ptr(q_l2), blk_begin=blk_begin,
        blk_count=blk_count)
    _lib.check(lib.bolt3_attend(ctypes.byref(a), _stream()), "bolt3_attend")
    _count(1)


def prefill(*, B: int, T: int, H: int, HKV: int, HD: int, q_rope, q_raw, eta, k_raw, k_rope, v, beta,
            kappa, gamma, coef, inv_freq, res_w, eps: float, workspace: torch.Tensor, bank: dict,
            y: torch.Tensor, status: torch.Tensor | None = None, q_l2: torch.Tensor | None = None) -> None:
    """Phases B + C of Bolt3Attn.forward on prepared q/k/v (bolt3_prefill_fwd)."""
    lib = _lib.load()
    a = _lib.PrefillArgs(
        B=B, T=T, H=H, HKV=HKV, HD=HD, q_rope=q_rope.data_ptr(), q_raw=q_raw.data_ptr(),
        eta=eta.data_ptr(), k_raw=k_raw.data_ptr(), k_rope=k_rope.data_ptr(), v=v.data_ptr(),
        beta=beta.data_ptr(), kappa=kappa.data_ptr(), gamma=gamma.data_ptr(), coef=coef.data_ptr(),
        inv_freq=inv_freq.data_ptr(), res_w=res_w.data_ptr(), eps=eps,
        workspace=workspace.data_ptr(), workspace_bytes=workspace.numel() * workspace.element_size(),
        ak=bank["ak"].data_ptr(), av=bank["av"].data_ptr(), ak_rope=_ptr(bank.get("ak_rope")),
        mass=bank["mass"].data_ptr(), util=bank["util"].data_ptr(), pm=bank["pm"].data_ptr(),
        act=bank["act"].data_ptr(), m_res=bank["m_res"].data_ptr(), n_filled=bank["n_filled"].data_ptr(),
        y=y.data_ptr(), status=_ptr(status), q_l2=_ptr(q_l2))
    _lib.check(lib.bolt3_prefill_fwd(ctypes.byref(a), _stream()), "bolt3_prefill_fwd")
    _count(2)  # the scan, then the attention


def prefill_noalloc(*, B: int, T: int, H: int, HKV: int, HD: int, q_rope, q_raw, eta, k_raw, k_rope, v, beta,
                    kappa, gamma, coef, inv_freq, res_w, eps: float, bank: dict, y: torch.Tensor,
                    status: torch.Tensor | None = None, q_l2: torch.Tensor | None = None) -> None:
    """Phases B + C like `prefill`, with the snapshot workspace taken from the library's fixed
    per-GPU array instead of the caller (bolt3_prefill_fwd_noalloc). For hosts that cannot allocate
    device memory on their hot path; the work must fit in `_lib.NOALLOC_SCRATCH_BYTES`."""
    lib = _lib.load()
    need = prefill_workspace_bytes(B * HKV, T, HD)
    if need > _lib.NOALLOC_SCRATCH_BYTES:
        raise ValueError(f"prefill of {B} x {T} tokens needs {need} bytes of scratch; the no-alloc entry point "
                         f"has a fixed {_lib.NOALLOC_SCRATCH_BYTES} bytes (use `prefill` with a workspace)")
    a = _lib.PrefillArgs(
        B=B, T=T, H=H, HKV=HKV, HD=HD, q_rope=q_rope.data_ptr(), q_raw=q_raw.data_ptr(),
        eta=eta.data_ptr(), k_raw=k_raw.data_ptr(), k_rope=k_rope.data_ptr(), v=v.data_ptr(),
        beta=beta.data_ptr(), kappa=kappa.data_ptr(), gamma=gamma.data_ptr(), coef=coef.data_ptr(),
        inv_freq=inv_freq.data_ptr(), res_w=res_w.data_ptr(), eps=eps, workspace=None, workspace_bytes=0,
        ak=bank["ak"].data_ptr(), av=bank["av"].data_ptr(), ak_rope=_ptr(bank.get("ak_rope")),
        mass=bank["mass"].data_ptr(), util=bank["util"].data_ptr(), pm=bank["pm"].data_ptr(),
        act=bank["act"].data_ptr(), m_res=bank["m_res"].data_ptr(), n_filled=bank["n_filled"].data_ptr(),
        y=y.data_ptr(), status=_ptr(status), q_l2=_ptr(q_l2))
    _lib.check(lib.bolt3_prefill_fwd_noalloc(ctypes.byref(a), _stream()), "bolt3_prefill_fwd_noalloc")
    _count(2)


def new_bank(n_chains: int, HD: int, device, S: int = S_SLOTS) -> dict:
    """Uninitialised bank tensors (the consolidation kernel initialises them with init_blank)."""
    bf = dict(dtype=torch.bfloat16, device=device)
    f32 = dict(dtype=torch.float32, device=device)
    return dict(ak=torch.empty(n_chains, S, HD, **bf), av=torch.empty(n_chains, S, HD, **bf),
                ak_rope=torch.empty(n_chains, S, HD, **bf), mass=torch.empty(n_chains, S, **f32),
                util=torch.empty(n_chains, S, **f32), pm=torch.empty(n_chains, S, **f32),
                act=torch.zeros(n_chains, S, dtype=torch.uint8, device=device),
                m_res=torch.zeros(n_chains, HD, HD, **f32),
                n_filled=torch.zeros(n_chains, dtype=torch.int32, device=device))
