"""Torch-facing wrappers of the Bolt-3 C-ABI: check devices, dtypes, layouts and sizes, pass raw
pointers and the current CUDA stream. PyTorch only provides device memory and streams here; every
kernel is in libbolt3.so. Nothing here falls back to a CPU or PyTorch implementation.

The C side cannot tell a host pointer from a device pointer, nor a tensor of the current device
from one on another GPU, so every tensor argument is checked here before its address is passed:
a CPU tensor, a tensor on a device other than the current one, the wrong dtype, a non-contiguous
view or too few elements raise before anything is launched.
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


def traced(name: str):
    """Decorator: run the function inside an NVTX range `name` (torch.cuda.nvtx, NVTX's default
    domain, the one the C-ABI entry points write their own ranges to, so they nest). With no
    profiler attached a push or pop costs a fraction of a microsecond."""
    import functools
    from torch.cuda import nvtx

    def wrap(fn):
        @functools.wraps(fn)
        def run(*args, **kwargs):
            nvtx.range_push(name)
            try:
                return fn(*args, **kwargs)
            finally:
                nvtx.range_pop()
        return run
    return wrap


def _need(t: torch.Tensor, dtype: torch.dtype, name: str, numel: int | None = None) -> None:
    """`t` is a contiguous `dtype` tensor on the current CUDA device holding at least `numel`
    elements (when given)."""
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor, got {type(t).__name__}")
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (the Bolt-3 path has no CPU implementation)")
    cur = torch.cuda.current_device()
    if t.device.index != cur:
        raise RuntimeError(f"{name} is on {t.device}, but the current device is cuda:{cur}; the kernels are "
                           f"launched on the current device")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if numel is not None and t.numel() < numel:
        raise ValueError(f"{name} holds {t.numel()} elements; the described work needs {numel}")


def _need_rows(t: torch.Tensor, name: str, n_chains: int, chain_tokens: int, length: int, HD: int) -> None:
    """`t` holds bf16 rows of HD values, chain_tokens rows per chain, and the kernel reads rows
    [0, length) of each of n_chains chains from t's first element. `t` may be a view into a larger
    buffer (a window ring slot): its rows must be dense, consecutive chains chain_tokens rows apart,
    and every row read must lie inside t's storage."""
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (the Bolt-3 path has no CPU implementation)")
    cur = torch.cuda.current_device()
    if t.device.index != cur:
        raise RuntimeError(f"{name} is on {t.device}, but the current device is cuda:{cur}")
    if t.dtype != torch.bfloat16:
        raise TypeError(f"{name} must be torch.bfloat16, got {t.dtype}")
    if length < 0 or length > chain_tokens:
        raise ValueError(f"{name}: {length} rows in a segment of {chain_tokens} rows per chain")
    if t.dim() < 2 or t.shape[-1] != HD or t.stride(-1) != 1 or (t.shape[-2] > 1 and t.stride(-2) != HD):
        raise ValueError(f"{name} must hold dense rows of {HD} values")
    if t.dim() == 3 and t.shape[0] > 1 and t.stride(0) != chain_tokens * HD:
        raise ValueError(f"{name}: chains must be {chain_tokens} rows apart")
    if length > 0:
        end = t.storage_offset() + ((n_chains - 1) * chain_tokens + length) * HD
        if end * t.element_size() > t.untyped_storage().nbytes():
            raise ValueError(f"{name}: the rows read run past the tensor's storage")


def _opt(t: torch.Tensor | None, dtype: torch.dtype, name: str, numel: int | None = None) -> None:
    if t is not None:
        _need(t, dtype, name, numel)


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def n_consolidations(T: int, C: int = CHUNK) -> int:
    """Consolidations Bolt3Attn.forward runs for T tokens (vsa_lm/config/bolt3.py:262)."""
    full = T // C
    return max(0, full - 2) if T % C == 0 else max(0, full - 1)


class DeviceStatus:
    """The device status word the kernels OR error bits into (include/bolt3.h), and its host side.

    `word` is one int32 on the device, passed as `status` to every kernel call. `arm()` enqueues an
    asynchronous copy of it into pinned host memory on the current stream, behind the kernels just
    launched, and records an event. `check(block)` reads that copy once the event has completed
    (waiting for it when `block`) and raises RuntimeError if any bit is set, clearing the word so
    that later calls start clean. Nothing here synchronises unless `block` is true."""

    def __init__(self, device):
        self.word = torch.zeros(1, dtype=torch.int32, device=device)
        self.host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self.event = None
        self.what = ""

    def arm(self, what: str) -> None:
        self.host.copy_(self.word, non_blocking=True)
        self.event = torch.cuda.Event()
        self.event.record()
        self.what = what

    def check(self, block: bool = False) -> None:
        ev = self.event
        if ev is None:
            return
        if block:
            ev.synchronize()
        elif not ev.query():
            return
        self.event = None
        bits = int(self.host[0])
        if bits:
            self.word.zero_()
            why = "; ".join(msg for b, msg in _lib.DEVICE_STATUS_BITS.items() if bits & b) or "unknown bits"
            raise RuntimeError(f"{self.what}: device status {bits:#x} ({why}); the outputs of that call are invalid")


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
    if proj.dim() != 2 or proj.shape[0] < B * T:
        raise ValueError(f"proj must be [tokens >= {B * T}, ld], got {tuple(proj.shape)}")
    outs = []
    q_rows = B * H * (q_head_stride if q_head_stride else T)
    k_rows = B * HKV * (k_head_stride if k_head_stride else T)
    if parts & 1:
        outs += [("q_raw", q_raw, torch.bfloat16, q_rows * HD), ("q_rope", q_rope, torch.bfloat16, q_rows * HD),
                 ("eta", eta, torch.float32, q_rows)]
    if parts & 2:
        outs += [("k_raw", k_raw, torch.bfloat16, k_rows * HD), ("k_rope", k_rope, torch.bfloat16, k_rows * HD),
                 ("v", v, torch.bfloat16, k_rows * HD), ("beta", beta, torch.float32, k_rows)]
    for name, t, dt, n in outs:
        _need(t, dt, name, n)
    _need(inv_freq, torch.float32, "inv_freq", HD // 2)
    _opt(q_norm_w, torch.float32, "q_norm_w", HD)
    _opt(k_norm_w, torch.float32, "k_norm_w", HD)
    _opt(q_l2, torch.float32, "q_l2", q_rows)
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


def check_bank(bank: dict, n_chains: int, HD: int, S: int = S_SLOTS) -> None:
    """The state tensors of n_chains chains (new_bank's layout)."""
    bf, f32 = torch.bfloat16, torch.float32
    _need(bank["ak"], bf, "bank ak", n_chains * S * HD)
    _need(bank["av"], bf, "bank av", n_chains * S * HD)
    if bank.get("ak_rope") is not None:
        _need(bank["ak_rope"], bf, "bank ak_rope", n_chains * S * HD)
    for k in ("mass", "util", "pm"):
        _need(bank[k], f32, "bank " + k, n_chains * S)
    _need(bank["act"], torch.uint8, "bank act", n_chains * S)
    _need(bank["m_res"], f32, "bank m_res", n_chains * HD * HD)
    _need(bank["n_filled"], torch.int32, "bank n_filled", n_chains)


def _status(status) -> int | None:
    if status is None:
        return None
    if isinstance(status, DeviceStatus):
        status = status.word
    _need(status, torch.int32, "status", 1)
    return status.data_ptr()


def _check_snaps(sn: dict, n_chains: int, n_cons: int, HD: int) -> None:
    ns = n_chains * n_cons
    _need(sn["ak_rope"], torch.bfloat16, "snapshot ak_rope", ns * S_SLOTS * HD)
    _need(sn["av"], torch.bfloat16, "snapshot av", ns * S_SLOTS * HD)
    _need(sn["mass"], torch.float32, "snapshot mass", ns * S_SLOTS)
    _need(sn["act"], torch.uint8, "snapshot act", ns * S_SLOTS)
    _need(sn["m"], torch.float32, "snapshot M_res", ns * HD * HD)


def consolidate(*, n_chains: int, hkv: int, HD: int, bank: dict, init_blank: bool,
                kr: torch.Tensor, kp: torch.Tensor, v: torch.Tensor, beta: torch.Tensor,
                chain_tokens: int, token0: int, step_tokens: int, skip0: int, chunk_len: int,
                pos0: int, n_steps: int, kappa: torch.Tensor, gamma: torch.Tensor,
                inv_freq: torch.Tensor, snaps: dict | None = None, snap0: int = 0,
                status=None, wait_probe: int = 0) -> None:
    """Run n_steps consolidations on every chain (bolt3_consolidate). `bank` holds the state
    tensors ak, av, ak_rope (bf16 [chains,S,HD]), mass, util, pm (fp32 [chains,S]), act (uint8),
    m_res (fp32 [chains,HD,HD]) and n_filled (int32 [chains]); they are updated in place.
    `status`: a DeviceStatus or a device int32 tensor the kernel ORs error bits into."""
    lib = _lib.load()
    snaps = snaps or {}
    check_bank(bank, n_chains, HD)
    for name, t in (("kr", kr), ("kp", kp), ("v", v)):
        _need(t, torch.bfloat16, name, n_chains * chain_tokens * HD)
    _need(beta, torch.float32, "beta", n_chains * chain_tokens)
    _need(kappa, torch.float32, "kappa", hkv)
    _need(gamma, torch.float32, "gamma", hkv)
    _need(inv_freq, torch.float32, "inv_freq", HD // 2)
    snap_cap = 0
    if snaps:
        snap_cap = int(snaps["ak_rope"].shape[1])
        _check_snaps(snaps, n_chains, snap_cap, HD)
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
        snap_cap=snap_cap, snap0=snap0, status=_status(status), wait_probe=wait_probe)
    _lib.check(lib.bolt3_consolidate(ctypes.byref(a), _stream()), "bolt3_consolidate")
    _count(1 if a.n_steps > 0 else 0)


def attend_decode(*, n_chains: int, hkv: int, G: int, HD: int, q_rope: torch.Tensor, q_raw: torch.Tensor,
                  eta: torch.Tensor, Tq: int, seg0_k: torch.Tensor, seg0_v: torch.Tensor,
                  seg0_chain_tokens: int, seg0_len: int, seg1_k: torch.Tensor, seg1_v: torch.Tensor,
                  seg1_chain_tokens: int, seg1_len: int, len_before: int,
                  sinks: tuple | None, bank: dict | None, kappa: torch.Tensor, coef: torch.Tensor,
                  res_w: torch.Tensor, eps: float, y: torch.Tensor, q_l2: torch.Tensor | None = None,
                  status=None, wait_probe: int = 0) -> None:
    """Attention of Tq new tokens over sinks, the current bank and the two-chunk window."""
    lib = _lib.load()
    nq = n_chains * G * Tq
    _need(q_rope, torch.bfloat16, "q_rope", nq * HD)
    _need(q_raw, torch.bfloat16, "q_raw", nq * HD)
    _need(eta, torch.float32, "eta", nq)
    _opt(q_l2, torch.float32, "q_l2", nq)
    _need(y, torch.bfloat16, "y", nq * HD)
    for name, t, ct, ln in (("seg0_k", seg0_k, seg0_chain_tokens, seg0_len),
                            ("seg0_v", seg0_v, seg0_chain_tokens, seg0_len),
                            ("seg1_k", seg1_k, seg1_chain_tokens, seg1_len),
                            ("seg1_v", seg1_v, seg1_chain_tokens, seg1_len)):
        _need_rows(t, name, n_chains, ct, ln, HD)
    if sinks:
        _need(sinks[0], torch.bfloat16, "sink_k", n_chains * N_SINKS * HD)
        _need(sinks[1], torch.bfloat16, "sink_v", n_chains * N_SINKS * HD)
    if bank:
        _need(bank["ak_rope"], torch.bfloat16, "bank ak_rope", n_chains * S_SLOTS * HD)
        _need(bank["av"], torch.bfloat16, "bank av", n_chains * S_SLOTS * HD)
        _need(bank["mass"], torch.float32, "bank mass", n_chains * S_SLOTS)
        _need(bank["act"], torch.uint8, "bank act", n_chains * S_SLOTS)
        _need(bank["m_res"], torch.float32, "bank m_res", n_chains * HD * HD)
    _need(kappa, torch.float32, "kappa", hkv)
    _need(coef, torch.float32, "coef", hkv)
    _need(res_w, torch.float32, "res_w", HD)
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
        y=y.data_ptr(), y_tokens=Tq, q_l2=_ptr(q_l2), status=_status(status), wait_probe=wait_probe)
    _lib.check(lib.bolt3_attend(ctypes.byref(a), _stream()), "bolt3_attend")
    _count(1)


class DecodeStepArgs:
    """The decoder's per-step bolt3_prep and bolt3_attend argument blocks, built once for a (layer,
    state, step size) and launched every step with only the fields that move rewritten: the
    projection output, RoPE position and ring write offset (prep), the ring slots, window lengths and
    whether sinks and a bank exist yet (attend). The buffers the blocks point at are the caller's
    and must stay alive; they belong to the plan and state that built the blocks."""

    def __init__(self, prep_fields: dict, attend_fields: dict):
        self.lib = _lib.load()
        self.prep = _lib.PrepArgs(**prep_fields)
        self.attend = _lib.AttendArgs(**attend_fields)

    def launch_prep(self, proj: torch.Tensor, pos0: int, k_t_off: int, dev_pos: "DevicePosition | None" = None) -> None:
        a = self.prep
        _need(proj, torch.bfloat16, "proj", a.B * a.T * a.ld)
        if proj.stride(0) != a.ld:
            raise ValueError("proj must be a contiguous [tokens, ld] projection output")
        a.proj, a.pos0, a.k_t_off, a.beta_t_off = proj.data_ptr(), pos0, k_t_off, k_t_off
        _set_dev_pos(a, dev_pos)
        _lib.check(self.lib.bolt3_prep(ctypes.byref(a), _stream()), "bolt3_prep")
        _count(1)

    def launch_attend(self, *, seg0_k: int, seg0_v: int, seg0_len: int, seg1_k: int, seg1_v: int,
                      seg1_len: int, len_before: int, has_sinks: bool, has_bank: bool, bank_m: int,
                      dev_pos: "DevicePosition | None" = None) -> None:
        a = self.attend
        a.seg0_k, a.seg0_v, a.seg0_len = seg0_k, seg0_v, seg0_len
        a.seg1_k, a.seg1_v, a.seg1_len, a.len_before = seg1_k, seg1_v, seg1_len, len_before
        a.has_sinks, a.has_bank, a.bank_m = int(has_sinks), int(has_bank), bank_m
        _set_dev_pos(a, dev_pos)
        _lib.check(self.lib.bolt3_attend(ctypes.byref(a), _stream()), "bolt3_attend")
        _count(1)


class DevicePosition:
    """The device step position of a decode step replayed from a CUDA graph: an int64 on the device
    that holds the step's token position, the position the launches were built for (`ref`), and how
    many positions after it the launches stay valid for (`span`). Kernels shift the RoPE position,
    the window write offset and the window length by (*word - ref)."""

    def __init__(self, device):
        self.word = torch.zeros(1, dtype=torch.int64, device=device)
        self.ref, self.span = 0, 1

    def set(self, pos: int) -> None:
        """Stream-ordered write of the next step's position (a fill kernel, nothing waits)."""
        self.word.fill_(pos)


def _set_dev_pos(a, dev_pos: "DevicePosition | None") -> None:
    if dev_pos is None:
        a.pos_dev, a.pos_ref, a.pos_span = None, 0, 0
    else:
        a.pos_dev, a.pos_ref, a.pos_span = dev_pos.word.data_ptr(), dev_pos.ref, dev_pos.span


def silu_mul(gu: torch.Tensor) -> torch.Tensor:
    """bolt3_silu_mul: bf16(bf16(silu(g)) * u) for gu = [..., 2I] holding the gate projection in the
    first I columns and the up projection in the last I. Returns [..., I]."""
    I2 = gu.shape[-1]
    if I2 % 16:
        raise ValueError(f"the gate/up width {I2} must be a multiple of 16")
    g2 = gu.reshape(-1, I2)
    _need(g2, torch.bfloat16, "gu")
    y = torch.empty(*gu.shape[:-1], I2 // 2, dtype=torch.bfloat16, device=gu.device)
    a = _lib.SiluMulArgs(gu=g2.data_ptr(), y=y.data_ptr(), rows=g2.shape[0], I=I2 // 2)
    _lib.check(_lib.load().bolt3_silu_mul(ctypes.byref(a), _stream()), "bolt3_silu_mul")
    _count(1)
    return y


def add_rmsnorm(x: torch.Tensor, r: torch.Tensor, w: torch.Tensor, eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """bolt3_rmsnorm with a residual: s = bf16(x + r) and RMSNorm(s) in one kernel. x and r are bf16
    tensors of the same shape (r contiguous); returns (s, normed), both new tensors shaped like x."""
    if not isinstance(r, torch.Tensor) or r.shape != x.shape or r.dtype != torch.bfloat16 or r.device != x.device:
        raise ValueError(f"the residual must be a bf16 tensor shaped like x {tuple(x.shape)} on {x.device}")
    return _rmsnorm(x, w, eps, r.contiguous())


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """bolt3_rmsnorm: RMSNorm over the last dimension of bf16 `x` with weight `w` [D] (bf16 or fp32),
    fp32 inside, one bf16 rounding of the result. Returns a new tensor shaped like x."""
    return _rmsnorm(x, w, eps, None)


def _rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, r: torch.Tensor | None):
    D = x.shape[-1]
    if not isinstance(x, torch.Tensor) or not x.is_cuda or x.dtype != torch.bfloat16:
        raise TypeError("x must be a bf16 CUDA tensor (the Bolt-3 path has no CPU implementation)")
    if x.device.index != torch.cuda.current_device():
        raise RuntimeError(f"x is on {x.device}, but the current device is cuda:{torch.cuda.current_device()}")
    if w.dtype not in (torch.bfloat16, torch.float32) or w.numel() != D or w.device != x.device:
        raise ValueError(f"the weight must be [{D}] bf16 or fp32 on {x.device}")
    x2 = x.reshape(-1, D)
    if x2.stride(-1) != 1 or x2.stride(0) % 8 or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    wc = w.contiguous()
    y = torch.empty(x2.shape[0], D, dtype=torch.bfloat16, device=x.device)
    sm = torch.empty_like(y) if r is not None else None
    a = _lib.RMSNormArgs(x=x2.data_ptr(), w=wc.data_ptr(), y=y.data_ptr(), rows=x2.shape[0], x_stride=x2.stride(0),
                         D=D, w_fp32=int(wc.dtype == torch.float32), eps=eps, r=_ptr(r), sum=_ptr(sm))
    _lib.check(_lib.load().bolt3_rmsnorm(ctypes.byref(a), _stream()), "bolt3_rmsnorm")
    _count(1)
    return y.view(x.shape) if r is None else (sm.view(x.shape), y.view(x.shape))


def anchor_decode(*, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, k_cache: torch.Tensor,
                  v_cache: torch.Tensor, n: int, y: torch.Tensor, scale: float, status=None,
                  dev_pos: DevicePosition | None = None, inv_freq: torch.Tensor | None = None,
                  pos0: int = 0) -> None:
    """bolt3_anchor_decode: append k_new / v_new [B, HKV, HD] at cache position n (n + the device
    shift with dev_pos) of k_cache / v_cache [B, HKV, cap, HD] and write the one-token GQA attention
    of q [B, H, HD] over positions 0..n to y [B, H, HD] (all bf16). With inv_freq (fp32 [HD/2]) the
    kernel applies RoPE at position pos0 (shifted like n) to q and k_new first."""
    B, H, HD = q.shape
    HKV, cap = k_cache.shape[1], k_cache.shape[2]
    _need(q, torch.bfloat16, "q", B * H * HD)
    _need(y, torch.bfloat16, "y", B * H * HD)
    for t, name in ((k_new, "k_new"), (v_new, "v_new")):
        _need(t, torch.bfloat16, name, B * HKV * HD)
    for t, name in ((k_cache, "k_cache"), (v_cache, "v_cache")):
        _need(t, torch.bfloat16, name, B * HKV * cap * HD)
    if tuple(k_cache.shape) != (B, HKV, cap, HD) or tuple(v_cache.shape) != (B, HKV, cap, HD):
        raise ValueError(f"caches must be [B, HKV, cap, HD] = [{B}, {HKV}, {cap}, {HD}]")
    _opt(inv_freq, torch.float32, "inv_freq", HD // 2)
    a = _lib.AnchorArgs(B=B, H=H, HKV=HKV, HD=HD, q=q.data_ptr(), k_new=k_new.data_ptr(), v_new=v_new.data_ptr(),
                        k_cache=k_cache.data_ptr(), v_cache=v_cache.data_ptr(), cap=cap, n=n, y=y.data_ptr(),
                        scale=scale, status=_status(status), inv_freq=_ptr(inv_freq), pos0=pos0)
    _set_dev_pos(a, dev_pos)
    _lib.check(_lib.load().bolt3_anchor_decode(ctypes.byref(a), _stream()), "bolt3_anchor_decode")
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


def _check_prepared(B: int, T: int, H: int, HKV: int, HD: int, q_rope, q_raw, eta, k_rope, v, kappa, coef,
                    res_w, y, q_l2) -> None:
    nq, nk = B * H * T, B * HKV * T
    _need(q_rope, torch.bfloat16, "q_rope", nq * HD)
    _need(q_raw, torch.bfloat16, "q_raw", nq * HD)
    _need(eta, torch.float32, "eta", nq)
    _opt(q_l2, torch.float32, "q_l2", nq)
    _need(k_rope, torch.bfloat16, "k_rope", nk * HD)
    _need(v, torch.bfloat16, "v", nk * HD)
    _need(kappa, torch.float32, "kappa", HKV)
    _need(coef, torch.float32, "coef", HKV)
    _need(res_w, torch.float32, "res_w", HD)
    _need(y, torch.bfloat16, "y", nq * HD)


def attend_prefill(*, n_chains: int, hkv: int, G: int, HD: int, T: int, q_rope, q_raw, eta, k_rope, v,
                   snaps: dict | None, n_cons: int, kappa, coef, res_w, eps: float, y: torch.Tensor,
                   blk_begin: int = 0, blk_count: int = 0, q_l2=None, status=None, wait_probe: int = 0) -> None:
    """Attention of prefill query blocks [blk_begin, blk_begin + blk_count) (bolt3_attend, prefill
    mode): chunk r reads snapshot r - 2 of the consolidation scan."""
    lib = _lib.load()
    if n_chains % hkv:
        raise ValueError(f"{n_chains} chains are not a whole number of sequences of {hkv} KV heads")
    _check_prepared(n_chains // hkv, T, hkv * G, hkv, HD, q_rope, q_raw, eta, k_rope, v, kappa, coef, res_w, y,
                    q_l2)
    sn = snaps or {}
    if n_cons > 0 and T > 2 * CHUNK:
        if not sn:
            raise ValueError("a prefill of more than two chunks reads consolidation snapshots")
        _check_snaps(sn, n_chains, n_cons, HD)
    a = _lib.AttendArgs(
        n_chains=n_chains, hkv=hkv, G=G, HD=HD, q_rope=q_rope.data_ptr(), q_raw=q_raw.data_ptr(),
        eta=eta.data_ptr(), Tq=T, prefill=1, seg0_k=k_rope.data_ptr(), seg0_v=v.data_ptr(),
        seg0_chain_tokens=T, seg1_k=k_rope.data_ptr(), seg1_v=v.data_ptr(), seg1_chain_tokens=T,
        bank_ak_rope=_ptr(sn.get("ak_rope")), bank_av=_ptr(sn.get("av")), bank_mass=_ptr(sn.get("mass")),
        bank_act=_ptr(sn.get("act")), bank_m=_ptr(sn.get("m")), bank_cap=n_cons,
        kappa=kappa.data_ptr(), coef=coef.data_ptr(), res_w=res_w.data_ptr(), eps=eps,
        y=y.data_ptr(), y_tokens=T, status=_status(status), q_l2=_ptr(q_l2), blk_begin=blk_begin,
        blk_count=blk_count, wait_probe=wait_probe)
    _lib.check(lib.bolt3_attend(ctypes.byref(a), _stream()), "bolt3_attend")
    _count(1)


def _prefill_args(B, T, H, HKV, HD, q_rope, q_raw, eta, k_raw, k_rope, v, beta, kappa, gamma, coef, inv_freq,
                  res_w, eps, bank, y, status, q_l2, workspace=None) -> "_lib.PrefillArgs":
    if B <= 0 or T <= 0 or HKV <= 0 or H % HKV:
        raise ValueError(f"unsupported prefill shape B={B} T={T} H={H} HKV={HKV}")
    _check_prepared(B, T, H, HKV, HD, q_rope, q_raw, eta, k_rope, v, kappa, coef, res_w, y, q_l2)
    _need(k_raw, torch.bfloat16, "k_raw", B * HKV * T * HD)
    _need(beta, torch.float32, "beta", B * HKV * T)
    _need(gamma, torch.float32, "gamma", HKV)
    _need(inv_freq, torch.float32, "inv_freq", HD // 2)
    check_bank(bank, B * HKV, HD)
    ws_bytes = 0
    if workspace is not None:
        _need(workspace, torch.uint8, "workspace", prefill_workspace_bytes(B * HKV, T, HD))
        ws_bytes = workspace.numel()
    return _lib.PrefillArgs(
        B=B, T=T, H=H, HKV=HKV, HD=HD, q_rope=q_rope.data_ptr(), q_raw=q_raw.data_ptr(),
        eta=eta.data_ptr(), k_raw=k_raw.data_ptr(), k_rope=k_rope.data_ptr(), v=v.data_ptr(),
        beta=beta.data_ptr(), kappa=kappa.data_ptr(), gamma=gamma.data_ptr(), coef=coef.data_ptr(),
        inv_freq=inv_freq.data_ptr(), res_w=res_w.data_ptr(), eps=eps,
        workspace=_ptr(workspace), workspace_bytes=ws_bytes,
        ak=bank["ak"].data_ptr(), av=bank["av"].data_ptr(), ak_rope=_ptr(bank.get("ak_rope")),
        mass=bank["mass"].data_ptr(), util=bank["util"].data_ptr(), pm=bank["pm"].data_ptr(),
        act=bank["act"].data_ptr(), m_res=bank["m_res"].data_ptr(), n_filled=bank["n_filled"].data_ptr(),
        y=y.data_ptr(), status=_status(status), q_l2=_ptr(q_l2))


def prefill(*, B: int, T: int, H: int, HKV: int, HD: int, q_rope, q_raw, eta, k_raw, k_rope, v, beta,
            kappa, gamma, coef, inv_freq, res_w, eps: float, workspace: torch.Tensor, bank: dict,
            y: torch.Tensor, status=None, q_l2: torch.Tensor | None = None) -> None:
    """Phases B + C of Bolt3Attn.forward on prepared q/k/v (bolt3_prefill_fwd)."""
    lib = _lib.load()
    a = _prefill_args(B, T, H, HKV, HD, q_rope, q_raw, eta, k_raw, k_rope, v, beta, kappa, gamma, coef, inv_freq,
                      res_w, eps, bank, y, status, q_l2, workspace=workspace)
    _lib.check(lib.bolt3_prefill_fwd(ctypes.byref(a), _stream()), "bolt3_prefill_fwd")
    _count(2)  # the scan, then the attention


def noalloc_fits(B: int, T: int, HKV: int, HD: int) -> bool:
    """Whether a prefill of B x T tokens fits the fixed scratch of bolt3_prefill_fwd_noalloc."""
    return prefill_workspace_bytes(B * HKV, T, HD) <= _lib.NOALLOC_SCRATCH_BYTES


def prefill_noalloc(*, B: int, T: int, H: int, HKV: int, HD: int, q_rope, q_raw, eta, k_raw, k_rope, v, beta,
                    kappa, gamma, coef, inv_freq, res_w, eps: float, bank: dict, y: torch.Tensor,
                    status=None, q_l2: torch.Tensor | None = None) -> None:
    """Phases B + C like `prefill`, with the snapshot workspace taken from the library's fixed
    per-GPU array instead of the caller (bolt3_prefill_fwd_noalloc). For hosts that cannot allocate
    device memory on their hot path; the work must fit in `_lib.NOALLOC_SCRATCH_BYTES` (checked
    here, before anything else, and again by the library)."""
    lib = _lib.load()
    need = prefill_workspace_bytes(B * HKV, T, HD)
    if need > _lib.NOALLOC_SCRATCH_BYTES:
        raise ValueError(f"prefill of {B} x {T} tokens needs {need} bytes of scratch; the no-alloc entry point "
                         f"has a fixed {_lib.NOALLOC_SCRATCH_BYTES} bytes (use `prefill` with a workspace)")
    a = _prefill_args(B, T, H, HKV, HD, q_rope, q_raw, eta, k_raw, k_rope, v, beta, kappa, gamma, coef, inv_freq,
                      res_w, eps, bank, y, status, q_l2)
    _lib.check(lib.bolt3_prefill_fwd_noalloc(ctypes.byref(a), _stream()), "bolt3_prefill_fwd_noalloc")
    _count(2)


def new_bank(n_chains: int, HD: int, device, S: int = S_SLOTS, m_res: bool = True) -> dict:
    """Uninitialised bank tensors (the consolidation kernel initialises them with init_blank).
    m_res=False leaves out the [n_chains, HD, HD] fp32 M_res, for a holder whose M_res lives
    elsewhere (a decoder's M_res is the caller's states[li]) and is put into the dict per call."""
    bf = dict(dtype=torch.bfloat16, device=device)
    f32 = dict(dtype=torch.float32, device=device)
    bank = dict(ak=torch.empty(n_chains, S, HD, **bf), av=torch.empty(n_chains, S, HD, **bf),
                ak_rope=torch.empty(n_chains, S, HD, **bf), mass=torch.empty(n_chains, S, **f32),
                util=torch.empty(n_chains, S, **f32), pm=torch.empty(n_chains, S, **f32),
                act=torch.zeros(n_chains, S, dtype=torch.uint8, device=device),
                n_filled=torch.zeros(n_chains, dtype=torch.int32, device=device))
    if m_res:
        bank["m_res"] = torch.zeros(n_chains, HD, HD, **f32)
    return bank
