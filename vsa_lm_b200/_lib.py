"""ctypes binding of the C-ABI in include/bolt3.h (libbolt3.so, built in-tree).

The structs below mirror the header field for field. Loading fails loudly: there is no CPU or
PyTorch fallback for the Bolt-3 kernels.
"""
from __future__ import annotations

import ctypes
import os
import threading

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_F = ctypes.c_float
_SZ = ctypes.c_size_t

STATUS = {0: "ok", 1: "invalid argument", 2: "unsupported shape", 3: "misaligned pointer",
          4: "buffer too small", 5: "CUDA error"}

# Bits of the device status word the kernels OR into (include/bolt3.h)
DEVICE_STATUS_BITS = {1: "a bounds check of the consolidation's tie-order emulation fired",
                      2: "a bounded wait in an attention kernel expired",
                      4: "a bounded wait in the consolidation scan expired",
                      8: "a decode step's device position was outside the range its launch was built for"}


class PrepArgs(ctypes.Structure):
    _fields_ = [
        ("proj", _P), ("ld", _I64),
        ("B", _I), ("T", _I), ("H", _I), ("HKV", _I), ("HD", _I),
        ("q_norm_w", _P), ("k_norm_w", _P), ("eps", _F),
        ("inv_freq", _P), ("pos0", _I64),
        ("q_raw", _P), ("q_rope", _P), ("q_head_stride", _I64), ("q_t_off", _I64),
        ("eta", _P), ("eta_head_stride", _I64), ("eta_t_off", _I64),
        ("k_raw", _P), ("k_rope", _P), ("v", _P), ("k_head_stride", _I64), ("k_t_off", _I64),
        ("beta", _P), ("beta_head_stride", _I64), ("beta_t_off", _I64),
        ("q_l2", _P),
        ("parts", _I),
        ("q_col", _I64), ("k_col", _I64), ("v_col", _I64), ("beta_col", _I64), ("eta_col", _I64),
        ("pos_dev", _P), ("pos_ref", _I64), ("pos_span", _I64),
    ]


class ConsolidateArgs(ctypes.Structure):
    _fields_ = [
        ("n_chains", _I), ("hkv", _I), ("HD", _I),
        ("ak", _P), ("av", _P), ("ak_rope", _P),
        ("mass", _P), ("util", _P), ("pm", _P), ("act", _P), ("m_res", _P), ("n_filled", _P),
        ("init_blank", _I),
        ("kr", _P), ("kp", _P), ("v", _P), ("beta", _P),
        ("chain_tokens", _I64),
        ("token0", _I64), ("step_tokens", _I64), ("skip0", _I), ("chunk_len", _I), ("pos0", _I64),
        ("n_steps", _I),
        ("kappa", _P), ("gamma", _P), ("inv_freq", _P),
        ("snap_ak_rope", _P), ("snap_av", _P), ("snap_mass", _P), ("snap_act", _P), ("snap_m", _P),
        ("snap_cap", _I64), ("snap0", _I64),
        ("status", _P),
        ("wait_probe", ctypes.c_uint32),
    ]


class AttendArgs(ctypes.Structure):
    _fields_ = [
        ("n_chains", _I), ("hkv", _I), ("G", _I), ("HD", _I),
        ("q_rope", _P), ("q_raw", _P), ("eta", _P), ("Tq", _I64),
        ("prefill", _I),
        ("seg0_k", _P), ("seg0_v", _P), ("seg0_chain_tokens", _I64), ("seg0_len", _I),
        ("seg1_k", _P), ("seg1_v", _P), ("seg1_chain_tokens", _I64), ("seg1_len", _I),
        ("len_before", _I),
        ("sink_k", _P), ("sink_v", _P), ("sink_chain_tokens", _I64), ("has_sinks", _I),
        ("bank_ak_rope", _P), ("bank_av", _P), ("bank_mass", _P), ("bank_act", _P), ("bank_m", _P),
        ("bank_cap", _I64), ("has_bank", _I),
        ("kappa", _P), ("coef", _P), ("res_w", _P), ("eps", _F),
        ("y", _P), ("y_tokens", _I64),
        ("status", _P),
        ("q_l2", _P),
        ("blk_begin", _I64), ("blk_count", _I64),
        ("wait_probe", ctypes.c_uint32),
        ("pos_dev", _P), ("pos_ref", _I64), ("pos_span", _I64),
    ]


class AnchorArgs(ctypes.Structure):
    _fields_ = [
        ("B", _I), ("H", _I), ("HKV", _I), ("HD", _I),
        ("q", _P), ("k_new", _P), ("v_new", _P),
        ("k_cache", _P), ("v_cache", _P), ("cap", _I64), ("n", _I64),
        ("y", _P), ("scale", _F),
        ("status", _P),
        ("pos_dev", _P), ("pos_ref", _I64), ("pos_span", _I64),
        ("inv_freq", _P), ("pos0", _I64),
    ]


class RMSNormArgs(ctypes.Structure):
    _fields_ = [
        ("x", _P), ("w", _P), ("y", _P),
        ("rows", _I64), ("x_stride", _I64),
        ("D", _I), ("w_fp32", _I), ("eps", _F),
        ("r", _P), ("sum", _P),
    ]


class SiluMulArgs(ctypes.Structure):
    _fields_ = [("gu", _P), ("y", _P), ("rows", _I64), ("I", _I64)]


class PrefillArgs(ctypes.Structure):
    _fields_ = [
        ("B", _I), ("T", _I), ("H", _I), ("HKV", _I), ("HD", _I),
        ("q_rope", _P), ("q_raw", _P), ("eta", _P),
        ("k_raw", _P), ("k_rope", _P), ("v", _P), ("beta", _P),
        ("kappa", _P), ("gamma", _P), ("coef", _P), ("inv_freq", _P),
        ("res_w", _P), ("eps", _F),
        ("workspace", _P), ("workspace_bytes", _SZ),
        ("ak", _P), ("av", _P), ("ak_rope", _P), ("mass", _P), ("util", _P), ("pm", _P), ("act", _P),
        ("m_res", _P), ("n_filled", _P),
        ("y", _P),
        ("status", _P),
        ("q_l2", _P),
    ]


# entry point -> (argtypes, restype); every name here is declared in include/bolt3.h
SIGNATURES = {
    "bolt3_prep": ([ctypes.POINTER(PrepArgs), _P], _I),
    "bolt3_consolidate": ([ctypes.POINTER(ConsolidateArgs), _P], _I),
    "bolt3_attend": ([ctypes.POINTER(AttendArgs), _P], _I),
    "bolt3_anchor_decode": ([ctypes.POINTER(AnchorArgs), _P], _I),
    "bolt3_rmsnorm": ([ctypes.POINTER(RMSNormArgs), _P], _I),
    "bolt3_silu_mul": ([ctypes.POINTER(SiluMulArgs), _P], _I),
    "bolt3_prefill_fwd": ([ctypes.POINTER(PrefillArgs), _P], _I),
    "bolt3_prefill_fwd_noalloc": ([ctypes.POINTER(PrefillArgs), _P], _I),
    "bolt3_prefill_workspace_size": ([_I, _I64, _I], _SZ),
    "bolt3_abi_version": ([], _I),
    "bolt3_args_size": ([_I], _SZ),
    "bolt3_status_string": ([_I], ctypes.c_char_p),
    "bolt3_topk_order_host": ([_P, _I, _I, _I, _P], _I),
}

ABI_VERSION = 10   # BOLT3_ABI_VERSION in include/bolt3.h

# Fixed scratch of bolt3_prefill_fwd_noalloc (BOLT3_NOALLOC_SCRATCH_BYTES in include/bolt3.h)
NOALLOC_SCRATCH_BYTES = 32 << 20

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libbolt3.so")
_lib = None
_lock = threading.Lock()


def load(build_if_missing: bool = True) -> ctypes.CDLL:
    """Load libbolt3.so (building it first if it is missing and nvcc is available)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH) and build_if_missing:
            from .build import build
            build()
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"Bolt-3 CUDA library not found at {LIB_PATH}; run `python -m vsa_lm_b200.build`")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (argt, rest) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argt
            fn.restype = rest
        if lib.bolt3_abi_version() != ABI_VERSION:
            raise RuntimeError("libbolt3.so ABI version mismatch; rebuild with `python -m vsa_lm_b200.build`")
        for i, st in enumerate((PrepArgs, ConsolidateArgs, AttendArgs, PrefillArgs, AnchorArgs, RMSNormArgs,
                                SiluMulArgs)):
            if lib.bolt3_args_size(i) != ctypes.sizeof(st):
                raise RuntimeError(f"{st.__name__} has {ctypes.sizeof(st)} bytes here but "
                                   f"{lib.bolt3_args_size(i)} in libbolt3.so: the bindings and the header differ")
        _lib = lib
        return lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load().bolt3_status_string(rc).decode()
        raise RuntimeError(f"{what} failed: status {rc} ({msg})")
