"""The torch-facing wrappers refuse bad arguments before anything reaches the C-ABI.

The library cannot tell a host pointer from a device pointer, so a CPU tensor, a tensor of the
wrong dtype or too small a buffer must raise in Python: passed on, it would make a kernel read or
write memory it does not own. These run without a GPU: every case raises before a launch.
"""
import ctypes

import pytest
import torch

from vsa_lm_b200 import _lib
from vsa_lm_b200 import kernels as K


def _prefill_kwargs(B=1, T=300, H=4, HKV=2, HD=64, device="cpu", dtype=torch.bfloat16):
    bf = dict(dtype=dtype, device=device)
    f32 = dict(dtype=torch.float32, device=device)
    return dict(B=B, T=T, H=H, HKV=HKV, HD=HD,
                q_rope=torch.zeros(B * H, T, HD, **bf), q_raw=torch.zeros(B * H, T, HD, **bf),
                eta=torch.zeros(B * H, T, **f32), k_raw=torch.zeros(B * HKV, T, HD, **bf),
                k_rope=torch.zeros(B * HKV, T, HD, **bf), v=torch.zeros(B * HKV, T, HD, **bf),
                beta=torch.zeros(B * HKV, T, **f32), kappa=torch.ones(HKV, **f32), gamma=torch.ones(HKV, **f32),
                coef=torch.ones(HKV, **f32), inv_freq=torch.ones(HD // 2, **f32), res_w=torch.ones(HD, **f32),
                eps=1e-5, bank=K.new_bank(B * HKV, HD, device), y=torch.zeros(B, T, H, HD, **bf))


def test_prefill_rejects_cpu_tensors():
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        K.prefill(workspace=torch.zeros(1 << 20, dtype=torch.uint8), **_prefill_kwargs())


def test_noalloc_prefill_rejects_cpu_tensors():
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        K.prefill_noalloc(**_prefill_kwargs())


def test_noalloc_capacity_boundary():
    """32 MiB holds 254 chain-consolidations at HD = 128: one Qwen3-4B-shape sequence (8 KV heads)
    of up to 4224 tokens (31 consolidations) fits, 4225 tokens (32) does not."""
    lib = _lib.load()
    cap = _lib.NOALLOC_SCRATCH_BYTES
    assert cap == 32 << 20
    assert lib.bolt3_prefill_workspace_size(8, 4224, 128) <= cap
    assert lib.bolt3_prefill_workspace_size(8, 4225, 128) > cap
    assert K.noalloc_fits(1, 4224, 8, 128) and not K.noalloc_fits(1, 4225, 8, 128)
    # the wrapper refuses the larger case with ValueError before checking or launching anything
    with pytest.raises(ValueError, match="fixed"):
        K.prefill_noalloc(**_prefill_kwargs(T=4225, H=32, HKV=8, HD=128))


def test_noalloc_entry_point_returns_capacity_status_at_the_boundary():
    """The C entry point itself: BOLT3_ERR_CAPACITY (4) past the limit, returned before any device
    call (the pointers are never read)."""
    lib = _lib.load()
    a = _lib.PrefillArgs(B=1, T=4225, H=32, HKV=8, HD=128)
    assert lib.bolt3_prefill_fwd_noalloc(ctypes.byref(a), None) == 4


def test_consolidate_and_attend_reject_cpu_tensors():
    kw = _prefill_kwargs()
    bank = kw["bank"]
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        K.consolidate(n_chains=2, hkv=2, HD=64, bank=bank, init_blank=True, kr=kw["k_raw"], kp=kw["k_rope"],
                      v=kw["v"], beta=kw["beta"], chain_tokens=300, token0=0, step_tokens=128, skip0=4,
                      chunk_len=128, pos0=0, n_steps=1, kappa=kw["kappa"], gamma=kw["gamma"],
                      inv_freq=kw["inv_freq"])
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        K.attend_prefill(n_chains=2, hkv=2, G=2, HD=64, T=300, q_rope=kw["q_rope"], q_raw=kw["q_raw"],
                         eta=kw["eta"], k_rope=kw["k_rope"], v=kw["v"], snaps=None, n_cons=0,
                         kappa=kw["kappa"], coef=kw["coef"], res_w=kw["res_w"], eps=1e-5, y=kw["y"])


def test_prep_rejects_cpu_projection():
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        K.prep(torch.zeros(4, 1024, dtype=torch.bfloat16), B=1, T=4, H=4, HKV=2, HD=64,
               inv_freq=torch.ones(32), eps=1e-5, q_norm_w=None, k_norm_w=None, pos0=0, cols={})
