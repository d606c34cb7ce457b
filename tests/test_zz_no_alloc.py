"""bolt3_prefill_fwd_noalloc: the prefill entry point that allocates nothing.

Hosts that cannot call cudaMalloc on their hot path (an engine that pools all of HBM itself, a C-ABI
host without a device allocator, a loop that cannot afford cudaMalloc's implicit device
synchronisation) use this entry point; its snapshot workspace is a fixed array inside the library.
This file is collected last so that a run stopping at the first failure has run every other test.
"""
import ctypes

import pytest
import torch

from helpers import bf16_module, inputs, output_close
from vsa_lm_b200 import _lib
from vsa_lm_b200 import kernels as K

pytestmark = pytest.mark.gpu


def _prepared(m, x):
    b, T, D = x.shape
    H, HKV, HD = m.H, m.HKV, m.HD
    f = m.fused(x.device)
    c = f.consts
    bf = dict(dtype=torch.bfloat16, device=x.device)
    t = dict(q_raw=torch.empty(b * H, T, HD, **bf), q_rope=torch.empty(b * H, T, HD, **bf),
             k_raw=torch.empty(b * HKV, T, HD, **bf), k_rope=torch.empty(b * HKV, T, HD, **bf),
             v=torch.empty(b * HKV, T, HD, **bf), beta=torch.empty(b * HKV, T, device=x.device),
             eta=torch.empty(b * H, T, device=x.device), q_l2=torch.empty(b * H, T, device=x.device))
    K.prep(m.project(x.reshape(b * T, D), f), B=b, T=T, H=H, HKV=HKV, HD=HD, inv_freq=c["inv_freq"], eps=m.eps,
           q_norm_w=c["qn"], k_norm_w=c["kn"], pos0=0, cols=f.cols, q_head_stride=T, q_t_off=0, k_head_stride=T,
           k_t_off=0, **t)
    t.update(kappa=c["kappa"], gamma=c["gamma"], coef=c["coef"], inv_freq=c["inv_freq"], res_w=c["res_w"],
             eps=m.eps, B=b, T=T, H=H, HKV=HKV, HD=HD)
    return t


@pytest.mark.parametrize("shape,B,T", [("qwen3_4b", 1, 2048), ("tiny", 2, 1300)])   # HD = 128 and HD = 64
def test_noalloc_prefill_matches_workspace_prefill_twice(shape, B, T):
    """Two calls in a row, on different inputs, each against the allocating entry point."""
    cfg, _, x1 = inputs(shape, B, T, 0.3, seed=11)
    _, _, x2 = inputs(shape, B, T, 0.3, seed=12)
    m = bf16_module(cfg, 0)
    for x in (x1, x2):
        t = _prepared(m, x)
        b, T = x.shape[:2]
        ws = torch.empty(K.prefill_workspace_bytes(b * m.HKV, T, m.HD), dtype=torch.uint8, device=x.device)
        bank_ref = K.new_bank(b * m.HKV, m.HD, x.device)
        y_ref = torch.empty(b, T, m.H, m.HD, dtype=torch.bfloat16, device=x.device)
        K.prefill(workspace=ws, bank=bank_ref, y=y_ref, **t)
        bank = K.new_bank(b * m.HKV, m.HD, x.device)
        y = torch.empty_like(y_ref)
        K.prefill_noalloc(bank=bank, y=y, **t)
        torch.cuda.synchronize()
        output_close(y, y_ref, "no-alloc prefill output")
        torch.testing.assert_close(bank["m_res"], bank_ref["m_res"], rtol=1e-4, atol=1e-6)
        assert torch.equal(bank["mass"], bank_ref["mass"])


def test_noalloc_rejects_work_beyond_its_scratch():
    lib = _lib.load()
    a = _lib.PrefillArgs(B=8, T=8192, H=32, HKV=8, HD=128)   # 64 chains x 62 snapshots: > 32 MiB
    assert lib.bolt3_prefill_fwd_noalloc(ctypes.byref(a), None) == 4   # BOLT3_ERR_CAPACITY
