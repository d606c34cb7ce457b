"""Device-side failure reporting, tested without faulting the GPU.

Every wait in the kernels (TMA and MMA completion on mbarriers) is bounded; a wait that runs out
sets a bit in the caller's status word and the kernel skips the dependent work. These tests make a
wait run out on purpose through the `wait_probe` argument: the kernel's first thread polls a barrier
that nothing arrives at, records the expired wait and the kernel returns before it allocates tensor
memory or starts any copy or MMA. The host must turn the bit into a RuntimeError, and the context
must stay usable afterwards.
"""
import pytest
import torch

from helpers import bf16_module, inputs
from vsa_lm_b200 import Bolt3Decoder, Bolt3LayerState
from vsa_lm_b200 import kernels as K
from vsa_lm_b200.workloads import layer_cfg, make_input

pytestmark = pytest.mark.gpu
PROBE = 4096   # polls of the probe barrier (a few microseconds)


def _prepared(m, x):
    p, prep_q = m._prepare(x)
    prep_q()
    return p


def test_scan_wait_expiry_raises_and_context_survives():
    cfg, _, x = inputs("qwen3_4b", 1, 640, 0.3)
    m = bf16_module(cfg, 0)
    p = _prepared(m, x)
    c = p.consts
    bank = K.new_bank(m.HKV, m.HD, x.device)
    status = K.DeviceStatus(x.device)
    kw = dict(n_chains=m.HKV, hkv=m.HKV, HD=m.HD, bank=bank, init_blank=True, kr=p.k_raw, kp=p.k_rope, v=p.v,
              beta=p.beta, chain_tokens=640, token0=0, step_tokens=128, skip0=4, chunk_len=128, pos0=0, n_steps=3,
              kappa=c["kappa"], gamma=c["gamma"], inv_freq=c["inv_freq"], status=status)
    K.consolidate(wait_probe=PROBE, **kw)
    status.arm("probed scan")
    with pytest.raises(RuntimeError, match="consolidation scan expired"):
        status.check(block=True)
    assert int(status.word.item()) == 0, "a reported error clears the word"
    K.consolidate(**kw)                      # the same call without the probe runs normally
    status.arm("scan")
    status.check(block=True)
    assert int(bank["n_filled"][0].item()) > 0


def test_prefill_attention_wait_expiry_raises():
    cfg, _, x = inputs("qwen3_4b", 1, 256, 0.3)
    m = bf16_module(cfg, 0)
    p = _prepared(m, x)
    c = p.consts
    y = torch.zeros(1, 256, m.H, m.HD, dtype=torch.bfloat16, device=x.device)
    status = K.DeviceStatus(x.device)
    # two chunks read no bank, so no snapshots are needed
    kw = dict(n_chains=m.HKV, hkv=m.HKV, G=m.G, HD=m.HD, T=256, q_rope=p.q_rope, q_raw=p.q_raw, eta=p.eta,
              k_rope=p.k_rope, v=p.v, snaps=None, n_cons=0, kappa=c["kappa"], coef=c["coef"], res_w=c["res_w"],
              eps=m.eps, y=y, blk_begin=0, blk_count=2, status=status)
    K.attend_prefill(wait_probe=PROBE, **kw)
    status.arm("probed attention")
    with pytest.raises(RuntimeError, match="attention kernel expired"):
        status.check(block=True)
    assert torch.count_nonzero(y) == 0, "a probed launch writes no output"
    K.attend_prefill(**kw)
    status.arm("attention")
    status.check(block=True)
    assert torch.count_nonzero(y) > 0


def test_decode_stream_wait_expiry_raises():
    """The one-token decode kernel (tensor-core streaming kernel at HD = 128, G = 4)."""
    cfg = layer_cfg("qwen3_4b")
    m = bf16_module(cfg, 0)
    B = 2
    x = make_input(B, 260, cfg["dim"], dup=0.3, seed=2).to(torch.bfloat16).cuda()
    st = Bolt3LayerState(m, B, "cuda")
    m_res = torch.zeros(B, m.HKV, m.HD, m.HD, device="cuda")
    for pos, n in ((0, 128), (128, 128), (256, 1)):
        Bolt3Decoder.layer_step(m, st, x[:, pos:pos + n], pos, m_res)
    Bolt3Decoder.check_status([st])
    plan = st._plans[1]
    plan.args.attend.wait_probe = PROBE
    try:
        Bolt3Decoder.layer_step(m, st, x[:, 257:258], 257, m_res)
    finally:
        plan.args.attend.wait_probe = 0
    st.status.arm("probed decode step")
    with pytest.raises(RuntimeError, match="attention kernel expired"):
        Bolt3Decoder.check_status([st])
    Bolt3Decoder.layer_step(m, st, x[:, 258:259], 258, m_res)
    st.status.arm("decode step")
    Bolt3Decoder.check_status([st])


def test_forward_reports_a_set_status_bit():
    """The product forward checks its status word: a bit left set by an earlier call surfaces as a
    RuntimeError at the next check."""
    cfg, _, x = inputs("tiny", 1, 300, 0.3)
    m = bf16_module(cfg, 0)
    m(x)
    m.check_status()
    m.device_status(x.device).word.fill_(1)
    m(x)
    with pytest.raises(RuntimeError, match="tie-order emulation"):
        m.check_status()
    m(x)
    m.check_status()
