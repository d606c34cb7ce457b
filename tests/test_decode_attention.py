"""The decode-step attention kernels against the oracle's attention (oracle/bolt3_oracle.py `attend`,
which restates vsa_lm/config/bolt3.py:365-402) on random decoder states, with more chains than the
GPU has SMs, so that the persistent streaming kernel walks several chains per CTA (the decoder tests
use a handful of chains only)."""
import pytest
import torch

from helpers import BF16, output_close
from oracle import attend, gamma_delta, llama_inv_freq, rope_at
from vsa_lm_b200 import kernels as K

pytestmark = pytest.mark.gpu
C, S = 128, 128


@pytest.mark.parametrize("HD,G,B,L0,len_before,Tq,bank,q_l2", [
    (128, 4, 40, 128, 36, 1, True, False),     # one-token step with a full window and a bank
    (128, 4, 40, 128, 36, 1, True, True),      # the same with |q_raw| supplied by the projection
    (128, 4, 40, 0, 4, 1, False, False),       # first chunk: no previous chunk, no bank
    (128, 4, 40, 128, 0, 1, False, True),      # second chunk's first token, bank not yet formed
    (128, 2, 40, 128, 70, 2, True, False),     # two tokens of two query heads (4 rows)
    (128, 1, 40, 128, 10, 1, True, False),     # one query head per KV head: 1 row, 3 padded
    (128, 3, 40, 128, 50, 1, True, True),      # three query heads per KV head: 3 rows
    (64, 3, 40, 128, 100, 1, True, False),     # HD = 64: the warp-per-chain kernel
])
def test_decode_attention_matches_oracle(HD, G, B, L0, len_before, Tq, bank, q_l2):
    torch.manual_seed(7)
    HKV = 8
    H = HKV * G
    nc = B * HKV
    L1 = len_before + Tq
    bf = lambda t: t.to(torch.bfloat16).float()       # values as the kernel receives them
    q_p = bf(torch.randn(B, H, Tq, HD))
    q_r = bf(torch.randn(B, H, Tq, HD) * 1.5)
    eta = torch.randn(B, H, Tq) * 0.5
    loc_k = bf(torch.randn(B, HKV, L0 + L1, HD))
    loc_v = bf(torch.randn(B, HKV, L0 + L1, HD))
    sink_k, sink_v = bf(torch.randn(B, HKV, 4, HD)), bf(torch.randn(B, HKV, 4, HD))
    inv_freq = llama_inv_freq(HD, 1e6)
    kappa = torch.rand(HKV) + 0.5
    gam = gamma_delta(torch.full((HKV,), 3.5) + torch.randn(HKV) * 0.1)
    res_w = torch.rand(HD) * 0.1
    eps = 1e-6
    bk = None
    if bank:
        bk = dict(ak=bf(torch.randn(nc, S, HD)), av=bf(torch.randn(nc, S, HD)),
                  mass=torch.rand(nc, S) * 5.0, pm=torch.rand(nc, S) * 4000.0,
                  act=torch.rand(nc, S) > 0.2, m_res=torch.randn(nc, HD, HD) * 0.05)
    ref = attend(q_p, q_r, eta, loc_k, loc_v, L0 + len_before, (sink_k, sink_v), bk, kappa=kappa, gam=gam,
                 inv_freq=inv_freq, res_w=res_w, eps=eps, G=G, store=BF16)            # [B, H, Tq, HD]

    cu = lambda t, dt=torch.bfloat16: t.to(device="cuda", dtype=dt).contiguous()
    # the decoder's window ring: two chunk slots per chain, the previous chunk in slot 1 here
    ring_k = torch.zeros(nc, 2 * C, HD, dtype=torch.bfloat16, device="cuda")
    ring_v = torch.zeros_like(ring_k)
    ring_k[:, C:C + L0] = cu(loc_k[:, :, :L0].reshape(nc, L0, HD))
    ring_v[:, C:C + L0] = cu(loc_v[:, :, :L0].reshape(nc, L0, HD))
    ring_k[:, :L1] = cu(loc_k[:, :, L0:].reshape(nc, L1, HD))
    ring_v[:, :L1] = cu(loc_v[:, :, L0:].reshape(nc, L1, HD))
    b = None
    if bank:
        ak_rope = rope_at(bk["ak"].view(B, HKV, S, HD), bk["pm"].view(B, HKV, S), inv_freq, BF16)
        b = dict(ak_rope=cu(ak_rope.reshape(nc, S, HD)), av=cu(bk["av"]), mass=cu(bk["mass"], torch.float32),
                 act=cu(bk["act"], torch.uint8), m_res=cu(bk["m_res"], torch.float32))
    y = torch.full((B, Tq, H, HD), float("nan"), dtype=torch.bfloat16, device="cuda")
    q_raw = cu(q_r.reshape(B * H, Tq, HD))
    l2 = q_raw.float().norm(dim=-1).contiguous() if q_l2 else None
    K.attend_decode(n_chains=nc, hkv=HKV, G=G, HD=HD, q_rope=cu(q_p.reshape(B * H, Tq, HD)), q_raw=q_raw,
                    eta=cu(eta.reshape(B * H, Tq), torch.float32), Tq=Tq,
                    seg0_k=ring_k[:, C:], seg0_v=ring_v[:, C:], seg0_chain_tokens=2 * C, seg0_len=L0,
                    seg1_k=ring_k, seg1_v=ring_v, seg1_chain_tokens=2 * C, seg1_len=L1, len_before=len_before,
                    sinks=(cu(sink_k.reshape(nc, 4, HD)), cu(sink_v.reshape(nc, 4, HD))), bank=b,
                    kappa=cu(kappa, torch.float32), coef=cu((1.0 - gam) / HD ** 0.5, torch.float32),
                    res_w=cu(res_w, torch.float32), eps=eps, y=y, q_l2=l2)
    got = y.float().cpu().permute(0, 2, 1, 3)
    assert torch.isfinite(got).all(), "every output row must be written"
    output_close(got, ref, f"decode attention HD={HD} G={G} Tq={Tq}")
