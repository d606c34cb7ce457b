"""Parity of the CUDA path (through the C-ABI) with the CPU oracle, on seeded inputs.

Tolerances (the north star's): bf16 outputs within rtol 2e-2 (atol 2e-2 x RMS for near-zero
elements); fp32 state (M_res, mass, pm, util) within 1e-4 relative; merge/evict decisions identical
except for chains where a cosine lies within 1e-3 of the 0.88 / 0.80 thresholds, which are counted.
"""
import pytest
import torch

from helpers import (BF16, STATE_RTOL, bf16_module, inputs, near_threshold, near_tie_chains, oracle_cfg_of,
                     oracle_params, output_close)
from oracle import LayerDecoderOracle, forward, gamma_delta, project, rope_at
from vsa_lm_b200 import Bolt3Decoder, Bolt3LayerState
from vsa_lm_b200 import kernels as K
from vsa_lm_b200.workloads import layer_cfg, make_input

pytestmark = pytest.mark.gpu
C = 128


@pytest.mark.parametrize("shape", ["config0", "qwen3_4b"])
def test_prep_matches_oracle(shape):
    B, T = 2, 300
    cfg, x_cpu, x = inputs(shape, B, T, 0.0)
    m = bf16_module(cfg, 0)
    f = m.fused(x.device)
    c = f.consts
    H, HKV, HD = m.H, m.HKV, m.HD
    proj = m.project(x.reshape(B * T, -1), f)
    bf = dict(dtype=torch.bfloat16, device="cuda")
    q_raw, q_rope = torch.empty(B * H, T, HD, **bf), torch.empty(B * H, T, HD, **bf)
    k_raw, k_rope, v = (torch.empty(B * HKV, T, HD, **bf) for _ in range(3))
    beta = torch.empty(B * HKV, T, dtype=torch.float32, device="cuda")
    eta = torch.empty(B * H, T, dtype=torch.float32, device="cuda")
    K.prep(proj, B=B, T=T, H=H, HKV=HKV, HD=HD, inv_freq=c["inv_freq"], eps=m.eps, q_norm_w=c["qn"],
           k_norm_w=c["kn"], pos0=0, q_raw=q_raw, q_rope=q_rope, eta=eta, k_raw=k_raw, k_rope=k_rope, v=v,
           beta=beta, q_head_stride=T, q_t_off=0, k_head_stride=T, k_t_off=0)
    oc = oracle_cfg_of(m, cfg)
    qr, kr, vo, bo, eo = project(oracle_params(m), oc, x_cpu, BF16)
    pos = torch.arange(T, dtype=torch.float32)
    # projections: equal up to the GEMM's accumulation order: one bf16 ulp of the projection, which
    # the qk RMSNorm scale can stretch to two ulps of its output
    for name, got, ref in (("q_raw", q_raw, qr), ("k_raw", k_raw, kr), ("v", v, vo), ("beta", beta, bo),
                           ("eta", eta, eo)):
        ref = ref.reshape(got.shape)
        g = got.float().cpu()
        err = (g - ref).abs()
        worst = int(err.argmax())
        assert (err <= 1.6e-2 * ref.abs() + 2e-4).all(), \
            f"{name}: max |diff| {err.max().item():.3e} at {worst}: got {g.flatten()[worst].item()} ref {ref.flatten()[worst].item()}"
        same = (g == ref).float().mean().item()
        assert same > 0.98, f"{name}: only {same:.4f} identical"
    # RoPE in the storage dtype: bit-exact given the same input
    for name, got, src in (("q_rope", q_rope, q_raw), ("k_rope", k_rope, k_raw)):
        ref = rope_at(src.float().cpu(), pos, oc["inv_freq"], BF16)
        assert torch.equal(got.float().cpu(), ref), f"{name} differs from RoPE of the same input"


def _oracle_run(shape, B, T, dup, seed=0):
    cfg, x_cpu, x = inputs(shape, B, T, dup)
    m = bf16_module(cfg, seed)
    P, oc = oracle_params(m), oracle_cfg_of(m, cfg)
    rec, snaps = [], []
    y_ref = forward(P, oc, x_cpu, BF16, record=rec, snapshots=snaps)
    return cfg, m, P, oc, x_cpu, x, y_ref, rec, snaps


@pytest.mark.parametrize("shape,B,T,dup", [("config0", 1, 1024, "chunks"), ("qwen3_4b", 2, 1024, 0.3),
                                           ("tiny", 2, 1152, 0.3)])
def test_consolidation_teacher_forced(shape, B, T, dup):
    """Each native consolidation, fed the oracle's pre-state, reproduces the oracle's post-state."""
    cfg, m, P, oc, x_cpu, x, y_ref, rec, snaps = _oracle_run(shape, B, T, dup)
    qr, kr, vo, bo, eo = project(P, oc, x_cpu, BF16)
    pos = torch.arange(T, dtype=torch.float32)
    kp = rope_at(kr, pos, oc["inv_freq"], BF16)
    gam = gamma_delta(P["log_gamma"]).cuda()
    inv = oc["inv_freq"].cuda()
    flips = 0
    assert len(snaps) >= 3, "case must reach the full-bank path"
    for i, post in enumerate(snaps):
        pre = snaps[i - 1] if i > 0 else None
        skip = 4 if i == 0 else 0
        s, e = i * C + skip, (i + 1) * C
        cu = lambda t, dt=torch.bfloat16: t.to(device="cuda", dtype=dt)
        args = [None] * 7 if pre is None else [cu(pre["ak"]), cu(pre["av"]), cu(pre["mass"], torch.float32),
                                                cu(pre["util"], torch.float32), cu(pre["pm"], torch.float32),
                                                cu(pre["act"], torch.bool), cu(pre["m_res"], torch.float32)]
        out = m._consolidate_functional(*args, cu(kr[:, :, s:e]), cu(kp[:, :, s:e]), cu(vo[:, :, s:e]),
                                        pos[s:e].cuda(), cu(bo[:, :, s:e], torch.float32), inv, None, gam,
                                        n_filled=0 if pre is None else pre["n_filled"])
        ak, av, mass, util, pmv, act, m_res, n_f = out
        assert n_f == post["n_filled"]
        near = near_threshold(rec[i]) | near_tie_chains(rec[i])
        flips += int(near.sum())
        ok = ~near
        if rec[i]["kind"] == "fill":
            # the fill's slot order follows the score ranking: compare slots sorted by token position
            order_g, order_r = torch.argsort(pmv.cpu(), dim=-1), torch.argsort(post["pm"], dim=-1)
            take = lambda t, o: torch.gather(t, 1, o) if t.dim() == 2 else torch.gather(t, 1, o.unsqueeze(-1).expand_as(t))
            ak, av, mass, util, pmv, act = (take(t.cpu(), order_g) for t in (ak, av, mass, util, pmv, act))
            post = dict(post)
            for k in ("ak", "av", "mass", "util", "pm", "act"):
                post[k] = take(post[k], order_r)
        assert torch.equal(act.cpu()[ok], post["act"][ok]), f"act @ {i}"
        assert torch.equal(mass.cpu()[ok], post["mass"][ok]), f"mass (merge/evict decisions) @ {i}"
        torch.testing.assert_close(pmv.cpu()[ok], post["pm"][ok], rtol=STATE_RTOL, atol=1e-3, msg=f"pm @ {i}")
        torch.testing.assert_close(util.cpu()[ok], post["util"][ok], rtol=STATE_RTOL, atol=1e-6, msg=f"util @ {i}")
        torch.testing.assert_close(ak.float().cpu()[ok], post["ak"][ok], rtol=8e-3, atol=1e-6, msg=f"ak @ {i}")
        torch.testing.assert_close(av.float().cpu()[ok], post["av"][ok], rtol=8e-3, atol=1e-6, msg=f"av @ {i}")
        ref_m = post["m_res"][ok]
        scale = ref_m.abs().amax(dim=(-1, -2), keepdim=True).clamp_min(1e-30)
        err = ((m_res.cpu()[ok] - ref_m).abs() / scale).max().item() if ok.any() else 0.0
        assert err < STATE_RTOL, f"M_res @ {i}: max error {err:.2e} of the chain's max |M|"
    print(f"near-threshold / near-tie chains excluded: {flips}")


@pytest.mark.parametrize("shape,B,T,dup", [
    ("config0", 1, 1024, "chunks"),
    ("qwen3_4b", 2, 1024, 0.3),
    ("tiny", 2, 700, 0.3),
    ("tiny", 1, 100, 0.0), ("tiny", 1, 128, 0.0), ("tiny", 1, 132, 0.0), ("tiny", 1, 256, 0.0),
    ("tiny", 1, 257, 0.0), ("tiny", 3, 300, 0.0), ("tiny", 1, 1, 0.0),
])
def test_forward_matches_oracle(shape, B, T, dup):
    cfg, m, P, oc, x_cpu, x, y_ref, rec, snaps = _oracle_run(shape, B, T, dup)
    y = m(x)
    torch.cuda.synchronize()
    flips = sum(int(near_threshold(r).sum()) for r in rec)
    assert flips == 0, f"{flips} near-threshold decisions in this seeded case; pick another seed"
    output_close(y, y_ref, "Bolt3Attn.forward")


def test_forward_is_deterministic():
    cfg, x_cpu, x = inputs("qwen3_4b", 2, 900, 0.3)
    m = bf16_module(cfg, 0)
    assert torch.equal(m(x), m(x))


@pytest.mark.parametrize("shape,prompt,n_dec", [("tiny", 300, 150), ("qwen3_4b", 512, 140)])
def test_decoder_matches_oracle(shape, prompt, n_dec):
    cfg = layer_cfg(shape)
    B = 2
    m = bf16_module(cfg, 0)
    P, oc = oracle_params(m), oracle_cfg_of(m, cfg)
    x = make_input(B, prompt + n_dec, cfg["dim"], dup=0.3, seed=3).to(torch.bfloat16)
    dec = LayerDecoderOracle(P, oc, B, BF16)
    st = Bolt3LayerState(m, B, "cuda")
    m_res = torch.zeros(B, m.HKV, m.HD, m.HD, device="cuda")
    steps = [(s, min(128, prompt - s)) for s in range(0, prompt, 128)] + [(prompt + i, 1) for i in range(n_dec)]
    outs, refs = [], []
    for pos, n in steps:
        h = x[:, pos:pos + n]
        outs.append(Bolt3Decoder.layer_step(m, st, h.cuda(), pos, m_res).float().cpu())
        refs.append(dec.step(h.float(), pos))
    flips = sum(int(near_threshold(r).sum()) for r in dec.record)
    assert flips == 0
    output_close(torch.cat(outs, 1), torch.cat(refs, 1), "decoder step outputs")
    # free-running state: the GPU's own bf16 projections feed it, so it is held to the output
    # tolerance; the 1e-4 state bound is checked teacher-forced in test_consolidation_teacher_forced
    scale = dec.m_res.abs().max().clamp_min(1e-30)
    assert ((m_res.cpu() - dec.m_res).abs().max() / scale).item() < 1e-2
