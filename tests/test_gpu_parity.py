"""Parity of the CUDA path (through the C-ABI) with the CPU oracle, on seeded inputs.

Tolerances (the north star's): bf16 outputs within rtol 2e-2 (atol 2e-2 x RMS for near-zero
elements); fp32 state (M_res, pm, util) within 1e-4 relative, mass and act exactly; merge / evict
decisions identical. A consolidation may differ from the oracle's only where `decision_ties` flags a
decision that rounding can change (a cosine within 1e-3 of 0.88 / 0.80, or distinct ranking keys
within 1e-5 relative at a decision boundary); such differences are counted, printed with their
reason and bounded at 2% of chain-steps. Banks are compared up to a permutation of slots: a near-tie
that only reorders slots changes no output.

Every chunk of every case is compared:
- teacher-forced: each native consolidation starts from the oracle's pre-state;
- re-synced forward: the native scan runs one consolidation per launch on the oracle's projections;
  after each, its bank is checked and then replaced by the oracle's, so only the attention chunk
  that reads the snapshot of a counted flip is left out;
- product forward (Bolt3Attn.forward itself): the oracle runs on the GPU's own projections, so both
  sides consolidate the same inputs; a chain may leave the comparison only after a flagged decision;
- decoder: the native state is checked and re-synced after every consolidation, so every step's
  output is compared.
"""
import pytest
import torch

from helpers import (ATOL_RMS, BF16, RTOL, STATE_RTOL, FlipLedger, bf16_module, chain_of, decision_ties,
                     decoder_projections, inputs, m_res_error, match_slots, oracle_cfg_of, oracle_params,
                     output_close, sync_bank)
from oracle import LayerDecoderOracle, forward, gamma_delta, project, rope_at
from vsa_lm_b200 import Bolt3Decoder, Bolt3LayerState
from vsa_lm_b200 import kernels as K
from vsa_lm_b200.workloads import layer_cfg, make_input

pytestmark = pytest.mark.gpu
C = 128


@pytest.mark.parametrize("shape,split", [("config0", False), ("qwen3_4b", False), ("qwen3_4b", True)])
def test_prep_matches_oracle(shape, split):
    """Fused projection with one prep call (the decoder's form), or the k/v/beta and q/eta row blocks
    as two GEMMs with one prep call each (the prefill's form)."""
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
    common = dict(B=B, T=T, H=H, HKV=HKV, HD=HD, inv_freq=c["inv_freq"], eps=m.eps, q_norm_w=c["qn"],
                  k_norm_w=c["kn"], pos0=0, q_head_stride=T, q_t_off=0, k_head_stride=T, k_t_off=0)
    if split:
        x2 = x.reshape(B * T, -1)
        K.prep(m.project(x2, f, "kv"), cols=f.cols_kv, parts=2, k_raw=k_raw, k_rope=k_rope, v=v, beta=beta, **common)
        K.prep(m.project(x2, f, "q"), cols=f.cols_q, parts=1, q_raw=q_raw, q_rope=q_rope, eta=eta, **common)
    else:
        K.prep(proj, cols=f.cols, q_raw=q_raw, q_rope=q_rope, eta=eta, k_raw=k_raw, k_rope=k_rope, v=v, beta=beta,
               **common)
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
    y_ref, yh_ref = forward(P, oc, x_cpu, BF16, record=rec, snapshots=snaps, return_y_heads=True)
    return cfg, m, P, oc, x_cpu, x, y_ref, yh_ref, rec, snaps


@pytest.mark.parametrize("shape,B,T,dup", [("config0", 1, 1024, "chunks"), ("qwen3_4b", 2, 1024, 0.3),
                                           ("tiny", 2, 1152, 0.3), ("llama3_8b", 1, 896, 0.2)])
def test_consolidation_teacher_forced(shape, B, T, dup):
    """Each native consolidation, fed the oracle's pre-state and inputs, reproduces the oracle's
    post-state: the bank as a set of slots (act, mass exact; pm, util 1e-4; ak, av one bf16 step) and
    M_res to 1e-4 of its largest element."""
    cfg, m, P, oc, x_cpu, x, y_ref, yh_ref, rec, snaps = _oracle_run(shape, B, T, dup)
    qr, kr, vo, bo, eo = project(P, oc, x_cpu, BF16)
    pos = torch.arange(T, dtype=torch.float32)
    kp = rope_at(kr, pos, oc["inv_freq"], BF16)
    gam = gamma_delta(P["log_gamma"]).cuda()
    inv = oc["inv_freq"].cuda()
    ledger = FlipLedger(f"teacher-forced {shape} B{B} T{T}")
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
        got = dict(ak=ak, av=av, mass=mass, util=util, pm=pmv, act=act)
        flags = ledger.step(rec[i], mass.shape[0])
        for c in range(mass.shape[0]):
            perm, why = match_slots(chain_of(got, c), chain_of(post, c))
            if perm is not None:
                err = m_res_error(m_res[c], post["m_res"][c])
                if err >= STATE_RTOL:
                    perm, why = None, f"M_res differs by {err:.2e} of its max"
            if perm is None:
                ledger.flip(i, c, why, bool(flags[c]))
    ledger.report()


def _upload_oracle_inputs(m, qr, kr, vo, bo, eo, inv_freq, T):
    """The oracle's projections and RoPE'd q/k, in the head-major layouts bolt3_prep writes."""
    b = qr.shape[0]
    pos = torch.arange(T, dtype=torch.float32)
    qp, kp = rope_at(qr, pos, inv_freq, BF16), rope_at(kr, pos, inv_freq, BF16)
    cu = lambda t, dt=torch.bfloat16: t.to(device="cuda", dtype=dt).contiguous()
    H, HKV, HD = m.H, m.HKV, m.HD
    return dict(q_rope=cu(qp.reshape(b * H, T, HD)), q_raw=cu(qr.reshape(b * H, T, HD)),
                k_raw=cu(kr.reshape(b * HKV, T, HD)), k_rope=cu(kp.reshape(b * HKV, T, HD)),
                v=cu(vo.reshape(b * HKV, T, HD)), beta=cu(bo.reshape(b * HKV, T), torch.float32),
                eta=cu(eo.reshape(b * H, T), torch.float32))


def _compare_chunks(yh, yh_ref, G, excluded: set, what: str) -> tuple[int, int]:
    """Compare the attention output y [b, T, H, HD] with the oracle's [b, H, T, HD], chain by chain
    (the G heads of one KV head of one sequence) and chunk by chunk, except (chunk, chain) pairs in
    `excluded`. Returns (compared, total) chain-chunks."""
    b, T, H, HD = yh.shape
    HKV = H // G
    rms = yh_ref.float().pow(2).mean().sqrt().item()
    got = yh.float().cpu().permute(0, 2, 1, 3)
    n_chunks = (T + C - 1) // C
    compared = 0
    for r in range(n_chunks):
        for c in range(b * HKV):
            if (r, c) in excluded:
                continue
            bi, h = divmod(c, HKV)
            g_ = got[bi, h * G:(h + 1) * G, r * C:(r + 1) * C]
            f_ = yh_ref[bi, h * G:(h + 1) * G, r * C:(r + 1) * C].float()
            bad = (g_ - f_).abs() > RTOL * f_.abs() + ATOL_RMS * rms
            assert not bad.any(), (f"{what}: chunk {r}, chain {c}: {int(bad.sum())} elements outside tolerance, "
                                   f"max |diff| {(g_ - f_).abs().max().item():.3e} (rms {rms:.3e})")
            compared += 1
    return compared, n_chunks * b * HKV


@pytest.mark.parametrize("shape,B,T,dup", [
    ("config0", 1, 1024, "chunks"),
    ("qwen3_4b", 2, 1024, 0.3),
    ("llama3_8b", 1, 896, 0.2),     # configs[4]'s shape: no qk-norm, RoPE theta 5e5, D 4096
    ("tiny", 1, 8960, 0.2),         # 68 consolidations
    ("tiny", 2, 700, 0.3),
])
def test_forward_resynced_matches_oracle(shape, B, T, dup):
    """The scan and attention kernels on the oracle's projections, one consolidation per scan
    launch with the bank re-synced in between: every chunk of every chain is compared, except a
    chunk that reads the snapshot of a counted flip."""
    cfg, m, P, oc, x_cpu, x, y_ref, yh_ref, rec, snaps = _oracle_run(shape, B, T, dup)
    H, HKV, HD, G = m.H, m.HKV, m.HD, m.G
    inp = _upload_oracle_inputs(m, *project(P, oc, x_cpu, BF16), oc["inv_freq"], T)
    c_ = m.fused("cuda").consts
    nch, n_cons = B * HKV, len(snaps)
    ws = torch.empty(max(1, K.prefill_workspace_bytes(nch, T, HD)), dtype=torch.uint8, device="cuda")
    sn = K.snapshot_views(ws, nch, n_cons, HD) if n_cons else None
    bank = K.new_bank(nch, HD, "cuda")
    status = K.DeviceStatus("cuda")
    ledger = FlipLedger(f"re-synced forward {shape} B{B} T{T}")
    excluded = set()
    for i in range(n_cons):
        K.consolidate(n_chains=nch, hkv=HKV, HD=HD, bank=bank, init_blank=i == 0, kr=inp["k_raw"], kp=inp["k_rope"],
                      v=inp["v"], beta=inp["beta"], chain_tokens=T, token0=i * C, step_tokens=C,
                      skip0=4 if i == 0 else 0, chunk_len=C, pos0=0, n_steps=1, kappa=c_["kappa"],
                      gamma=c_["gamma"], inv_freq=c_["inv_freq"], snaps=sn, snap0=i, status=status)
        for c in sync_bank(ledger, i, rec[i], bank, snaps[i], snaps[i]["n_filled"], STATE_RTOL):
            excluded.add((i + 2, c))
    y = torch.empty(B, T, H, HD, dtype=torch.bfloat16, device="cuda")
    K.attend_prefill(n_chains=nch, hkv=HKV, G=G, HD=HD, T=T, q_rope=inp["q_rope"], q_raw=inp["q_raw"],
                     eta=inp["eta"], k_rope=inp["k_rope"], v=inp["v"], snaps=sn, n_cons=n_cons,
                     kappa=c_["kappa"], coef=c_["coef"], res_w=c_["res_w"], eps=m.eps, y=y, status=status)
    status.arm("re-synced forward")
    status.check(block=True)
    done, total = _compare_chunks(y, yh_ref, G, excluded, f"re-synced forward {shape}")
    ledger.report()
    print(f"compared {done} of {total} chain-chunks")
    assert total - done <= len(ledger.flips)


def _gpu_projections(m, x):
    """The projections Bolt3Attn.forward computes on the GPU for x, in the oracle's layouts."""
    p, prep_q = m._prepare(x)
    prep_q()
    torch.cuda.synchronize()
    b, T = p.b, p.T
    H, HKV, HD = m.H, m.HKV, m.HD
    f = lambda t, *shape: t.float().cpu().view(*shape)
    return (f(p.q_raw, b, H, T, HD), f(p.k_raw, b, HKV, T, HD), f(p.v, b, HKV, T, HD), f(p.beta, b, HKV, T),
            f(p.eta, b, H, T))


@pytest.mark.parametrize("shape,B,T,dup", [
    ("config0", 1, 1024, "chunks"),
    ("qwen3_4b", 2, 1024, 0.3),
    ("llama3_8b", 1, 896, 0.2),
    ("tiny", 1, 8960, 0.2),
    ("tiny", 2, 700, 0.3),
    ("tiny", 1, 100, 0.0), ("tiny", 1, 128, 0.0), ("tiny", 1, 132, 0.0), ("tiny", 1, 256, 0.0),
    ("tiny", 1, 257, 0.0), ("tiny", 3, 300, 0.0), ("tiny", 1, 1, 0.0),
    ("llama3_8b", 1, 131072, 0.2),  # configs[4] itself: 1022 consolidations, mean positions up to 1.3e5
])
def test_forward_matches_oracle(shape, B, T, dup):
    """Bolt3Attn.forward itself (projections, segmented scan overlapped with the attention,
    o_proj) against the oracle run on the GPU's own projections. Every chunk of every chain is
    compared; a chain may leave the comparison only at a chunk that reads a bank formed after a
    flagged decision of that chain, and the output rows of a sequence are compared wherever all its
    chains still are."""
    cfg, x_cpu, x = inputs(shape, B, T, dup)
    m = bf16_module(cfg, 0)
    P, oc = oracle_params(m), oracle_cfg_of(m, cfg)
    rec = []
    y_ref, yh_ref = forward(P, oc, x_cpu, BF16, record=rec, return_y_heads=True, proj=_gpu_projections(m, x))
    yh = m._attention_heads(x)
    out = m(x)
    m.check_status()
    HKV, G = m.HKV, m.G
    flags = [decision_ties(r) for r in rec]
    # chain c may deviate from chunk r on only if a consolidation j <= r - 2 of chain c is flagged
    rms = yh_ref.float().pow(2).mean().sqrt().item()
    got = yh.float().cpu().permute(0, 2, 1, 3)
    n_chunks = (T + C - 1) // C
    gone = {}
    for r in range(n_chunks):
        for c in range(B * HKV):
            if c in gone:
                continue
            bi, h = divmod(c, HKV)
            g_ = got[bi, h * G:(h + 1) * G, r * C:(r + 1) * C]
            f_ = yh_ref[bi, h * G:(h + 1) * G, r * C:(r + 1) * C].float()
            if ((g_ - f_).abs() > RTOL * f_.abs() + ATOL_RMS * rms).any():
                assert any(bool(flags[j][c]) for j in range(0, r - 1)), \
                    f"chunk {r}, chain {c} deviates with no flagged decision before it"
                gone[c] = r
    total = n_chunks * B * HKV
    left_out = sum(n_chunks - r for r in gone.values())
    print(f"{shape} B{B} T{T}: {total - left_out} of {total} chain-chunks compared; chains that left after a "
          f"flagged decision: {gone}")
    # o_proj output: rows of sequences whose chains are all still compared
    out_rms = y_ref.float().pow(2).mean().sqrt().item()
    for bi in range(B):
        end = min([gone[c] for c in range(bi * HKV, (bi + 1) * HKV) if c in gone] + [n_chunks]) * C
        if end:
            g_, f_ = out[bi, :end].float().cpu(), y_ref[bi, :end].float()
            bad = (g_ - f_).abs() > RTOL * f_.abs() + ATOL_RMS * out_rms
            assert not bad.any(), f"o_proj output of sequence {bi}: {int(bad.sum())} elements outside tolerance"
    # each chain that left is one flip of a flagged decision; bounded like the other tests' flips
    assert len(gone) <= max(1, 0.02 * len(rec) * B * HKV), f"{len(gone)} chains left the comparison"


def test_forward_is_deterministic():
    cfg, x_cpu, x = inputs("qwen3_4b", 2, 900, 0.3)
    m = bf16_module(cfg, 0)
    assert torch.equal(m(x), m(x))


@pytest.mark.parametrize("shape,prompt,n_dec,tps", [("tiny", 300, 250, 1), ("qwen3_4b", 512, 140, 1),
                                                    ("qwen3_4b", 384, 136, 4), ("llama3_8b", 384, 150, 1)])
def test_decoder_matches_oracle(shape, prompt, n_dec, tps):
    """Decoder (prefill slices + decode steps of `tps` tokens: G * tps <= 16 query rows take the
    decode-step kernels) against the oracle's decoder run on the same projections. After every
    consolidation the native bank is compared with the oracle's and re-synced to it (flips must be
    flagged and are counted), so every step's output is compared."""
    cfg = layer_cfg(shape)
    B = 2
    m = bf16_module(cfg, 0)
    P, oc = oracle_params(m), oracle_cfg_of(m, cfg)
    x = make_input(B, prompt + n_dec, cfg["dim"], dup=0.3, seed=3).to(torch.bfloat16)
    dec = LayerDecoderOracle(P, oc, B, BF16)
    st = Bolt3LayerState(m, B, "cuda")
    m_res = torch.zeros(B, m.HKV, m.HD, m.HD, device="cuda")
    steps = [(s, min(128, prompt - s)) for s in range(0, prompt, 128)] + \
        [(prompt + i, tps) for i in range(0, n_dec, tps)]
    ledger = FlipLedger(f"decoder {shape} prompt {prompt} steps of {tps}")
    HKV, HD = m.HKV, m.HD
    outs, refs = [], []
    for pos, n in steps:
        h = x[:, pos:pos + n].cuda()
        n_rec = len(dec.record)
        proj = decoder_projections(m, h, pos)
        got = Bolt3Decoder.layer_step(m, st, h, pos, m_res).float().cpu()
        ref = dec.step(h.float().cpu(), pos, proj=proj)
        outs.append(got)
        refs.append(ref)
        output_close(got, ref, f"decoder step at position {pos}")
        if len(dec.record) > n_rec:
            bank = dict(st.bank)
            bank["m_res"] = m_res.view(B * HKV, HD, HD)
            ref_bank = dict(dec.sc, m_res=dec.m_res.view(B * HKV, HD, HD))
            rope = lambda c: rope_at(dec.sc["ak"][c], dec.sc["pm"][c], oc["inv_freq"], BF16)
            sync_bank(ledger, len(dec.record) - 1, dec.record[-1], bank, ref_bank, dec.n_filled, STATE_RTOL, rope)
    Bolt3Decoder.check_status([st])
    assert len(dec.record) >= 3, "case must reach the full-bank path"
    output_close(torch.cat(outs, 1), torch.cat(refs, 1), "decoder step outputs")
    ledger.report()
