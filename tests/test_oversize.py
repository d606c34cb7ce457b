"""Decoder steps that push the pending chunk past C tokens (vsa_lm/config/bolt3.py:355-363, 406-425):
the chunk grows by the whole step and is later consolidated as one call of more than C tokens.
vsa_lm_b200/oversize.py takes these steps; they are checked here against the oracle's decoder, which
restates the reference's step, on the same projections, with the bank re-synced after every
consolidation (flips must be flagged near-ties and are counted), through the drop-in decoder API,
through the CUDA-graph runner and through the reference-format state conversion."""
import copy

import pytest
import torch

from helpers import (BF16, STATE_RTOL, FlipLedger, bf16_module, decoder_projections, oracle_cfg_of, oracle_params,
                     output_close, sync_bank)
from oracle import rope_at
from oracle.bolt3_oracle import LayerDecoderOracle
from vsa_lm_b200 import Bolt3Decoder, Bolt3LayerState
from vsa_lm_b200.bolt3 import AnchorKV
from vsa_lm_b200.model import Bolt3LM
from vsa_lm_b200.workloads import MODEL_SHAPES, layer_cfg, make_input, make_model_params

pytestmark = pytest.mark.gpu

# (position, tokens): a 100-token slice on top of 100 pending tokens (an oversize chunk of 200, which
# the one-token steps then attend to and the boundary at 328 consolidates on the fill path), a 120-token
# slice on top of 22 (a 142-token chunk; the ring chunk before it is consolidated natively), and steps
# to the boundary at 598, where the 142 tokens are consolidated on the full-bank path
STEPS = [(0, 100), (100, 100)] + [(200 + i, 1) for i in range(150)] + [(350, 120)] + \
        [(470 + i, 1) for i in range(140)]


@pytest.mark.parametrize("shape", ["qwen3_4b", "tiny"])
def test_oversize_chunks_match_oracle(shape):
    cfg = layer_cfg(shape)
    B = 2
    m = bf16_module(cfg, 0)
    P, oc = oracle_params(m), oracle_cfg_of(m, cfg)
    T = STEPS[-1][0] + STEPS[-1][1]
    x = make_input(B, T, cfg["dim"], dup=0.3, seed=8).to(torch.bfloat16)
    dec = LayerDecoderOracle(P, oc, B, BF16)
    st = Bolt3LayerState(m, B, "cuda")
    m_res = torch.zeros(B, m.HKV, m.HD, m.HD, device="cuda")
    ledger = FlipLedger(f"oversize chunks {shape}")
    HKV, HD = m.HKV, m.HD
    sizes = []
    for pos, n in STEPS:
        h = x[:, pos:pos + n].cuda()
        n_rec = len(dec.record)
        proj = decoder_projections(m, h, pos)
        got = Bolt3Decoder.layer_step(m, st, h, pos, m_res).float().cpu()
        ref = dec.step(h.float().cpu(), pos, proj=proj)
        output_close(got, ref, f"{shape} step of {n} at position {pos}")
        if len(dec.record) > n_rec:
            sizes.append(dec.record[-1]["l_tok"])
            bank = dict(st.bank)
            bank["m_res"] = m_res.view(B * HKV, HD, HD)
            ref_bank = dict(dec.sc, m_res=dec.m_res.view(B * HKV, HD, HD))
            rope = lambda c: rope_at(dec.sc["ak"][c], dec.sc["pm"][c], oc["inv_freq"], BF16)
            sync_bank(ledger, len(dec.record) - 1, dec.record[-1], bank, ref_bank, dec.n_filled, STATE_RTOL, rope)
    Bolt3Decoder.check_status([st])
    # the oversize chunks were consolidated whole (200 - 4 sinks on the fill path, then 142 on the full path)
    assert 196 in sizes and 142 in sizes and dec.record[-1]["kind"] == "full", sizes
    assert st.big_prev is None and st.prev_slot >= 0
    ledger.report()


def test_oversize_state_round_trip_and_graph_steps():
    """A hybrid model's state holding an oversize previous chunk: exported to the reference's format
    and imported, it decodes on bit-identically; and the graph runner (eager while the oversize chunk
    is in the window, replayed after its consolidation) matches eager steps bit for bit."""
    mcfg = dict(MODEL_SHAPES["small_lm"])
    model = Bolt3LM(**mcfg)
    model.load_state_dict(make_model_params(mcfg, 0), strict=True)
    model = model.to(device="cuda", dtype=torch.bfloat16).eval()
    dec = Bolt3Decoder(model)
    g = torch.Generator().manual_seed(4)
    ids = torch.randint(0, mcfg["vocab_size"], (2, 200), generator=g).cuda()
    steps = torch.randint(0, mcfg["vocab_size"], (2, 200), generator=g).cuda()
    sa, ka = Bolt3Decoder.blank_state(model, 2, "cuda", max_kv_len=512)
    dec.step(ids[:, :100], 0, sa, ka)
    dec.step(ids[:, 100:], 100, sa, ka)            # pending 100 + 100: an oversize chunk of 200
    assert all(st.big_prev is not None for st in ka if isinstance(st, Bolt3LayerState))
    ref_s, ref_kv = Bolt3Decoder.state_to_reference(model, sa, ka)
    assert ref_kv[0]["prev_kp"].shape[2] == 200
    sb, kb = Bolt3Decoder.state_from_reference(model, [s.clone() if s is not None else None for s in ref_s],
                                               ref_kv, "cuda")
    # the anchors' caches pass through the conversion as they are: give the copy caches of its own
    kb = [copy.deepcopy(c) if isinstance(c, AnchorKV) else c for c in kb]
    run = dec.step_graph(sb, kb)
    for i in range(steps.shape[1]):
        tok = steps[:, i:i + 1]
        ha, sa, ka = dec.step(tok, 200 + i, sa, ka)
        hb = run.step(tok, 200 + i)
        assert torch.equal(ha, hb), f"step {i}"
    assert run.captures >= 1                        # graphs again once the oversize chunk was consolidated
    for a, b in zip(sa, sb):
        if a is not None:
            assert torch.equal(a, b)


def test_continue_generate_after_unaligned_memorize():
    """The memory-bank flow the native decoder used to refuse: memorize a document whose length is
    not a multiple of C, then continue_generate a question that does not fit the pending chunk;
    greedy tokens equal those of eager steps through the same decoder (the oversize steps themselves
    are checked against the oracle above)."""
    mcfg = dict(MODEL_SHAPES["tiny_lm"])
    model = Bolt3LM(**mcfg)
    model.load_state_dict(make_model_params(mcfg, 0), strict=True)
    model = model.to(device="cuda", dtype=torch.bfloat16).eval()
    g = torch.Generator().manual_seed(12)
    doc = torch.randint(0, mcfg["vocab_size"], (1, 700), generator=g).cuda()
    q = torch.randint(0, mcfg["vocab_size"], (1, 100), generator=g).cuda()
    outs = []
    for graphs in (True, False):
        dec = Bolt3Decoder(model, cuda_graphs=graphs)
        states, kv = Bolt3Decoder.blank_state(model, 1, "cuda", max_kv_len=2048)
        states, kv, pos, traces = dec.memorize(doc, states, kv, 0)
        assert pos == 700
        toks, states, kv, pos = dec.continue_generate(q, states, kv, 700, 40, temperature=0.0)
        assert pos == 840 and toks.shape == (1, 40)
        outs.append(toks)
        Bolt3Decoder.check_status(kv)
    assert torch.equal(outs[0], outs[1])
