"""Pin the CPU oracle against the reference's own outputs (fixtures from tests/golden/make_golden.py)."""
import glob
import os

import pytest
import torch

from oracle import Store, forward, LayerDecoderOracle, oracle_cfg
from vsa_lm_b200.workloads import make_input, make_model_params, make_params

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")
FORWARD = sorted(p for p in glob.glob(os.path.join(GOLD, "*.pt")) if "decoder" not in p and "model" not in p)


def row_digest(y):
    y = y.double()
    w = torch.linspace(-1.0, 1.0, y.shape[-1], dtype=torch.float64)
    return torch.stack([y.sum(-1), (y * y).sum(-1), (y * w).sum(-1)], dim=-1)


def load(path):
    return torch.load(path, weights_only=False)


@pytest.mark.parametrize("path", FORWARD, ids=[os.path.basename(p)[:-3] for p in FORWARD])
def test_forward_matches_reference(path):
    g = load(path)
    cfg = dict(g["cfg"], qkv_bias=g["qkv_bias"])
    params = make_params(cfg, g["seed"])
    x = make_input(g["B"], g["T"], cfg["dim"], dup=g["dup"], seed=g["xseed"])
    assert torch.allclose(row_digest(x.view(-1, cfg["dim"])), g["x_digest"], rtol=0, atol=1e-9), \
        "seeded input generator is not reproducing the fixture's input"
    rec, snaps = [], []
    y = forward(params, oracle_cfg(cfg), x, Store("fp32"), record=rec, snapshots=snaps)
    calls = g["consolidations"]
    assert len(snaps) == len(calls)
    for i, (mine, ref) in enumerate(zip(snaps, calls)):
        assert mine["n_filled"] == ref["n_filled"]
        assert torch.equal(mine["act"], ref["act"]), f"act differs at consolidation {i}"
        torch.testing.assert_close(mine["mass"], ref["mass"], rtol=1e-6, atol=1e-6)
        for k in ("m_res", "ak", "av", "util", "pm"):
            if k in ref:
                torch.testing.assert_close(mine[k], ref[k], rtol=1e-4, atol=2e-5, msg=f"{k} @ cons {i}")
        assert abs(mine["m_res"].double().sum().item() - ref["m_res_sum"]) <= 1e-4 * (1 + ref["m_res_abs"])
    yf = y.view(-1, cfg["dim"])
    torch.testing.assert_close(yf[g["rows"]], g["y_rows"], rtol=1e-4, atol=2e-5)
    torch.testing.assert_close(row_digest(yf), g["y_digest"], rtol=1e-4, atol=1e-4)
    if "y" in g:
        torch.testing.assert_close(y, g["y"], rtol=1e-4, atol=2e-5)


def test_decoder_matches_reference():
    g = load(os.path.join(GOLD, "decoder_tiny_fp32.pt"))
    cfg = dict(g["cfg"])
    params = make_params(cfg, g["seed"])
    T = g["prompt_T"] + g["n_decode"]
    x = make_input(g["B"], T, cfg["dim"], dup=0.3, seed=g["xseed"])
    dec = LayerDecoderOracle(params, oracle_cfg(cfg), g["B"], Store("fp32"))
    outs = []
    for pos, n in g["steps"]:
        outs.append(dec.step(x[:, pos:pos + n], pos))
    out = torch.cat(outs, dim=1)
    torch.testing.assert_close(out[:1], g["outs"], rtol=1e-4, atol=2e-5)
    assert dec.n_filled == g["final"]["n_filled"]
    torch.testing.assert_close(dec.m_res, g["m_res"], rtol=1e-4, atol=2e-5)
    for k in ("ak", "av", "mass", "util", "pm"):
        torch.testing.assert_close(dec.sc[k], g["final"][k], rtol=1e-4, atol=2e-5)
    assert torch.equal(dec.sc["act"], g["final"]["act"])


def _model_oracle(g, store):
    from oracle import ModelDecoderOracle

    mcfg = g["mcfg"]
    params = make_model_params(mcfg, g["seed"])
    lcfg = oracle_cfg(dict(dim=mcfg["dim"], num_heads=mcfg["num_heads"], num_kv_heads=mcfg["num_kv_heads"],
                           head_dim=mcfg["head_dim"], eps=mcfg["eps"], rope_theta=mcfg["rope_theta"],
                           qk_norm=mcfg["qk_norm"]))
    return lambda: ModelDecoderOracle(params, lcfg, g["layer_types"], 1, store, mcfg["eps"])


def test_model_decoder_matches_reference():
    """The model-level decode oracle (embedding, norms, Bolt-3 layers, softmax anchor, MLP) against
    the reference UniversalVSALM under Bolt3Decoder: prefill, one-token steps, and the memory-bank
    flow (memorize twice, forget, greedy continue_generate)."""
    g = load(os.path.join(GOLD, "model_tiny_lm_fp32.pt"))
    new = _model_oracle(g, Store("fp32"))
    ids = g["ids"]
    T = ids.shape[1] - g["logits"].shape[1] + 1
    o = new()
    h, pos = o.feed(ids[:, :T], 0)
    hs, lg = [h[:, -1]], [o.logits(h[:, -1])]
    for i in range(g["logits"].shape[1] - 1):
        h = o.step(ids[:, T + i:T + i + 1], T + i)
        hs.append(h[:, -1])
        lg.append(o.logits(h[:, -1]))
    torch.testing.assert_close(torch.stack(hs, 1), g["h_last"], rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(torch.stack(lg, 1), g["logits"], rtol=1e-4, atol=1e-4)

    o = new()
    doc, na = g["doc"], g["pos_a"]
    pos_a, _ = o.memorize(doc[:, :na], 0)
    pos_b, traces = o.memorize(doc[:, na:], pos_a)
    assert (pos_a, pos_b) == (g["pos_a"], g["pos_b"])
    vsa = [i for i, t in enumerate(g["layer_types"]) if t == "vsa"]
    for i in vsa:
        torch.testing.assert_close(o.m_res(i), g["states_after_b"][i], rtol=1e-4, atol=1e-5)
        assert traces[i][0] == g["traces"][i][0]
        torch.testing.assert_close(traces[i][1], g["traces"][i][1], rtol=1e-4, atol=1e-5)
    o.forget(traces, pos_b)
    for i in vsa:
        torch.testing.assert_close(o.m_res(i), g["states_after_forget"][i], rtol=1e-4, atol=1e-5)
    h, pos = o.feed(g["q_ids"], pos_b)
    toks = []
    for _ in range(g["gen"].shape[1]):
        nxt = o.logits(h[:, -1]).argmax(-1, keepdim=True)
        toks.append(nxt)
        h = o.step(nxt, pos)
        pos += 1
    assert torch.equal(torch.cat(toks, 1), g["gen"])
    assert pos == g["gen_pos"]
    for i in vsa:
        torch.testing.assert_close(o.m_res(i), g["states_final"][i], rtol=1e-4, atol=1e-5)
