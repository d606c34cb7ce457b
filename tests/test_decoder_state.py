"""Decoder state in the reference's format (vsa_lm/config/bolt3.py:302-319, :343-425): export from
the native decoder, import into it, and continue decoding."""
import pytest
import torch

from helpers import BF16, bf16_module, oracle_cfg_of, oracle_params, output_close
from oracle.bolt3_oracle import LayerDecoderOracle
from vsa_lm_b200 import Bolt3Decoder, Bolt3LayerState
from vsa_lm_b200.workloads import layer_cfg, make_input

pytestmark = pytest.mark.gpu


class _Model:
    """The parts of a model the state conversions read: blocks with a .vsa Bolt-3 layer."""

    def __init__(self, layer):
        blk = torch.nn.Module()
        blk.vsa = layer
        self.blocks = [blk]


def _run(m, st, m_res, x, steps):
    return [Bolt3Decoder.layer_step(m, st, x[:, p:p + n].cuda(), p, m_res).float().cpu() for p, n in steps]


@pytest.mark.parametrize("shape,prompt", [("qwen3_4b", 300), ("tiny", 260)])
def test_state_round_trip_continues_identically(shape, prompt):
    """Export after a prefill and some decode steps, import, and decode on across a consolidation:
    the imported state must produce bit-identical outputs and M_res."""
    cfg = layer_cfg(shape)
    B = 2
    m = bf16_module(cfg, 0)
    model = _Model(m)
    x = make_input(B, prompt + 180, cfg["dim"], dup=0.3, seed=5).to(torch.bfloat16)
    st = Bolt3LayerState(m, B, "cuda")
    m_res = torch.zeros(B, m.HKV, m.HD, m.HD, device="cuda")
    head = [(s, min(128, prompt - s)) for s in range(0, prompt, 128)] + [(prompt + i, 1) for i in range(20)]
    _run(m, st, m_res, x, head)
    states, ref = Bolt3Decoder.state_to_reference(model, [m_res.clone()], [st])
    d = ref[0]
    assert d["prev_kp"].shape[2] == m.C and d["cur_kp"].shape[2] == (prompt + 20) % m.C
    assert d["ak"].shape == (B * m.HKV, m.S, m.HD) and d["act"].dtype == torch.bool
    assert d["cur_pos"].shape == (1, 1, d["cur_kp"].shape[2])
    states2, caches2 = Bolt3Decoder.state_from_reference(model, states, ref, "cuda")
    tail = [(prompt + 20 + i, 1) for i in range(150)]  # crosses at least one consolidation
    a = _run(m, st, m_res, x, tail)
    b = _run(m, caches2[0], states2[0], x, tail)
    for i, (u, v) in enumerate(zip(a, b)):
        assert torch.equal(u, v), f"outputs differ at tail step {i}"
    assert torch.equal(m_res, states2[0])


def test_import_reference_state_matches_oracle_continuation():
    """The oracle decoder's own (reference-format) state, imported into the native decoder, decodes
    on like the oracle does."""
    cfg = layer_cfg("qwen3_4b")
    B = 2
    m = bf16_module(cfg, 0)
    model = _Model(m)
    P, oc = oracle_params(m), oracle_cfg_of(m, cfg)
    prompt = 300
    x = make_input(B, prompt + 40, cfg["dim"], dup=0.3, seed=6).to(torch.bfloat16)
    dec = LayerDecoderOracle(P, oc, B, BF16)
    for s in range(0, prompt, 128):
        dec.step(x[:, s:min(prompt, s + 128)].float(), s)
    # the oracle keeps the reference dict (positions as 1-D tensors); move it to CUDA in the model dtype
    d = {}
    for k, v in dec.sc.items():
        if v is None:
            d[k] = None
        elif k.endswith("_pos"):
            d[k] = v.view(1, 1, -1).cuda()
        elif k in ("mass", "util", "pm") or v.dtype == torch.bool:
            d[k] = v.cuda()
        else:
            d[k] = v.to(torch.bfloat16).cuda()
    d["n_filled"] = dec.n_filled
    states, caches = Bolt3Decoder.state_from_reference(model, [dec.m_res.clone()], [d], "cuda")
    st, m_res = caches[0], states[0]
    outs, refs = [], []
    for i in range(40):
        p = prompt + i
        h = x[:, p:p + 1]
        outs.append(Bolt3Decoder.layer_step(m, st, h.cuda(), p, m_res).float().cpu())
        refs.append(dec.step(h.float(), p))
    output_close(torch.cat(outs, 1), torch.cat(refs, 1), "decode after importing the oracle's state")
