"""Generate the golden fixtures of the Bolt-3 hot path from the real reference module.

Runs the reference `vsa_lm.config.bolt3` (Bolt3Attn.forward, Bolt3Decoder.step) on the CPU in fp32
on seeded inputs and writes the outputs, the per-consolidation bank states and the merge/evict
decisions to `tests/golden/*.pt`. The reference source tree (the vsa_lm checkout, given by the
VSA_LM_REF environment variable) is needed only here; the fixtures travel with the repository.

    VSA_LM_REF=<vsa_lm checkout> PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
sys.dont_write_bytecode = True
REF = os.environ.get("VSA_LM_REF")
if not REF:
    sys.exit("set VSA_LM_REF to the reference vsa_lm source tree")
sys.path.insert(0, REF)

from vsa_lm.config.bolt3 import Bolt3Attn, Bolt3Decoder  # noqa: E402  (reference)

from vsa_lm_b200.workloads import (MODEL_SHAPES, layer_cfg, make_input, make_model_params,  # noqa: E402
                                   make_params)

torch.set_num_threads(max(1, os.cpu_count() or 1))

BANK_KEYS = ("ak", "av", "mass", "util", "pm", "act")


def build_ref(cfg, seed, qkv_bias=False):
    cfg = dict(cfg, qkv_bias=qkv_bias)
    m = Bolt3Attn(cfg, max_T=2048)
    params = make_params(cfg, seed)
    missing, unexpected = m.load_state_dict(params, strict=False)
    assert not unexpected, unexpected
    assert all(k.startswith("rope.") for k in missing), missing
    return m.eval(), params


def instrument(m, keep=()):
    """Record every _consolidate_functional call's outputs on the reference module: the full bank
    and M_res for the call indices in `keep`, float64 digests for the others."""
    calls = []
    orig = m._consolidate_functional

    def wrapped(*args, **kw):
        out = orig(*args, **kw)
        ak, av, mass, util, pm, act, m_res, n_filled = out
        rec = {"n_filled": int(n_filled), "mass": mass.clone(), "act": act.clone(),
               "util_sum": util.double().sum().item(), "pm_sum": pm.double().sum().item(),
               "m_res_sum": m_res.double().sum().item(), "m_res_abs": m_res.double().abs().sum().item(),
               "ak_sum": ak.double().sum().item(), "av_sum": av.double().sum().item()}
        if len(calls) in keep:
            rec.update(ak=ak.clone(), av=av.clone(), util=util.clone(), pm=pm.clone(),
                       m_res=m_res.clone())
        calls.append(rec)
        return out

    m._consolidate_functional = wrapped
    return calls


def row_digest(y):
    """Per-row (sum, sum of squares, index-weighted sum) in float64: a checksum of every row."""
    y = y.double()
    w = torch.linspace(-1.0, 1.0, y.shape[-1], dtype=torch.float64)
    return torch.stack([y.sum(-1), (y * y).sum(-1), (y * w).sum(-1)], dim=-1)


def forward_case(name, shape, B, T, dup, seed=0, xseed=1, qkv_bias=False, keep=(),
                 full_y=False, sample_rows=64):
    cfg = layer_cfg(shape)
    m, params = build_ref(cfg, seed, qkv_bias)
    x = make_input(B, T, cfg["dim"], dup=dup, seed=xseed)
    calls = instrument(m, keep)
    with torch.no_grad():
        y = m(x)
    g = torch.Generator().manual_seed(1234)
    rows = torch.sort(torch.randperm(B * T, generator=g)[:sample_rows]).values
    out = {
        "kind": "forward", "shape": shape, "cfg": cfg, "B": B, "T": T, "dup": dup, "seed": seed,
        "xseed": xseed, "qkv_bias": qkv_bias, "x_digest": row_digest(x.view(B * T, -1)),
        "y_digest": row_digest(y.view(B * T, -1)), "rows": rows,
        "y_rows": y.view(B * T, -1)[rows].clone(), "consolidations": calls,
    }
    if full_y:
        out["y"] = y.clone()
    torch.save(out, os.path.join(HERE, f"{name}.pt"))
    print(name, "consolidations", len(calls), "y |max|", y.abs().max().item())


def decoder_case(name, shape, B, prompt_T, n_decode, seed=0, xseed=3):
    """Drive the reference Bolt3Decoder.step over one Bolt-3 layer and record (h_in, attn_out).

    The model shell is a single block whose Bolt3Attn output is captured with hooks: the layer input
    is norm1's output, the branch output is o_proj's output (bolt3.py:342-404).
    """
    import torch.nn as nn

    cfg = layer_cfg(shape)
    ly, params = build_ref(cfg, seed)
    D = cfg["dim"]

    class Blk(nn.Module):
        def __init__(self):
            super().__init__()
            self.norm1 = nn.Identity()
            self.vsa = ly
            self.norm2 = nn.Identity()
            self.mlp = lambda x: torch.zeros_like(x)

    class Shell(nn.Module):
        def __init__(self):
            super().__init__()
            self.blocks = nn.ModuleList([Blk()])
            self.embed_tokens = nn.Embedding.from_pretrained(table)
            self.norm = nn.Identity()
            self.config = {"max_T": 2048, "bolt3_C": 128}

    x = make_input(B, prompt_T + n_decode, D, dup=0.3, seed=xseed)
    table = x.reshape(-1, D)                      # token id = row of x: embed_tokens returns x
    ids = torch.arange(B * (prompt_T + n_decode)).view(B, -1)
    model = Shell()
    dec = Bolt3Decoder(model)
    outs = []
    ly.o_proj.register_forward_hook(lambda mod, inp, o: outs.append(o.detach().clone()))
    calls = instrument(ly)
    states, kv = Bolt3Decoder.blank_state(model, B, "cpu")
    steps, pos = [], 0
    with torch.no_grad():
        for s in range(0, prompt_T, 128):                              # prefill (bolt3.py:454-456)
            e = min(prompt_T, s + 128)
            steps.append((pos, e - s))
            dec.step(ids[:, s:e], pos, states, kv)
            pos = e
        for i in range(n_decode):
            steps.append((pos, 1))
            dec.step(ids[:, pos:pos + 1], pos, states, kv)
            pos += 1
    sc = kv[0]
    final = {k: (sc[k].clone() if torch.is_tensor(sc[k]) else sc[k]) for k in BANK_KEYS + ("n_filled",)}
    torch.save({
        "kind": "decoder", "shape": shape, "cfg": cfg, "B": B, "prompt_T": prompt_T,
        "n_decode": n_decode, "seed": seed, "xseed": xseed, "steps": steps,
        "x_digest": row_digest(x.view(-1, D)), "outs": torch.cat(outs, dim=1)[:1].clone(),
        "m_res": states[0].clone(), "final": final, "consolidations": calls,
    }, os.path.join(HERE, f"{name}.pt"))
    print(name, "steps", len(steps), "consolidations", len(calls))


def model_case(name, shape="tiny_lm", seed=0, prompt_T=300, n_steps=24, doc_a=768, doc_b=256, question=50,
               n_new=12):
    """A whole hybrid model (reference UniversalVSALM with is_bolt3=True) under the reference
    Bolt3Decoder: prefill + teacher-forced one-token steps (final hidden states and logits), then
    the memory-bank flow: memorize document A from a blank state, memorize B after it, forget B,
    continue_generate a question greedily (bolt3.py:449-557). Document A is long enough for full-bank
    consolidations to write M_res before B starts, so that forgetting B leaves a nonzero state."""
    from vsa_lm.config.standard import UniversalVSALM

    mcfg = dict(MODEL_SHAPES[shape])
    model = UniversalVSALM(**mcfg, max_T=2048, chunk_size=128, is_bolt3=True, bolt3_S=128, bolt3_C=128)
    params = make_model_params(mcfg, seed)
    missing, unexpected = model.load_state_dict(params, strict=False)
    assert not unexpected and all(".rope." in k for k in missing), (missing, unexpected)
    model.eval()
    dec = Bolt3Decoder(model)
    V = mcfg["vocab_size"]
    g = torch.Generator().manual_seed(seed + 77)
    ids = torch.randint(0, V, (1, prompt_T + n_steps), generator=g)
    out = {"kind": "model", "shape": shape, "mcfg": mcfg, "seed": seed, "ids": ids,
           "layer_types": model.config["layer_types"]}
    clones = lambda xs: [x.clone() if x is not None else None for x in xs]
    with torch.no_grad():
        h, states, kv = dec.prefill(ids[:, :prompt_T])
        hs, logits = [h[:, -1].clone()], [model.lm_head(h[:, -1]).clone()]
        for i in range(n_steps):
            p0 = prompt_T + i
            h, states, kv = dec.step(ids[:, p0:p0 + 1], p0, states, kv)
            hs.append(h[:, -1].clone())
            logits.append(model.lm_head(h[:, -1]).clone())
        out.update(h_last=torch.stack(hs, 1), logits=torch.stack(logits, 1))
        doc = torch.randint(0, V, (1, doc_a + doc_b), generator=g)
        q_ids = torch.randint(0, V, (1, question), generator=g)
        states, kv = Bolt3Decoder.blank_state(model, 1, "cpu", max_kv_len=2048)
        states, kv, pos_a, _ = dec.memorize(doc[:, :doc_a], states, kv, 0)
        states, kv, pos_b, traces = dec.memorize(doc[:, doc_a:], states, kv, pos_a)
        after_b = clones(states)
        states = dec.forget(traces, states, next_pos=pos_b)
        toks, states, kv, pos = dec.continue_generate(q_ids, states, kv, pos_b, n_new, temperature=0.0)
        out.update(doc=doc, q_ids=q_ids, pos_a=pos_a, pos_b=pos_b, states_after_b=clones(after_b),
                   traces=[None if t is None else (t[0], t[1].clone()) for t in traces],
                   states_after_forget=clones(dec.forget(traces, clones(after_b), pos_b)),
                   gen=toks.clone(), gen_pos=pos, states_final=clones(states))
    torch.save(out, os.path.join(HERE, f"{name}.pt"))
    print(name, "layers", out["layer_types"], "generated", toks.tolist())


if __name__ == "__main__":
    forward_case("config0_fp32", "config0", 1, 1024, "chunks", keep=(0, 2, 5))
    forward_case("tiny_ragged_bias_fp32", "tiny", 2, 700, 0.3, seed=2, xseed=5, qkv_bias=True,
                 keep=(3,))
    forward_case("qwen_T1024_fp32", "qwen3_4b", 1, 1024, 0.3, seed=3, xseed=7)
    for T in (100, 128, 132, 256, 257, 300):
        forward_case(f"tiny_T{T}_fp32", "tiny", 1, T, 0.0, seed=4, xseed=T, keep=(0,),
                     full_y=T <= 132)
    decoder_case("decoder_tiny_fp32", "tiny", 2, 300, 150)
    model_case("model_tiny_lm_fp32")
