"""The decoder API of the drop-in Bolt3Decoder on a whole hybrid model (two Bolt-3 layers and one
softmax anchor): step / prefill, generate_batch, and the memory-bank flow (memorize, the state
pickled in the reference's format, forget, continue_generate), each against the model-level oracle
(oracle/model_oracle.py, pinned to the reference by tests/test_oracle_golden.py).

The oracle's Bolt-3 layers run in lockstep with the native ones (LockstepTap): each layer step is
checked on the projections the GPU computed for it, and after each consolidation the native bank is
checked and re-synced to the oracle's (flips must be flagged near-ties and are counted), so
rounding differences never accumulate into different histories. The oracle then runs the rest of
the model (embedding, softmax anchor with its KV cache, MLP, norms) itself. Greedy decoding is
compared token by token with the oracle fed the native tokens (teacher forcing): the native token
must be the oracle's argmax unless the oracle's two best logits are within the output tolerance of
each other.
"""
import io

import pytest
import torch

from helpers import ATOL_RMS, BF16, RTOL, STATE_RTOL, FlipLedger, LockstepTap, m_res_error, output_close
from oracle import ModelDecoderOracle, gamma_delta, oracle_cfg
from vsa_lm_b200 import Bolt3Decoder
from vsa_lm_b200.model import Bolt3LM
from vsa_lm_b200.workloads import MODEL_SHAPES, make_model_params

pytestmark = pytest.mark.gpu
SHAPE = "tiny_lm"


def _models(seed=0):
    mcfg = dict(MODEL_SHAPES[SHAPE])
    params = make_model_params(mcfg, seed)
    model = Bolt3LM(**mcfg)
    model.load_state_dict(params, strict=True)
    model = model.to(device="cuda", dtype=torch.bfloat16).eval()
    # the module's own bf16 parameters: gamma_delta follows the parameter dtype, as in the reference
    oracle_params = {k: v.detach().cpu() for k, v in model.state_dict().items()}
    lcfg = oracle_cfg(dict(dim=mcfg["dim"], num_heads=mcfg["num_heads"], num_kv_heads=mcfg["num_kv_heads"],
                           head_dim=mcfg["head_dim"], eps=mcfg["eps"], rope_theta=mcfg["rope_theta"],
                           qk_norm=mcfg["qk_norm"]))
    # module.to(bf16) rounds the RoPE inv_freq buffers too, in the reference as here: the oracle
    # uses the frequencies the model holds
    lcfg["inv_freq"] = model.blocks[0].vsa.rope.inv_freq.detach().float().cpu()
    types = model.config["layer_types"]
    return mcfg, model, lambda b: ModelDecoderOracle(oracle_params, lcfg, types, b, BF16, mcfg["eps"])


def _check_greedy(tokens, oracle_logits, what):
    """Each native greedy token is the oracle's argmax, unless the oracle's best two logits are
    closer than the output tolerance (then either is a correct greedy choice)."""
    for i, (tok, lg) in enumerate(zip(tokens, oracle_logits)):
        top2 = lg.topk(2, dim=-1)
        scale = lg.pow(2).mean(-1).sqrt()
        tie = (top2.values[:, 0] - top2.values[:, 1]) <= RTOL * top2.values[:, 0].abs() + ATOL_RMS * scale
        ok = (tok.cpu().view(-1) == top2.indices[:, 0]) | tie
        assert ok.all(), f"{what}: step {i}: native tokens {tok.view(-1).tolist()} vs oracle {top2.indices[:, 0].tolist()}"


def test_step_and_prefill_match_model_oracle():
    mcfg, model, oracle = _models()
    B, T, n = 2, 300, 40
    ids = torch.randint(0, mcfg["vocab_size"], (B, T + n), generator=torch.Generator().manual_seed(5))
    dec = Bolt3Decoder(model)
    o, ledger = oracle(B), FlipLedger("model step")
    with LockstepTap(model, o, ledger):
        h, states, kv = dec.prefill(ids[:, :T].cuda())
        h_ref, _ = o.feed(ids[:, :T], 0)
        output_close(h.float().cpu(), h_ref, "prefill hidden states")
        for i in range(n):
            p = T + i
            h, states, kv = dec.step(ids[:, p:p + 1].cuda(), p, states, kv)
            output_close(h.float().cpu(), o.step(ids[:, p:p + 1], p), f"hidden states at position {p}")
    Bolt3Decoder.check_status(kv)
    ledger.report()


def test_generate_batch_greedy_matches_model_oracle():
    mcfg, model, oracle = _models()
    B, T, n = 2, 260, 24
    ids = torch.randint(0, mcfg["vocab_size"], (B, T), generator=torch.Generator().manual_seed(9))
    # eager steps, so that the tap sees (and checks) every layer step; the runs below replay the
    # steps from CUDA graphs and must give the same tokens
    dec = Bolt3Decoder(model, cuda_graphs=False)
    o, ledger = oracle(B), FlipLedger("generate_batch")
    with LockstepTap(model, o, ledger):
        toks, lengths = dec.generate_batch(ids.cuda(), n, temperature=0.0)
    assert toks.shape == (B, n) and torch.equal(lengths.cpu(), torch.full((B,), n))
    h, pos = o.feed(ids, 0)
    logits = []
    for i in range(n):
        logits.append(o.logits(h[:, -1]))
        h = o.step(toks[:, i:i + 1].cpu(), pos)
        pos += 1
    _check_greedy([toks[:, i] for i in range(n)], logits, "generate_batch")
    ledger.report()
    # end-of-sequence ids: a row's length is the step of its first one, decoding continues for the
    # others; `generate` returns the prompt and the first row's tokens up to its length
    eos = {int(toks[0, 5])}
    toks2, lengths2 = Bolt3Decoder(model).generate_batch(ids.cuda(), n, temperature=0.0, eos_ids=eos)
    assert torch.equal(toks2, toks[:, :toks2.shape[1]])
    first = [next((i + 1 for i in range(n) if int(toks[r, i]) in eos), n) for r in range(B)]
    assert lengths2.tolist() == first
    if toks2.shape[1] < n:   # stopped early: only once every row had finished, at a multiple of 16 steps
        assert toks2.shape[1] % 16 == 0 and max(first) <= toks2.shape[1]
    one, n1 = Bolt3Decoder(model).generate_batch(ids[:1].cuda(), n, temperature=0.0, eos_ids=eos)
    full = Bolt3Decoder(model).generate(ids[:1].cuda(), n, eos_ids=eos)
    assert torch.equal(full.cpu(), torch.cat([ids[:1], one[:, :int(n1[0])].cpu()], 1))


def test_sampling_modes_draw_valid_tokens():
    """Temperature sampling with top-k and with top-p: every draw is a token of the restricted set."""
    logits = torch.randn(4, 512, device="cuda") * 3
    for _ in range(20):
        t = Bolt3Decoder._sample(logits, 0.7, top_k=5, top_p=1.0)
        allowed = logits.topk(5, dim=-1).indices
        assert (allowed == t).any(-1).all()
        t = Bolt3Decoder._sample(logits, 0.7, top_p=0.5)
        probs = torch.softmax(logits / 0.7, -1)
        sp, si = probs.sort(-1, descending=True)
        nucleus = (sp.cumsum(-1) - sp) <= 0.5
        ok = torch.zeros_like(probs, dtype=torch.bool).scatter(1, si, nucleus)
        assert ok.gather(1, t).all()
    assert torch.equal(Bolt3Decoder._sample(logits, 0.0), logits.argmax(-1, keepdim=True))


def test_memory_bank_flow_matches_model_oracle():
    """memorize document A from a blank state, memorize B after it, pickle the state in the
    reference's format and load it back, forget B, and continue_generate a question greedily
    (vsa_lm/memory_bank.py:34-139 drives these calls). The traces must be M_after - gamma^2 M_before
    of the oracle's (re-synced) states (bolt3.py:528-545), forget must subtract them (:547-557)."""
    mcfg, model, oracle = _models()
    g = torch.Generator().manual_seed(21)
    V = mcfg["vocab_size"]
    doc = torch.randint(0, V, (1, 768 + 256), generator=g)
    q_ids = torch.randint(0, V, (1, 50), generator=g)
    dec = Bolt3Decoder(model, cuda_graphs=False)   # eager steps: the tap checks each one
    o, ledger = oracle(1), FlipLedger("memory-bank flow")
    tap = LockstepTap(model, o, ledger)
    vsa = [i for i, t in enumerate(model.config["layer_types"]) if t == "vsa"]
    states, kv = Bolt3Decoder.blank_state(model, 1, "cuda", max_kv_len=2048)
    with tap:
        states, kv, pos_a, _ = dec.memorize(doc[:, :768].cuda(), states, kv, 0)
    o.feed(doc[:, :768], 0)
    before = {i: o.m_res(i).clone() for i in vsa}
    with tap:
        states, kv, pos_b, traces = dec.memorize(doc[:, 768:].cuda(), states, kv, pos_a)
    o.feed(doc[:, 768:], pos_a)
    assert (pos_a, pos_b) == (768, 1024)
    expected = [None] * len(traces)
    for i in vsa:
        gam = gamma_delta(o.p[f"blocks.{i}.vsa.log_gamma"]).view(1, -1, 1, 1)
        expected[i] = (pos_b, o.m_res(i) - gam ** 2 * before[i])
        assert traces[i][0] == pos_b
        assert m_res_error(states[i], o.m_res(i)) < STATE_RTOL, f"M_res of layer {i} after memorize"
        assert m_res_error(traces[i][1], expected[i][1]) < STATE_RTOL, f"trace of layer {i}"
    # the state as the memory bank stores it: the reference's dict format, pickled
    ref_states, ref_kv = Bolt3Decoder.state_to_reference(model, states, kv)
    buf = io.BytesIO()
    torch.save({"states": [s.cpu() if s is not None else None for s in ref_states],
                "kv": [{k: (v.cpu() if torch.is_tensor(v) else v) for k, v in d.items()} if isinstance(d, dict)
                       else (d.k[:, :, :d.n].cpu(), d.v[:, :, :d.n].cpu()) for d in ref_kv]}, buf)
    buf.seek(0)
    cart = torch.load(buf, weights_only=False)
    kv_in = []
    for li, item in enumerate(cart["kv"]):
        if isinstance(item, tuple):
            cache = type(kv[li])(1, item[0].shape[1], 2048, item[0].shape[3], "cuda")
            cache.append(item[0].cuda(), item[1].cuda())
            kv_in.append(cache)
        else:
            kv_in.append({k: (v.cuda() if torch.is_tensor(v) else v) for k, v in item.items()})
    states2, kv2 = Bolt3Decoder.state_from_reference(model, cart["states"], kv_in, "cuda")
    states2 = dec.forget(traces, states2, next_pos=pos_b)
    o.forget(expected, pos_b)
    for i in vsa:
        assert m_res_error(states2[i], o.m_res(i)) < STATE_RTOL, f"M_res of layer {i} after forget"
    with tap:
        toks, states2, kv2, pos = dec.continue_generate(q_ids.cuda(), states2, kv2, pos_b, 12, temperature=0.0)
    assert pos == pos_b + 50 + 12 and toks.shape == (1, 12)
    h, op = o.feed(q_ids, pos_b)
    logits = []
    for i in range(12):
        logits.append(o.logits(h[:, -1]))
        h = o.step(toks[:, i:i + 1].cpu(), op)
        op += 1
    _check_greedy([toks[:, i] for i in range(12)], logits, "continue_generate")
    Bolt3Decoder.check_status(kv2)
    ledger.report()
