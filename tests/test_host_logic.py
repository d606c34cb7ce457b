"""Host-side bookkeeping of the decoder's fused paths, on the CPU: the SwiGLU MLP's shared gate/up
weight, the cached fp32 RoPE frequencies the anchors' kernel reads, and the anchors' KV cache growth."""
import torch

from vsa_lm_b200.bolt3 import AnchorKV, LlamaRoPE, _fp32_inv_freq
from vsa_lm_b200.model import LlamaMLP


def test_gate_up_weight_is_the_parameters_storage():
    torch.manual_seed(0)
    mlp = LlamaMLP(dict(dim=32, intermediate=48)).bfloat16()
    g0, u0 = mlp.gate_proj.weight.detach().clone(), mlp.up_proj.weight.detach().clone()
    w = mlp._gate_up_weight()
    assert w.shape == (96, 32)
    assert torch.equal(w[:48], g0) and torch.equal(w[48:], u0)
    # the parameters now live in the fused weight: no second copy, and later calls return it as is
    assert mlp.gate_proj.weight.data_ptr() == w.data_ptr()
    assert mlp.up_proj.weight.data_ptr() == w[48:].data_ptr()
    assert mlp._gate_up_weight() is w
    # an in-place edit (a checkpoint load copies in place) is seen through the fused weight
    with torch.no_grad():
        mlp.up_proj.weight.mul_(2)
    assert torch.equal(mlp._gate_up_weight()[48:], u0 * 2)
    # a replaced parameter makes the fused weight again
    mlp.gate_proj.weight = torch.nn.Parameter(torch.ones(48, 32, dtype=torch.bfloat16))
    w2 = mlp._gate_up_weight()
    assert w2 is not w and torch.equal(w2[:48], torch.ones(48, 32, dtype=torch.bfloat16))
    assert torch.equal(w2[48:], u0 * 2)


def test_state_dict_round_trip_after_fusing():
    mlp = LlamaMLP(dict(dim=16, intermediate=24))
    mlp._gate_up_weight()
    sd = {k: v.clone() for k, v in mlp.state_dict().items()}
    other = LlamaMLP(dict(dim=16, intermediate=24))
    other.load_state_dict(sd, strict=True)
    for k in sd:
        assert torch.equal(other.state_dict()[k], sd[k])


def test_fp32_inv_freq_cache_follows_the_buffer():
    rope = LlamaRoPE(64, 1e4, None).bfloat16()
    f1 = _fp32_inv_freq(rope, "cpu")
    assert f1.dtype == torch.float32 and torch.equal(f1, rope.inv_freq.float())
    assert _fp32_inv_freq(rope, "cpu") is f1                 # kept between calls
    with torch.no_grad():
        rope.inv_freq.mul_(0.5)                                # an in-place change is noticed
    f2 = _fp32_inv_freq(rope, "cpu")
    assert f2 is not f1 and torch.equal(f2, rope.inv_freq.float())


def test_anchor_cache_reserve_and_append():
    c = AnchorKV(2, 3, 100, 8, "cpu", dt=torch.float32)
    assert c.capacity == 256 and c.n == 0
    k = torch.randn(2, 3, 200, 8)
    keys, vals = c.append(k, k + 1)
    assert c.n == 200 and torch.equal(keys, k) and torch.equal(vals, k + 1)
    c.reserve(100)                                            # 300 > 256: doubles, keeps the rows
    assert c.capacity == 512 and torch.equal(c.k[:, :, :200], k)
    c.reserve(10)
    assert c.capacity == 512                                  # room already there


def test_layer_state_holds_what_state_bytes_counts(monkeypatch):
    """A Bolt-3 layer's decode state allocates exactly Bolt3LayerState.bytes_per_sequence per
    sequence, with M_res counted once: it is the caller's states[li], and the state's bank holds
    no second copy. Decoder.state_bytes sums those over the Bolt-3 layers, plus the anchors' bf16
    k and v per token. (The device status word is the one CUDA-only member; it is stubbed here.)"""
    from vsa_lm_b200 import Bolt3Attn, Bolt3Decoder, Bolt3LayerState, kernels as K
    from vsa_lm_b200.model import Bolt3LM
    from vsa_lm_b200.workloads import MODEL_SHAPES, layer_cfg

    monkeypatch.setattr(K, "DeviceStatus", lambda device: None)
    m = Bolt3Attn(layer_cfg("tiny"))
    B = 3
    st = Bolt3LayerState(m, B, "cpu")
    assert "m_res" not in st.bank
    held = [st.ring_kr, st.ring_kp, st.ring_v, st.ring_b, st.sink_k, st.sink_v, *st.bank.values()]
    m_res = B * m.HKV * m.HD * m.HD * 4
    assert sum(t.numel() * t.element_size() for t in held) + m_res == B * Bolt3LayerState.bytes_per_sequence(m)

    model = Bolt3LM(**dict(MODEL_SHAPES["tiny_lm"]))
    fixed, per_token = Bolt3Decoder.state_bytes(model)
    vsa = [b.vsa for b in model.blocks if hasattr(b, "vsa")]
    anchors = [b.attn for b in model.blocks if not hasattr(b, "vsa")]
    assert vsa and anchors
    assert fixed == sum(Bolt3LayerState.bytes_per_sequence(ly) for ly in vsa)
    assert per_token == sum(2 * a.HKV * a.HD * 2 for a in anchors)
