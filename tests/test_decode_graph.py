"""One-token decode steps replayed from CUDA graphs (Bolt3Decoder.step_graph) and the pieces that
make them possible: the device step position of the Bolt-3 decode kernels, and the anchor layers'
one-token attention kernel (bolt3_anchor_decode), checked against a plain PyTorch fp32 reference.

A replayed step runs the same kernels on the same data as an eager step, so its hidden states must
equal step()'s bit for bit; the chunk-boundary consolidations run eagerly after the replay."""
import pytest
import torch
import torch.nn.functional as F

from vsa_lm_b200 import Bolt3Decoder, Bolt3LayerState, kernels as K
from vsa_lm_b200.model import Bolt3LM
from vsa_lm_b200.workloads import MODEL_SHAPES, layer_cfg, make_input, make_model_params
from helpers import bf16_module

pytestmark = pytest.mark.gpu


def _anchor_ref(q, kc, vc, n, k_new, v_new, scale):
    """fp32 softmax attention of q [B, H, HD] over cache rows 0..n-1 plus the new row."""
    B, H, HD = q.shape
    HKV = kc.shape[1]
    keys = torch.cat([kc[:, :, :n].float(), k_new.float()[:, :, None]], 2)
    vals = torch.cat([vc[:, :, :n].float(), v_new.float()[:, :, None]], 2)
    keys = keys.repeat_interleave(H // HKV, 1)
    vals = vals.repeat_interleave(H // HKV, 1)
    p = torch.softmax((q.float()[:, :, None] @ keys.transpose(-1, -2)) * scale, -1)
    return (p @ vals)[:, :, 0]


@pytest.mark.parametrize("HD,G,n", [(128, 4, 0), (128, 4, 255), (128, 4, 256), (128, 4, 2300), (64, 2, 700),
                                    (64, 8, 31), (128, 1, 1000)])
def test_anchor_decode_matches_fp32_reference(HD, G, n):
    torch.manual_seed(n + HD)
    B, HKV, cap = 3, 2, 2560
    H = HKV * G
    q = torch.randn(B, H, HD, device="cuda").bfloat16()
    kc = torch.randn(B, HKV, cap, HD, device="cuda").bfloat16()
    vc = torch.randn(B, HKV, cap, HD, device="cuda").bfloat16()
    k_new = torch.randn(B, HKV, HD, device="cuda").bfloat16()
    v_new = torch.randn(B, HKV, HD, device="cuda").bfloat16()
    ref = _anchor_ref(q, kc, vc, n, k_new, v_new, HD ** -0.5)
    y = torch.empty(B, H, HD, device="cuda", dtype=torch.bfloat16)
    K.anchor_decode(q=q, k_new=k_new, v_new=v_new, k_cache=kc, v_cache=vc, n=n, y=y, scale=HD ** -0.5)
    assert torch.equal(kc[:, :, n], k_new) and torch.equal(vc[:, :, n], v_new)
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=2e-2 * ref.pow(2).mean().sqrt().item())


@pytest.mark.parametrize("HD,G", [(128, 4), (64, 2)])
def test_anchor_decode_rope_in_kernel(HD, G):
    """RoPE of q and the new key inside bolt3_anchor_decode (inv_freq, pos0) against LlamaRoPE applied
    by torch before the call: the appended key within one bf16 rounding (the cos / sin come from a
    different routine), the output within the attention tolerance."""
    from vsa_lm_b200.bolt3 import LlamaRoPE

    torch.manual_seed(HD + G)
    B, HKV, cap, n, pos = 3, 2, 512, 300, 1234
    rope = LlamaRoPE(HD, 1e6, None).cuda()
    q = torch.randn(B, HKV * G, HD, device="cuda").bfloat16()
    kn = torch.randn(B, HKV, HD, device="cuda").bfloat16()
    vn = torch.randn(B, HKV, HD, device="cuda").bfloat16()
    kc = torch.randn(B, HKV, cap, HD, device="cuda").bfloat16()
    vc = torch.randn(B, HKV, cap, HD, device="cuda").bfloat16()
    qr = rope(q.unsqueeze(2), pos_start=pos).squeeze(2)
    kr = rope(kn.unsqueeze(2), pos_start=pos).squeeze(2)
    ya, yb = torch.empty_like(q), torch.empty_like(q)
    kca, kcb = kc.clone(), kc.clone()
    K.anchor_decode(q=qr, k_new=kr, v_new=vn, k_cache=kca, v_cache=vc.clone(), n=n, y=ya, scale=HD ** -0.5)
    K.anchor_decode(q=q, k_new=kn, v_new=vn, k_cache=kcb, v_cache=vc.clone(), n=n, y=yb, scale=HD ** -0.5,
                    inv_freq=rope.inv_freq.float(), pos0=pos)
    torch.testing.assert_close(kcb[:, :, n].float(), kca[:, :, n].float(), rtol=2 ** -7, atol=1e-6)
    ref = ya.float()
    torch.testing.assert_close(yb.float(), ref, rtol=2e-2, atol=2e-2 * ref.pow(2).mean().sqrt().item())


def test_anchor_decode_device_position():
    """The same launch, built for position 40 with a span of 8, replayed at 40 + d from the device."""
    torch.manual_seed(5)
    B, HKV, G, HD, cap = 2, 2, 4, 128, 512
    q = torch.randn(B, HKV * G, HD, device="cuda").bfloat16()
    kc = torch.randn(B, HKV, cap, HD, device="cuda").bfloat16()
    vc = torch.randn(B, HKV, cap, HD, device="cuda").bfloat16()
    k_new = torch.randn(B, HKV, HD, device="cuda").bfloat16()
    v_new = torch.randn(B, HKV, HD, device="cuda").bfloat16()
    pos = K.DevicePosition("cuda")
    pos.ref, pos.span = 40, 8
    status = K.DeviceStatus("cuda")
    for d in (0, 3, 7):
        kc2, vc2 = kc.clone(), vc.clone()
        y = torch.empty_like(q)
        y2 = torch.empty_like(q)
        pos.set(40 + d)
        K.anchor_decode(q=q, k_new=k_new, v_new=v_new, k_cache=kc2, v_cache=vc2, n=100, y=y, scale=HD ** -0.5,
                        dev_pos=pos, status=status)
        K.anchor_decode(q=q, k_new=k_new, v_new=v_new, k_cache=kc.clone(), v_cache=vc.clone(), n=100 + d, y=y2,
                        scale=HD ** -0.5)
        assert torch.equal(y, y2) and torch.equal(kc2[:, :, 100 + d], k_new)
    # a position outside the span: nothing is written and the status word says so
    pos.set(40 + 8)
    y = torch.zeros_like(q)
    K.anchor_decode(q=q, k_new=k_new, v_new=v_new, k_cache=kc, v_cache=vc, n=100, y=y, scale=HD ** -0.5,
                    dev_pos=pos, status=status)
    torch.cuda.synchronize()
    assert int(status.word.item()) & 8 and not y.any()
    status.word.zero_()


@pytest.mark.parametrize("shape", ["qwen3_4b", "tiny"])
def test_decode_kernels_device_position_equal_eager(shape):
    """A Bolt-3 layer's one-token launches built once at a chunk's first position and given later
    positions through the device give the eager steps' outputs bit for bit (the streaming kernel at
    HD = 128, the warp-per-chain kernel at HD = 64), across two chunk boundaries."""
    cfg = layer_cfg(shape)
    m = bf16_module(cfg, 0)
    B, prompt, n_dec = 2, 256, 200
    x = make_input(B, prompt + n_dec, cfg["dim"], dup=0.3, seed=6).to(torch.bfloat16).cuda()
    sts = [Bolt3LayerState(m, B, "cuda") for _ in range(2)]
    mres = [torch.zeros(B, m.HKV, m.HD, m.HD, device="cuda") for _ in range(2)]
    for s in range(0, prompt, 128):
        for st, mr in zip(sts, mres):
            Bolt3Decoder.layer_step(m, st, x[:, s:s + 128], s, mr)
    pos = K.DevicePosition("cuda")
    for p in range(prompt, prompt + n_dec):
        h = x[:, p:p + 1]
        ref = Bolt3Decoder.layer_step(m, sts[0], h, p, mres[0])
        st = sts[1]
        if st.cur_len == 0 or p == prompt:
            pos.ref, pos.span = p, m.C - st.cur_len
            launch_pos = p
        pos.set(p)
        # the launch is built as at its reference position, then the device position moves it
        cur = st.cur_len
        st.cur_len = cur - (p - launch_pos)
        got = Bolt3Decoder._layer_launch(m, st, h, launch_pos, mres[1], dev_pos=pos)
        st.cur_len = cur
        Bolt3Decoder._layer_advance(m, st, 1, p, mres[1])
        assert torch.equal(got, ref), f"position {p}"
    assert torch.equal(mres[0], mres[1])


def _model(shape):
    mcfg = dict(MODEL_SHAPES[shape])
    model = Bolt3LM(**mcfg)
    model.load_state_dict(make_model_params(mcfg, 0), strict=True)
    return mcfg, model.to(device="cuda", dtype=torch.bfloat16).eval()


@pytest.mark.parametrize("shape", ["small_lm", "tiny_lm"])
def test_step_graph_equals_eager_steps(shape):
    """Greedy decoding through Bolt3Decoder.step_graph (one capture per chunk) against eager step()
    calls on a copy of the state: the same hidden states bit for bit over 300 steps (three chunk
    boundaries), and the same final M_res."""
    mcfg, model = _model(shape)
    dec = Bolt3Decoder(model)
    g = torch.Generator().manual_seed(3)
    B, T = 2, 300
    ids = torch.randint(0, mcfg["vocab_size"], (B, T), generator=g).cuda()
    steps = torch.randint(0, mcfg["vocab_size"], (B, 300), generator=g).cuda()
    h0, st_e, kv_e = dec.prefill(ids, max_kv_len=T + 320)
    h1, st_g, kv_g = dec.prefill(ids, max_kv_len=T + 320)
    assert torch.equal(h0, h1)
    runner = dec.step_graph(st_g, kv_g)
    for i in range(steps.shape[1]):
        tok = steps[:, i:i + 1]
        he, st_e, kv_e = dec.step(tok, T + i, st_e, kv_e)
        hg = runner.step(tok, T + i)
        assert torch.equal(hg, he), f"step {i}"
    assert runner.captures == 3      # the chunk the prompt left open (300..383), then 384.., 512..
    for a, b in zip(st_e, st_g):
        if a is not None:
            assert torch.equal(a, b)
    Bolt3Decoder.check_status(kv_g)


def test_generate_batch_graphs_equal_eager():
    """generate_batch with graph replay and without it (cuda_graphs=False) gives the same tokens."""
    mcfg, model = _model("small_lm")
    ids = torch.randint(0, mcfg["vocab_size"], (3, 200), generator=torch.Generator().manual_seed(9)).cuda()
    a, la = Bolt3Decoder(model).generate_batch(ids, 150, temperature=0.0)
    b, lb = Bolt3Decoder(model, cuda_graphs=False).generate_batch(ids, 150, temperature=0.0)
    assert torch.equal(a, b) and torch.equal(la, lb)


@pytest.mark.parametrize("rows,D,wdt", [(64, 2560, torch.bfloat16), (1000, 128, torch.bfloat16), (3, 64, torch.float32),
                                        (130, 4096, torch.bfloat16), (5, 2048, torch.float32),
                                        (5000, 1024, torch.bfloat16)])
def test_rmsnorm_kernel_matches_fp32_reference(rows, D, wdt):
    """bolt3_rmsnorm against the fp32 formula of LlamaRMSNorm (surgery.py:43-53): within one bf16
    rounding of the exact value (a warp per row, and a block per row for few wide rows)."""
    torch.manual_seed(rows)
    x = (torch.randn(rows, D, device="cuda") * 3).bfloat16()
    w = (1 + 0.1 * torch.randn(D, device="cuda")).to(wdt)
    got = K.rmsnorm(x, w, 1e-6).float()
    xf = x.float()
    ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
    torch.testing.assert_close(got, ref, rtol=2 ** -7, atol=1e-6)
    # a strided input (a slice of a wider row) gives the same result
    wide = torch.cat([x, x[:, :8]], 1)
    assert torch.equal(K.rmsnorm(wide[:, :D], w, 1e-6), K.rmsnorm(x, w, 1e-6))


@pytest.mark.parametrize("rows,D", [(64, 2560), (1000, 128)])
def test_add_rmsnorm_matches_torch(rows, D):
    """The residual form of bolt3_rmsnorm: the sum equals torch's bf16 addition bit for bit, and the
    norm equals bolt3_rmsnorm of that sum bit for bit."""
    torch.manual_seed(rows + D)
    x = (torch.randn(rows, D, device="cuda") * 2).bfloat16()
    r = torch.randn(rows, D, device="cuda").bfloat16()
    w = (1 + 0.1 * torch.randn(D, device="cuda")).bfloat16()
    s, y = K.add_rmsnorm(x, r, w, 1e-6)
    assert torch.equal(s, x + r)
    assert torch.equal(y, K.rmsnorm(x + r, w, 1e-6))


def test_swiglu_fused_equals_torch():
    """LlamaMLP with the gate and up projections as one GEMM and the fused silu * up kernel against
    torch's two projections, silu and product on the same bf16 weights (within one bf16 rounding: the
    GEMMs may sum in another order), and its weights still the module's parameters afterwards."""
    from vsa_lm_b200.model import LlamaMLP

    torch.manual_seed(7)
    mlp = LlamaMLP(dict(dim=256, intermediate=512)).cuda().bfloat16()
    x = torch.randn(64, 256, device="cuda").bfloat16()
    with torch.no_grad():
        ref = torch.nn.functional.silu(mlp.gate_proj(x)) * mlp.up_proj(x)
        got = mlp.act(x)
        w = mlp._gate_up_weight()
        assert w.data_ptr() == mlp.gate_proj.weight.data_ptr()
        mlp.up_proj.weight.add_(1.0)                      # an in-place weight edit reaches the fused weight
        ref2 = torch.nn.functional.silu(mlp.gate_proj(x)) * mlp.up_proj(x)
        got2 = mlp.act(x)
    torch.testing.assert_close(got.float(), ref.float(), rtol=2 ** -7, atol=1e-3)
    torch.testing.assert_close(got2.float(), ref2.float(), rtol=2 ** -7, atol=1e-3)
