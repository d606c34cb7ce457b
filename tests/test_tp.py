"""KV-head tensor parallelism (vsa_lm_b200/tp.py): the shards' partial outputs sum to the full
layer's output. CPU: two gloo ranks run the oracle on their shards and all-reduce; two gloo ranks
split a softmax anchor by KV head and a SwiGLU MLP by feature. GPU: the native shards of one layer
on one device, for the forward and the decode step; a Qwen3-4B-width softmax anchor and MLP split
four and eight ways on one device; the whole hybrid model split over two ranks (gloo, one GPU;
NCCL, two GPUs) against the unsharded decoder."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from helpers import BF16, bf16_module, oracle_cfg_of, oracle_params, output_close
from oracle import Store, forward
from vsa_lm_b200 import AnchorKV, Bolt3Attn, Bolt3Decoder, Bolt3LayerState
from vsa_lm_b200.model import LlamaMLP, SoftmaxAttn
from vsa_lm_b200.tp import anchor_partial, kv_head_range, mlp_partial, shard_by_kv_head, shard_mlp, shard_softmax_attn
from vsa_lm_b200.workloads import layer_cfg, make_input, make_params

FP32 = Store("fp32")


def _local_cfg(m: Bolt3Attn, cfg: dict) -> dict:
    return dict(cfg, num_heads=m.H, num_kv_heads=m.HKV, head_dim=m.HD)


def _gloo_worker(rank: int, world: int, port: int, out):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = layer_cfg("tiny")
        full = Bolt3Attn(cfg)
        full.load_state_dict(make_params(cfg, 0))
        local = shard_by_kv_head(full, rank, world)
        x = make_input(1, 300, cfg["dim"], dup=0.3, seed=3)
        y = forward(oracle_params(local), oracle_cfg_of(local, _local_cfg(local, cfg)), x, FP32)
        dist.all_reduce(y, op=dist.ReduceOp.SUM)
        if rank == 0:
            out.put(y)
    finally:
        dist.destroy_process_group()


_ANCHOR_CFG = dict(dim=256, num_heads=8, num_kv_heads=4, head_dim=32, eps=1e-6, rope_theta=1e4, qk_norm=True,
                   intermediate=512)


def _anchor_mlp(seed: int = 0):
    torch.manual_seed(seed)
    attn, mlp = SoftmaxAttn(_ANCHOR_CFG), LlamaMLP(_ANCHOR_CFG)
    with torch.no_grad():
        attn.q_norm.weight.uniform_(0.5, 1.5)
        attn.k_norm.weight.uniform_(0.5, 1.5)
    return attn, mlp, torch.randn(2, 50, _ANCHOR_CFG["dim"], generator=torch.Generator().manual_seed(seed + 1))


def _gloo_anchor_mlp_worker(rank: int, world: int, port: int, out):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        attn, mlp, x = _anchor_mlp()
        with torch.no_grad():
            ya = anchor_partial(shard_softmax_attn(attn, rank, world), x)
            ym = mlp_partial(shard_mlp(mlp, rank, world), x)
        dist.all_reduce(ya, op=dist.ReduceOp.SUM)
        dist.all_reduce(ym, op=dist.ReduceOp.SUM)
        if rank == 0:
            out.put((ya, ym))
    finally:
        dist.destroy_process_group()


def _gloo_failing_rank_worker(rank: int, world: int, port: int, out, mode: str):
    """Rank 1 fails on the host: it leaves between steps before its all-reduce ("dies") or never
    joins the group ("absent"). Rank 0 reports what its next group call raised and how long it took."""
    import time
    from datetime import timedelta

    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    if rank == 1 and mode == "absent":
        return
    t0 = time.monotonic()
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
        attn, mlp, x = _anchor_mlp()
        with torch.no_grad():
            ym = mlp_partial(shard_mlp(mlp, rank, world), x)
        if rank == 1:
            dist.destroy_process_group()
            return
        dist.all_reduce(ym, op=dist.ReduceOp.SUM)
        out.put(("no error", time.monotonic() - t0))
    except Exception as exc:  # noqa: BLE001
        out.put((type(exc).__name__, time.monotonic() - t0))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["dies", "absent"])
def test_tp_rank_failure_ends_the_others_collective_with_an_error(mode):
    """A tensor-parallel rank that leaves before its all-reduce, or never joins, makes the surviving
    rank's next group call raise within the process group's short timeout instead of waiting for
    good: the failure reaches the host, no GPU is involved."""
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = 33600 + os.getpid() % 500 + (0 if mode == "dies" else 500)
    procs = [ctx.Process(target=_gloo_failing_rank_worker, args=(r, 2, port, out, mode)) for r in range(2)]
    for p in procs:
        p.start()
    what, seconds = _get_while_alive(out, procs, deadline_s=120)
    for p in procs:
        p.join(timeout=60)
    assert what != "no error", "the surviving rank's collective completed without its peer"
    assert seconds < 60


def _get_while_alive(q, procs, deadline_s: float):
    """The first item of `q`, polling in short waits; fails as soon as a rank has exited with an
    error or the deadline passes, instead of blocking on a rank that died."""
    import queue
    import time

    t0 = time.monotonic()
    while time.monotonic() - t0 < deadline_s:
        try:
            return q.get(timeout=2)
        except queue.Empty:
            dead = [p.exitcode for p in procs if p.exitcode not in (None, 0)]
            assert not dead, f"a rank exited with {dead}"
            assert any(p.exitcode is None for p in procs), "every rank exited without a result"
    for p in procs:
        p.kill()
    raise AssertionError(f"no result within {deadline_s} s")


def test_kv_head_range_splits_evenly():
    assert [kv_head_range(8, r, 4) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    with pytest.raises(ValueError):
        kv_head_range(8, 0, 3)


def test_shards_partition_the_parameters():
    cfg = layer_cfg("config0")   # 15 query heads over 5 KV heads (G = 3)
    full = Bolt3Attn(cfg)
    full.load_state_dict(make_params(cfg, 1))
    parts = [shard_by_kv_head(full, r, 5) for r in range(5)]
    cat = lambda name: torch.cat([dict(p.named_parameters())[name] for p in parts])
    for name in ("q_proj.weight", "k_proj.weight", "v_proj.weight", "beta_proj.weight", "beta_proj.bias",
                 "eta_proj.weight", "eta_proj.bias", "kappa", "log_gamma"):
        assert torch.equal(cat(name), dict(full.named_parameters())[name]), name
    assert torch.equal(torch.cat([p.o_proj.weight for p in parts], 1), full.o_proj.weight)
    assert all(p.H == 3 and p.HKV == 1 and p.G == full.G for p in parts)


def test_tp_oracle_allreduce_matches_full_layer_gloo():
    """Two gloo ranks, each the oracle on its KV heads, one all-reduce: the full layer's output."""
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_gloo_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    y = _get_while_alive(out, procs, deadline_s=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    cfg = layer_cfg("tiny")
    full = Bolt3Attn(cfg)
    full.load_state_dict(make_params(cfg, 0))
    x = make_input(1, 300, cfg["dim"], dup=0.3, seed=3)
    ref = forward(oracle_params(full), oracle_cfg_of(full, cfg), x, FP32)
    output_close(y, ref, "all-reduced shard outputs")


def test_tp_anchor_and_mlp_allreduce_gloo():
    """Two gloo ranks: a softmax anchor split by KV head and a SwiGLU MLP split by intermediate
    feature; their fp32 partials, all-reduced, are the unsharded modules' outputs."""
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = 30500 + os.getpid() % 1000
    procs = [ctx.Process(target=_gloo_anchor_mlp_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    ya, ym = _get_while_alive(out, procs, deadline_s=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    attn, mlp, x = _anchor_mlp()
    with torch.no_grad():
        torch.testing.assert_close(ya, attn(x), rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(ym, mlp(x), rtol=1e-5, atol=1e-5)


def _run_model_worker(tmp_path, backend: str, nproc: int):
    import subprocess
    import sys

    out = tmp_path / f"tp_model_{backend}.pt"
    here = os.path.dirname(os.path.abspath(__file__))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    port = 31600 + os.getpid() % 1000 + (7 if backend == "gloo" else 0)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}",
           "--master-addr=127.0.0.1", f"--master-port={port}", os.path.join(here, "tp_model_worker.py"),
           "--out", str(out), "--backend", backend]
    r = subprocess.run(cmd, env=env, timeout=240, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = torch.load(out, weights_only=False)
    assert res["world"] == nproc
    output_close(res["got"], res["ref"], f"{nproc}-rank tensor-parallel model over {backend}")
    if backend == "nccl":       # graph replay (captured NCCL all-reduces) equals the eager steps
        assert res["graphed"] is not None and torch.equal(res["graphed"], res["got"])
    else:                       # gloo all-reduces run on the host: no graphs
        assert res["graphed"] is None


@pytest.mark.gpu
def test_tp_model_two_ranks_gloo_one_gpu(tmp_path):
    """The whole hybrid model split over two ranks that share one GPU (gloo all-reduces through the
    host), prefill and one-token decode steps, against the unsharded decoder. Each rank's kernels
    are independent launches; only the host-side collective joins them."""
    _run_model_worker(tmp_path, "gloo", 2)


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp_model_nccl_two_gpus(tmp_path):
    """The whole hybrid model split over two GPUs (NCCL all-reduces after every attention and every
    MLP) against the unsharded decoder."""
    _run_model_worker(tmp_path, "nccl", 2)


@pytest.mark.gpu
@pytest.mark.parametrize("shape,world", [("qwen3_4b", 2), ("qwen3_4b", 8), ("tiny", 2)])
def test_tp_native_shards_sum_to_layer(shape, world):
    """The native forward of every shard, summed (the all-reduce on one device), against the
    oracle's full layer."""
    cfg = layer_cfg(shape)
    m = bf16_module(cfg, 0)
    B, T = 2, 700
    x = make_input(B, T, cfg["dim"], dup=0.3, seed=4).to(torch.bfloat16)
    ys = [shard_by_kv_head(m, r, world)._native_forward(x.cuda(), partial_fp32=True) for r in range(world)]
    y = torch.stack(ys).sum(0).to(torch.bfloat16).float()   # the fp32 all-reduce, rounded once
    ref = forward(oracle_params(m), oracle_cfg_of(m, cfg), x.float(), BF16)
    output_close(y.cpu(), ref, f"{world} KV-head shards")


@pytest.mark.gpu
def test_tp_decode_shards_sum_to_layer():
    """Decode steps on two KV-head shards, summed, against the unsharded native decoder."""
    cfg = layer_cfg("qwen3_4b")
    m = bf16_module(cfg, 0)
    B, prompt = 2, 260
    x = make_input(B, prompt + 30, cfg["dim"], dup=0.3, seed=6).to(torch.bfloat16).cuda()
    shards = [shard_by_kv_head(m, r, 2) for r in range(2)]
    states = [(Bolt3LayerState(s, B, "cuda"), torch.zeros(B, s.HKV, s.HD, s.HD, device="cuda")) for s in shards]
    st = Bolt3LayerState(m, B, "cuda")
    m_res = torch.zeros(B, m.HKV, m.HD, m.HD, device="cuda")
    steps = [(s, min(128, prompt - s)) for s in range(0, prompt, 128)] + [(prompt + i, 1) for i in range(30)]
    for p, n in steps:
        h = x[:, p:p + n]
        ref = Bolt3Decoder.layer_step(m, st, h, p, m_res)
        got = sum(Bolt3Decoder.layer_step(s, so, h, p, mr, partial_fp32=True) for s, (so, mr) in zip(shards, states))
        got = got.to(torch.bfloat16)
        output_close(got.cpu(), ref.float().cpu(), f"decode step at {p}")


@pytest.mark.gpu
@pytest.mark.parametrize("world", [4, 8])
def test_tp_anchor_and_mlp_shards_at_4b_widths(world):
    """A Qwen3-4B-width softmax anchor (32 query heads, 8 KV heads, per-head q/k norms) and SwiGLU
    MLP (9728 features) split `world` ways on one device, as Bolt3LMTP splits them: the anchors'
    one-token decode kernel with 1-2 KV heads per shard and the MLP's gate/up GEMM and silu_mul at
    9728 / world features. The shards' fp32 partial sums, rounded once, against the unsharded
    modules over a prompt and six decode steps."""
    torch.manual_seed(0)
    cfg = dict(dim=2560, num_heads=32, num_kv_heads=8, head_dim=128, eps=1e-6, rope_theta=1e6, qk_norm=True)
    attn = SoftmaxAttn(cfg)
    with torch.no_grad():
        attn.q_norm.weight.uniform_(0.5, 1.5)
        attn.k_norm.weight.uniform_(0.5, 1.5)
    attn = attn.to(device="cuda", dtype=torch.bfloat16).eval()
    mlp = LlamaMLP(dict(dim=2560, intermediate=9728)).to(device="cuda", dtype=torch.bfloat16).eval()
    B, prompt, steps = 4, 40, 6
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(B, prompt + steps, 2560, generator=g, device="cuda").to(torch.bfloat16)
    with torch.no_grad():
        shards = [shard_softmax_attn(attn, r, world) for r in range(world)]
        assert {s.HKV for s in shards} == {8 // world} and all(s.G == 4 for s in shards)
        caches = [AnchorKV(B, s.HKV, 256, s.HD, "cuda") for s in shards]
        cache = AnchorKV(B, attn.HKV, 256, attn.HD, "cuda")
        for p, n in [(0, prompt)] + [(prompt + i, 1) for i in range(steps)]:
            h = x[:, p:p + n]
            ref = Bolt3Decoder._anchor_attention(attn, cache, h, p)
            got = sum(Bolt3Decoder._anchor_attention(s, c, h, p, partial_fp32=True) for s, c in zip(shards, caches))
            output_close(got.to(torch.bfloat16), ref, f"anchor step at {p}, {world} shards")
        mlps = [shard_mlp(mlp, r, world) for r in range(world)]
        for h in (x[:, -1:], x[:, :prompt]):
            ref = mlp(h)
            got = sum(mlp_partial(m, h) for m in mlps)
            output_close(got.to(torch.bfloat16), ref, f"MLP of {h.shape[1]} tokens, {world} shards")



@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp_nccl_two_gpus_matches_layer(tmp_path):
    """Bolt3AttnTP over two GPUs (one NCCL all-reduce of the o_proj partials per call), forward and
    decode steps, against the unsharded native layer on GPU 0. The ranks run under
    torch.distributed.run as child processes with a hard time limit, so a rank that dies or hangs
    fails the test instead of stalling it; NVLS is off."""
    import subprocess
    import sys

    out = tmp_path / "tp.pt"
    here = os.path.dirname(os.path.abspath(__file__))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    port = 29600 + os.getpid() % 1000
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={port}", os.path.join(here, "tp_nccl_worker.py"),
           "--out", str(out)]
    r = subprocess.run(cmd, env=env, timeout=240, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = torch.load(out, weights_only=False)
    assert res["world"] == 2
    output_close(res["y"], res["ref"], "two-GPU tensor-parallel forward")
    output_close(res["dec"], res["ref_dec"], "two-GPU tensor-parallel decode steps")
