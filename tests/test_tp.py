"""KV-head tensor parallelism (vsa_lm_b200/tp.py): the shards' partial outputs sum to the full
layer's output. CPU: two gloo ranks run the oracle on their shards and all-reduce. GPU: the native
shards of one layer on one device, for the forward and the decode step."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from helpers import BF16, bf16_module, oracle_cfg_of, oracle_params, output_close
from oracle import Store, forward
from vsa_lm_b200 import Bolt3Attn, Bolt3Decoder, Bolt3LayerState
from vsa_lm_b200.tp import kv_head_range, shard_by_kv_head
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
