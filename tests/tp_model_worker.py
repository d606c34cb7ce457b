"""One rank of the whole-model tensor-parallel check (launched by tests/test_tp.py through
torch.distributed.run; not a test module itself).

Every rank builds the same seeded hybrid model (Bolt-3 layers and a softmax anchor), keeps its
KV heads and its block of MLP features (Bolt3LMTP) and runs a prompt prefill and teacher-forced
one-token decode steps through Bolt3DecoderTP; every attention and every MLP ends in an all-reduce.
Rank 0 also runs the unsharded model through Bolt3Decoder on the same tokens and writes both
results to --out. With --backend gloo every rank may share one GPU (the all-reduces pass through
the host); with nccl each rank takes its own GPU."""
import argparse
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [HERE, os.path.dirname(HERE)]

from vsa_lm_b200 import Bolt3Decoder  # noqa: E402
from vsa_lm_b200.model import Bolt3LM  # noqa: E402
from vsa_lm_b200.tp import Bolt3DecoderTP, Bolt3LMTP  # noqa: E402
from vsa_lm_b200.workloads import MODEL_SHAPES, make_model_params  # noqa: E402


def run_graphed(dec, ids, steps):
    """The same as run() with the one-token steps replayed from CUDA graphs. The runner, whose graphs
    hold captured NCCL all-reduces, is closed before this returns: a process group must not be
    destroyed while such a graph exists."""
    h, states, kv = dec.prefill(ids, max_kv_len=ids.shape[1] + steps.shape[1] + 8)
    runner = dec.step_graph(states, kv)
    try:
        outs = [h[:, -1:]]
        for i in range(steps.shape[1]):
            outs.append(runner.step(steps[:, i:i + 1], ids.shape[1] + i).clone())
        torch.cuda.synchronize()
        return torch.cat(outs, 1).float().cpu()
    finally:
        runner.close()


def run(dec, ids, steps):
    """Prefill ids [B, T], then one step per column of `steps` [B, n]; the hidden states of the
    prompt's last position and of every step, [B, 1 + n, D]."""
    h, states, kv = dec.prefill(ids, max_kv_len=ids.shape[1] + steps.shape[1] + 8)
    out = [h[:, -1:]]
    for i in range(steps.shape[1]):
        h, states, kv = dec.step(steps[:, i:i + 1], ids.shape[1] + i, states, kv)
        out.append(h)
    return torch.cat(out, 1).float().cpu()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    ap.add_argument("--backend", default="nccl", choices=("nccl", "gloo"))
    ap.add_argument("--shape", default="tiny_lm")
    args = ap.parse_args()
    rank, local = int(os.environ["RANK"]), int(os.environ["LOCAL_RANK"])
    dev = torch.device("cuda", local % torch.cuda.device_count())
    torch.cuda.set_device(dev)
    kw = dict(device_id=dev) if args.backend == "nccl" else {}
    dist.init_process_group(args.backend, timeout=timedelta(seconds=60), **kw)
    try:
        mcfg = dict(MODEL_SHAPES[args.shape])
        model = Bolt3LM(**mcfg)
        model.load_state_dict(make_model_params(mcfg, 0), strict=True)
        model = model.to(device=dev, dtype=torch.bfloat16).eval()
        g = torch.Generator().manual_seed(7)
        B, T, n = 2, 300, 20
        ids = torch.randint(0, mcfg["vocab_size"], (B, T), generator=g).to(dev)
        steps = torch.randint(0, mcfg["vocab_size"], (B, n), generator=g).to(dev)
        tp = Bolt3LMTP(model)
        dec = Bolt3DecoderTP(tp)
        got = run(dec, ids, steps)
        # the same steps replayed from CUDA graphs (NCCL all-reduces captured in them), where the group
        # allows it; they must equal the eager steps bit for bit
        graphed = run_graphed(dec, ids, steps) if dec.graphs_supported(dev) else None
        torch.cuda.synchronize()
        if rank == 0:
            ref = run(Bolt3Decoder(model), ids, steps)
            torch.save({"got": got, "ref": ref, "graphed": graphed, "world": dist.get_world_size()}, args.out)
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
