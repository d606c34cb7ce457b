"""One rank of the two-GPU tensor-parallel check (launched by tests/test_tp.py through
torch.distributed.run; not a test module itself).

Every rank builds the same seeded Bolt-3 layer, keeps its KV heads (Bolt3AttnTP) and runs the
forward and a prompt + one-token decode steps; the o_proj partials meet in one NCCL all-reduce per
call. Rank 0 also runs the unsharded layer on the same inputs and writes both results to --out."""
import argparse
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [HERE, os.path.dirname(HERE)]

from helpers import bf16_module  # noqa: E402
from vsa_lm_b200 import Bolt3Decoder, Bolt3LayerState  # noqa: E402
from vsa_lm_b200.tp import Bolt3AttnTP  # noqa: E402
from vsa_lm_b200.workloads import layer_cfg, make_input  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    args = ap.parse_args()
    rank, local = int(os.environ["RANK"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    try:
        cfg = layer_cfg("qwen3_4b")
        m = bf16_module(cfg, 0, device=dev)
        tp = Bolt3AttnTP(m)
        x = make_input(2, 700, cfg["dim"], dup=0.3, seed=4).to(device=dev, dtype=torch.bfloat16)
        y = tp(x)
        B, prompt, n_dec = 2, 260, 20
        h = make_input(B, prompt + n_dec, cfg["dim"], dup=0.3, seed=6).to(device=dev, dtype=torch.bfloat16)
        st, m_res = tp.new_decode_state(B, dev)
        steps = [(s, min(128, prompt - s)) for s in range(0, prompt, 128)] + [(prompt + i, 1) for i in range(n_dec)]
        dec = [tp.decode_step(st, h[:, p:p + n], p, m_res) for p, n in steps]
        torch.cuda.synchronize()
        if rank == 0:
            ref_st = Bolt3LayerState(m, B, dev)
            ref_m = torch.zeros(B, m.HKV, m.HD, m.HD, device=dev)
            ref_dec = [Bolt3Decoder.layer_step(m, ref_st, h[:, p:p + n], p, ref_m) for p, n in steps]
            torch.save({"y": y.float().cpu(), "ref": m(x).float().cpu(),
                        "dec": torch.cat(dec, 1).float().cpu(), "ref_dec": torch.cat(ref_dec, 1).float().cpu(),
                        "world": dist.get_world_size()}, args.out)
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
