"""Bolt-3 hot-path benchmark: prefill tok/s and decode tok/s on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference]

One process per GPU (launched by torch.distributed.run for N > 1). Prefill is weak-scaled: every
rank runs its own configs[1] workload (8 x 8192 tokens, Qwen3-4B shape); decode shards the 256
sequences of configs[2] across ranks. Inputs are seeded synthetic tensors; weights are seeded
random values of the Bolt3Attn parameter set. Rank 0 prints one JSON line.

`--impl reference` times the reference algorithm's CPU implementation (the oracle port of
vsa_lm/config/bolt3.py, fp32, all host threads) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from vsa_lm_b200.roofline import decode_step_bytes, prefill_flops  # noqa: E402
from vsa_lm_b200.workloads import layer_cfg, make_input, make_params  # noqa: E402

METRIC = "Bolt3 prefill tok/s + decode tok/s, Qwen3-4B shape, 1-8 B200, % roofline"
SHAPE = "qwen3_4b"
PREFILL_B, PREFILL_T, DUP = 8, 8192, 0.3
DEC_SEQ, DEC_PROMPT, DEC_STEPS = 256, 4096, 512
LONG_T = 131072


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def profile_traffic():
    """Per-launch DRAM bytes of kernels captured with ncu (profiles/traffic.json), if present."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    return json.load(open(p)) if os.path.exists(p) else {}


def pci_bus_id(dev) -> str:
    """The PCI bus id of a CUDA device as nvidia-smi names it. nvidia-smi ignores
    CUDA_VISIBLE_DEVICES, so on a leased GPU its index would select another device."""
    p = torch.cuda.get_device_properties(dev)
    return f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"


class Clocks:
    """Samples nvidia-smi clocks and throttle reasons of one GPU (by PCI bus id) while the timed
    region runs."""

    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, dev):
        self.bus_id, self.proc, self.out = pci_bus_id(dev), None, None

    def __enter__(self):
        try:
            self.out = open(os.path.join("/tmp", f"bolt3_clocks_{os.getpid()}.csv"), "w+")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self.bus_id, f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.out, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            self.proc.wait(timeout=10)

    def summary(self):
        if self.proc is None or self.out is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"],
                    "gpu_pci_bus_id": self.bus_id}
        self.out.seek(0)
        rows = [r.split(",") for r in self.out.read().strip().splitlines() if r.strip()]
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[0]))
                mx = float(r[1])
                for n, v in zip(names, r[3:7]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "samples": len(sm),
                "reasons": sorted(reasons), "gpu_pci_bus_id": self.bus_id}


def timed(fn, steps: int, warmup: int, world: int, stream=None):
    """Run fn() warmup + steps times; return max-over-ranks seconds of the `steps` timed calls."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        fn()
    e.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t = torch.tensor([s.elapsed_time(e) / 1e3], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def timed_e2e(m, xh, yh, dev, steps: int, warmup: int, world: int) -> float:
    """Seconds (max over ranks) for `steps` forwards through the public module, each with its input
    copied host -> device and its output device -> host inside the timed region. Copies run on their
    own streams with three device input buffers, so uploads, the forward and downloads of
    neighbouring steps overlap (the two PCIe directions run concurrently)."""
    main = torch.cuda.current_stream()
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    n_buf = 3
    xd = [torch.empty(xh.shape, dtype=xh.dtype, device=dev) for _ in range(n_buf)]
    freed = [torch.cuda.Event() for _ in range(n_buf)]   # compute has finished reading xd[slot]
    for ev in freed:
        ev.record(main)

    def run(n):
        for i in range(n):
            slot = i % n_buf
            with torch.cuda.stream(h2d):
                h2d.wait_event(freed[slot])
                xd[slot].copy_(xh, non_blocking=True)
                arrived = torch.cuda.Event()
                arrived.record(h2d)
            main.wait_event(arrived)
            y = m(xd[slot])
            freed[slot].record(main)
            done = torch.cuda.Event()
            done.record(main)
            with torch.cuda.stream(d2h):
                d2h.wait_event(done)
                yh[i % len(yh)].copy_(y, non_blocking=True)
                y.record_stream(d2h)
        main.wait_stream(d2h)

    run(warmup)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    run(steps)
    e.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t = torch.tensor([s.elapsed_time(e) / 1e3], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def build_layer(device):
    from vsa_lm_b200 import Bolt3Attn

    cfg = layer_cfg(SHAPE)
    m = Bolt3Attn(cfg)
    m.load_state_dict(make_params(cfg, 0))
    return cfg, m.to(device=device, dtype=torch.bfloat16).eval()


def phase_times(m, x, reps: int = 3):
    """CUDA-event time of each phase of one prefill (same launches as forward, timed one by one)."""
    from vsa_lm_b200 import kernels as K

    b, T, D = x.shape
    H, HKV, HD = m.H, m.HKV, m.HD
    dev = x.device
    f = m.fused(dev)
    c = f.consts
    bf = dict(dtype=torch.bfloat16, device=dev)
    q_raw, q_rope = torch.empty(b * H, T, HD, **bf), torch.empty(b * H, T, HD, **bf)
    k_raw, k_rope, v = (torch.empty(b * HKV, T, HD, **bf) for _ in range(3))
    beta = torch.empty(b * HKV, T, dtype=torch.float32, device=dev)
    eta = torch.empty(b * H, T, dtype=torch.float32, device=dev)
    q_l2 = torch.empty(b * H, T, dtype=torch.float32, device=dev)
    ws = torch.empty(max(1, K.prefill_workspace_bytes(b * HKV, T, HD)), dtype=torch.uint8, device=dev)
    bank = K.new_bank(b * HKV, HD, dev)
    y = torch.empty(b, T, H, HD, **bf)
    x2 = x.reshape(b * T, D)
    proj = m.project(x2, f)
    lib = K._lib.load()
    import ctypes

    from vsa_lm_b200 import _lib

    def prep():
        K.prep(proj, B=b, T=T, H=H, HKV=HKV, HD=HD, inv_freq=c["inv_freq"], eps=m.eps, q_norm_w=c["qn"],
               k_norm_w=c["kn"], pos0=0, cols=f.cols, q_raw=q_raw, q_rope=q_rope, eta=eta, k_raw=k_raw, k_rope=k_rope,
               v=v, beta=beta, q_head_stride=T, q_t_off=0, k_head_stride=T, k_t_off=0, q_l2=q_l2)

    n_cons = K.n_consolidations(T)
    snap = {}
    off = 0

    def carve(nbytes):
        nonlocal off
        t = ws[off:off + nbytes]
        off = (off + nbytes + 255) // 256 * 256
        return t

    ns = b * HKV * n_cons
    snap["ak_rope"] = carve(ns * 128 * HD * 2).view(torch.bfloat16).view(b * HKV, n_cons, 128, HD)
    snap["av"] = carve(ns * 128 * HD * 2).view(torch.bfloat16).view(b * HKV, n_cons, 128, HD)
    snap["mass"] = carve(ns * 128 * 4).view(torch.float32)
    snap["act"] = carve(ns * 128)
    snap["m"] = carve(ns * HD * HD * 4).view(torch.float32)

    def scan():
        K.consolidate(n_chains=b * HKV, hkv=HKV, HD=HD, bank=bank, init_blank=True, kr=k_raw, kp=k_rope, v=v,
                      beta=beta, chain_tokens=T, token0=0, step_tokens=128, skip0=4, chunk_len=128, pos0=0,
                      n_steps=n_cons, kappa=c["kappa"], gamma=c["gamma"], inv_freq=c["inv_freq"], snaps=snap)

    def attend():
        a = _lib.AttendArgs(
            n_chains=b * HKV, hkv=HKV, G=H // HKV, HD=HD, q_rope=q_rope.data_ptr(), q_raw=q_raw.data_ptr(),
            eta=eta.data_ptr(), Tq=T, prefill=1, seg0_k=k_rope.data_ptr(), seg0_v=v.data_ptr(),
            seg0_chain_tokens=T, seg1_k=k_rope.data_ptr(), seg1_v=v.data_ptr(), seg1_chain_tokens=T,
            bank_ak_rope=snap["ak_rope"].data_ptr(), bank_av=snap["av"].data_ptr(),
            bank_mass=snap["mass"].data_ptr(), bank_act=snap["act"].data_ptr(), bank_m=snap["m"].data_ptr(),
            bank_cap=n_cons, kappa=c["kappa"].data_ptr(), coef=c["coef"].data_ptr(),
            res_w=c["res_w"].data_ptr(), eps=m.eps, y=y.data_ptr(), y_tokens=T, q_l2=q_l2.data_ptr())
        _lib.check(lib.bolt3_attend(ctypes.byref(a), torch.cuda.current_stream().cuda_stream), "attend")

    phases = {
        "proj_in": lambda: m.project(x2, f),
        "prep": prep,
        "consolidate": scan,
        "attend": attend,
        "proj_out": lambda: torch.nn.functional.linear(y.view(b, T, H * HD), f.w_out),
    }
    out = {}
    for name, fn in phases.items():
        fn()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(reps):
            fn()
        e.record()
        torch.cuda.synchronize()
        out[name] = s.elapsed_time(e) / 1e3 / reps
    return out


def run_native(args, rank, world, local):
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    hbm, tf_burst, tf_sus, peak_kind = peaks()
    cfg, m = build_layer(dev)
    D, H, HKV, HD = cfg["dim"], m.H, m.HKV, m.HD
    B, T = args.batch, args.seq
    x = make_input(B, T, D, dup=DUP, seed=1 + rank, device=dev, dtype=torch.bfloat16)

    def step():
        m(x)

    from vsa_lm_b200 import kernels as K

    c0 = K.launch_count()
    step()
    launches_per_step = K.launch_count() - c0  # this library's kernels in one step (cuBLAS GEMMs excluded)
    with Clocks(dev) as clk:
        t_prefill = timed(step, args.steps, args.warmup, world)
    clocks = clk.summary()
    tok = B * T
    value = world * tok * args.steps / t_prefill
    flops = prefill_flops(B, T, D, H, HKV, HD)

    # per-phase times and the dominant kernel's roofline
    ph = phase_times(m, x)
    traffic = profile_traffic()
    ours = {"prep": None, "consolidate": "consolidate", "attend": "attend"}
    phase_rl = {}
    for name, t in ph.items():
        if name in ("proj_in", "proj_out", "attend", "consolidate"):
            ach = flops[name] / t / 1e12
            phase_rl[name] = {"ms": t * 1e3, "bound": "tensor", "achieved": ach, "unit": "TFLOP/s",
                              "frac": ach / tf_burst}
        else:  # prep: HBM-bound elementwise
            nbytes = tok * ((H * HD + 2 * HKV * HD + HKV + H) * 2 + (2 * H * HD + 3 * HKV * HD) * 2 + (H + HKV) * 4)
            ach = nbytes / t / 1e9
            phase_rl[name] = {"ms": t * 1e3, "bound": "hbm", "achieved": ach, "unit": "GB/s", "frac": ach / hbm}
    own = {k: v for k, v in ph.items() if k in ("prep", "consolidate", "attend")}
    dom = max(own, key=own.get)
    rl = dict(phase_rl[dom])
    rl.pop("ms")
    rl["kernel"] = dom
    rl["peak"] = tf_burst if rl["bound"] == "tensor" else hbm
    rl["peak_source"] = peak_kind
    rl["traffic"] = traffic.get(dom)
    step_rl = flops["total"] / (t_prefill / args.steps) / 1e12

    # end-to-end through the public module: every step copies its input from pinned host memory
    # and its output back to pinned host memory, pipelined as a serving host would run it
    xh = x.cpu().pin_memory()
    yh = [torch.empty(B, T, D, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    e2e_steps = max(48, args.steps)  # pipeline fill and drain (one upload, one download) amortised
    t_e2e = timed_e2e(m, xh, yh, dev, e2e_steps, max(1, args.warmup), world)
    e2e_value = world * tok * e2e_steps / t_e2e

    decode = None if args.no_decode else run_decode(args, rank, world, dev, m, cfg, hbm)
    decode_tp = run_decode_tp(args, rank, world, dev, m, cfg) if (world > 1 and not args.no_decode) else None
    long_ctx = None if args.no_long else run_long(args, rank, world, dev, tf_burst, steps=3, warmup=3)
    torch.cuda.empty_cache()
    full = None
    if not args.no_full:
        # a secondary leg: an error there is reported in the line instead of failing the run
        try:
            full = run_full_model(args, rank, world, dev)
        except Exception as exc:  # noqa: BLE001
            full = {"error": f"{type(exc).__name__}: {exc}"[:300]}
            torch.cuda.empty_cache()
    legs = cpu_baseline(args, m, cfg, dev) if (rank == 0 and world == 1 and not args.no_cpu) else {}
    cpu = legs.get("prefill")
    if decode is not None and legs:
        decode["cpu_baseline"] = legs["decode"]
    res = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t_prefill / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"configs[1]: Bolt3Attn prefill, Qwen3-4B shape (D2560 H32/8 HD128 theta1e6 "
                               f"qk_norm), {B} x {T} tokens per GPU, 30% near-duplicates, seeded random weights",
                   "global_batch": B * world, "seq_len": T, "parallelism": f"dp{world} (sequence batches)",
                   "l2": "inputs and intermediates larger than L2 (x alone 335 MB)"},
        "roofline": rl,
        "prefill_step_roofline": {"bound": "tensor", "achieved": step_rl, "peak": tf_burst, "unit": "TFLOP/s",
                                  "frac": step_rl / tf_burst, "flops_per_token": flops["total"] / tok},
        "phases": phase_rl,
        "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": xh.numel() * 2,
                "d2h_bytes_per_step": yh[0].numel() * 2, "steps": e2e_steps,
                "pipelining": "per-step copies on two copy streams, three device input buffers"},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
        "decode": decode,
        "decode_tp": decode_tp,
        "long_context": long_ctx,
        "full_model": full,
        "cpu_baseline": cpu,
    }
    if "parity" in legs:
        res["parity"] = legs["parity"]
    return res


def run_decode(args, rank, world, dev, m, cfg, hbm):
    """one Bolt-3 layer, 256 sequences (sharded), 4096-token prefill, then decode steps."""
    from vsa_lm_b200 import Bolt3Decoder, Bolt3LayerState

    n_seq = DEC_SEQ // world
    D = cfg["dim"]
    st = Bolt3LayerState(m, n_seq, dev)
    m_res = torch.zeros(n_seq, m.HKV, m.HD, m.HD, device=dev)
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    for s in range(0, DEC_PROMPT, 128):
        h = torch.randn(n_seq, 128, D, generator=g, device=dev).to(torch.bfloat16)
        Bolt3Decoder.layer_step(m, st, h, s, m_res)
    steps = args.decode_steps
    toks = torch.randn(steps + args.warmup, n_seq, 1, D, generator=g, device=dev).to(torch.bfloat16)
    pos = [DEC_PROMPT]
    i = [0]

    def one():
        Bolt3Decoder.layer_step(m, st, toks[i[0]], pos[0], m_res)
        pos[0] += 1
        i[0] += 1

    for _ in range(args.warmup):
        one()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        one()
    e.record()
    torch.cuda.synchronize()
    t = torch.tensor([s.elapsed_time(e) / 1e3], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    t = float(t.item())
    nb = decode_step_bytes(n_seq, D, m.H, m.HKV, m.HD)
    ach = nb["total"] * steps / t / 1e9
    ach_core = nb["state"] * steps / t / 1e9
    return {"value": world * n_seq * steps / t, "unit": "tok/s", "steps": steps, "seqs_per_gpu": n_seq,
            "prompt": DEC_PROMPT, "ms_per_step": t / steps * 1e3,
            "workload": "configs[2]: one Bolt-3 layer step (projections, attention, o_proj, consolidation "
                        "every 128 steps), 256 sequences after a 4096-token prefill",
            "roofline": {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm,
                         "attend_traffic": profile_traffic().get("attend_decode"),
                         "bytes_per_step": nb["total"], "state_only_frac": ach_core / hbm}}


FULL_B, FULL_T, FULL_NEW = 64, 2048, 256


def run_full_model(args, rank, world, dev):
    """the whole hybrid model (Qwen3-4B architecture: 36 layers, 27 Bolt-3 and 9 softmax
    anchors, SwiGLU 9728, vocab 151936, seeded random weights drawn on the GPU), 64 prompts of 2048
    random token ids prefilled through the decoder, then greedy decoding of 256 tokens with the
    logits read on the device. Under torchrun the model is split over the N ranks (Bolt3LMTP:
    attention by KV head, the MLP by feature, an NCCL all-reduce of fp32 partials after each) and
    every rank steps all 64 sequences. The prompt prefill and the decode steps are timed separately
    with CUDA events (max over ranks), after one warm-up round."""
    from vsa_lm_b200 import Bolt3Decoder
    from vsa_lm_b200.model import Bolt3LM
    from vsa_lm_b200.tp import Bolt3DecoderTP, Bolt3LMTP
    from vsa_lm_b200.workloads import MODEL_SHAPES, init_model_on_device

    mcfg = dict(MODEL_SHAPES["qwen3_4b_lm"])
    with torch.device(dev):
        model = Bolt3LM(**mcfg)
    init_model_on_device(model, seed=0)     # the same weights on every rank
    # the device move also takes the RoPE frequency buffers, which the modules create on the host
    model = model.to(device=dev, dtype=torch.bfloat16).eval()
    if world > 1:
        model = Bolt3LMTP(model)            # this rank's shards; the unsharded blocks are released
        torch.cuda.empty_cache()
        dec = Bolt3DecoderTP(model)
    else:
        dec = Bolt3Decoder(model)
    B, T, n_new = FULL_B, FULL_T, args.full_new_tokens
    ids = torch.randint(0, mcfg["vocab_size"], (B, T), generator=torch.Generator(device=dev).manual_seed(100),
                        device=dev)

    graphs = dec.graphs_supported(dev)
    captures = [0]

    @torch.no_grad()
    def greedy(h, states, kv, n):
        # one-token steps replayed from CUDA graphs (captured once per chunk of 128 positions, inside
        # the timed region), as Bolt3Decoder.generate_batch runs them
        logits = model.lm_head(h[:, -1, :])
        runner = dec.step_graph(states, kv) if graphs else None
        for i in range(n):
            nxt = logits.argmax(-1, keepdim=True)
            if runner is not None:
                h = runner.step(nxt, T + i)
            else:
                h, states, kv = dec.step(nxt, T + i, states, kv)
            logits = model.lm_head(h[:, -1, :])
        if runner is not None:
            captures[0] = runner.captures
            runner.close()          # its graphs hold NCCL calls under torchrun: released before teardown
        return logits

    def ev():
        return torch.cuda.Event(enable_timing=True)

    # warm-up round: plans, workspaces, library heuristics
    h, states, kv = dec.prefill(ids, max_kv_len=T + n_new + 64)
    greedy(h, states, kv, 8)
    del h, states, kv
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1, e2 = ev(), ev(), ev()
    e0.record()
    h, states, kv = dec.prefill(ids, max_kv_len=T + n_new + 64)
    e1.record()
    greedy(h, states, kv, n_new)
    e2.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / 1e3, e1.elapsed_time(e2) / 1e3], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    t_pre, t_dec = float(t[0]), float(t[1])
    n_vsa = sum(1 for lt in model.config["layer_types"] if lt == "vsa")
    del model, dec, h, states, kv
    torch.cuda.empty_cache()
    return {"workload": f"configs[3]: hybrid LM with the Qwen3-4B architecture ({mcfg['num_layers']} layers, {n_vsa} "
                        f"Bolt-3, hybrid_every {mcfg['hybrid_every']}, SwiGLU {mcfg['intermediate']}, vocab "
                        f"{mcfg['vocab_size']}), seeded random weights, {B} prompts of {T} random token ids, "
                        f"then {n_new} greedy tokens",
            "parallelism": (f"tp{world}: attention split by KV head, the MLP by intermediate feature, an NCCL "
                            f"all-reduce of the fp32 partial sums after every attention and every MLP (72 per step)"
                            if world > 1 else "one GPU"),
            "prefill": {"value": B * T / t_pre, "unit": "tok/s", "ms": t_pre * 1e3},
            "decode": {"value": B * n_new / t_dec, "unit": "tok/s", "ms_per_step": t_dec / n_new * 1e3,
                       "steps": n_new, "sequences": B, "cuda_graphs": graphs, "graph_captures": captures[0]}}


def run_anchor(args, dev, hbm):
    """The softmax anchors' one-token attention (bolt3_anchor_decode) at configs[3]'s decode shape:
    64 sequences x 8 KV heads x 4 query heads, HD 128, 2200 cached tokens (the middle of the 256
    decode steps after a 2048-token prompt). L2 is flushed before every timed launch."""
    from vsa_lm_b200 import kernels as K

    B, HKV, G, HD, n, cap = FULL_B, 8, 4, 128, 2200, 2368
    g = torch.Generator(device=dev).manual_seed(11)
    mk = lambda *shape: torch.randn(*shape, generator=g, device=dev).to(torch.bfloat16)
    q, kn, vn = mk(B, HKV * G, HD), mk(B, HKV, HD), mk(B, HKV, HD)
    kc, vc = mk(B, HKV, cap, HD), mk(B, HKV, cap, HD)
    y = torch.empty_like(q)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    ts = []
    for i in range(args.warmup + args.steps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        K.anchor_decode(q=q, k_new=kn, v_new=vn, k_cache=kc, v_cache=vc, n=n, y=y, scale=HD ** -0.5)
        e1.record()
        torch.cuda.synchronize()
        if i >= args.warmup:
            ts.append(e0.elapsed_time(e1) / 1e3)
    t = sorted(ts)[len(ts) // 2]
    nb = B * HKV * (n + 1) * HD * 2 * 2
    return {"workload": f"configs[3] anchor decode step: {B} sequences x {HKV} KV heads x {G} query heads, HD {HD}, "
                        f"{n} cached tokens", "us": t * 1e6, "bytes": nb,
            "roofline": {"bound": "hbm", "achieved": nb / t / 1e9, "peak": hbm, "unit": "GB/s",
                         "frac": nb / t / 1e9 / hbm}}


def run_decode_tp(args, rank, world, dev, m, cfg):
    """configs[2] decode with the layer split by KV head over the N ranks (Bolt3AttnTP): every rank
    steps all 256 sequences on its KV heads and the o_proj partials meet in one NCCL all-reduce per
    step. Total work is fixed, so this is the strong-scaling alternative to sharding sequences."""
    from vsa_lm_b200.tp import Bolt3AttnTP

    tp = Bolt3AttnTP(m)
    n_seq, D = DEC_SEQ, cfg["dim"]
    st, m_res = tp.new_decode_state(n_seq, dev)
    g = torch.Generator(device=dev).manual_seed(100)
    for s in range(0, DEC_PROMPT, 128):
        tp.decode_step(st, torch.randn(n_seq, 128, D, generator=g, device=dev).to(torch.bfloat16), s, m_res)
    steps = min(args.decode_steps, 128)
    toks = torch.randn(steps + args.warmup, n_seq, 1, D, generator=g, device=dev).to(torch.bfloat16)
    pos, i = [DEC_PROMPT], [0]

    def one():
        tp.decode_step(st, toks[i[0]], pos[0], m_res)
        pos[0] += 1
        i[0] += 1

    t = timed(one, steps, args.warmup, world)
    return {"value": n_seq * steps / t, "unit": "tok/s", "ms_per_step": t / steps * 1e3, "steps": steps,
            "sequences": n_seq, "parallelism": f"tp{world} by KV head",
            "collective": "NCCL all-reduce of the fp32 o_proj partials, one per step"}


def run_long(args, rank, world, dev, tf_peak, steps=None, warmup=None):
    """Llama-3-8B-shape Bolt3Attn prefill of 1 x 131072 tokens. On N GPUs every rank
    holds HKV/N KV heads (Bolt3AttnTP: one NCCL all-reduce of the o_proj partials per forward)."""
    steps = args.steps if steps is None else steps
    warmup = args.warmup if warmup is None else warmup
    from vsa_lm_b200 import Bolt3Attn
    from vsa_lm_b200.tp import Bolt3AttnTP

    cfg = layer_cfg("llama3_8b")
    full = Bolt3Attn(cfg)
    full.load_state_dict(make_params(cfg, 0))
    full = full.to(device=dev, dtype=torch.bfloat16).eval()
    layer = Bolt3AttnTP(full) if world > 1 else full
    T = LONG_T
    x = make_input(1, T, cfg["dim"], dup=0.2, seed=7, device=dev, dtype=torch.bfloat16)
    t = timed(lambda: layer(x), steps, warmup, world)
    flops = prefill_flops(1, T, cfg["dim"], full.H, full.HKV, full.HD)["total"]
    return {"value": T * steps / t, "unit": "tok/s", "ms_per_step": t / steps * 1e3, "steps": steps,
            "warmup": warmup, "collective": "NCCL all-reduce of the fp32 o_proj partials" if world > 1 else None,
            "workload": "configs[4]: Bolt3Attn prefill, Llama-3-8B shape (D4096 H32/8 HD128 theta5e5), "
                        "1 x 131072 tokens, 20% near-duplicates, seeded random weights",
            "parallelism": f"tp{world} by KV head" if world > 1 else "one GPU, all 8 KV heads",
            "roofline": {"bound": "tensor", "achieved": flops * args.steps / t / 1e12, "peak": tf_peak,
                         "unit": "TFLOP/s", "frac": flops * args.steps / t / 1e12 / tf_peak}}


def _oracle_setup(m, cfg):
    from oracle import oracle_cfg

    P = {k: v.detach().cpu() for k, v in m.state_dict().items()}
    oc = oracle_cfg(cfg)
    oc["inv_freq"] = m.rope.inv_freq.detach().float().cpu()
    return P, oc


def _flag_counts(rec: list) -> tuple:
    """Per consolidation, the chains whose outcome rounding may change; totals split by reason."""
    from oracle.parity import decision_ties, near_threshold

    flags = [decision_ties(r) for r in rec]
    thr = sum(int(near_threshold(r).sum()) for r in rec)
    return flags, thr, sum(int(f.sum()) for f in flags) - thr


def parity_prefill(m, cfg, dev, n_seq: int = 2):
    """configs[1] check: n_seq sequences of PREFILL_T tokens through Bolt3Attn's native forward,
    against the oracle run on the GPU's own projections. A chain may deviate from the oracle only
    after a consolidation whose decision rounding can change (oracle.parity.decision_ties); such
    chains are counted as flips."""
    from oracle import Store, forward

    T = PREFILL_T
    x = make_input(n_seq, T, cfg["dim"], dup=DUP, seed=1, device=dev, dtype=torch.bfloat16)
    P, oc = _oracle_setup(m, cfg)
    p, prep_q = m._prepare(x)
    prep_q()
    H, HKV, HD, G = m.H, m.HKV, m.HD, m.G
    cpu = lambda t, *shape: t.float().cpu().view(*shape)
    proj = (cpu(p.q_raw, n_seq, H, T, HD), cpu(p.k_raw, n_seq, HKV, T, HD), cpu(p.v, n_seq, HKV, T, HD),
            cpu(p.beta, n_seq, HKV, T), cpu(p.eta, n_seq, H, T))
    rec = []
    _, yh_ref = forward(P, oc, x, Store("bf16"), record=rec, return_y_heads=True, proj=proj)
    got = m._attention_heads(x).float().cpu().permute(0, 2, 1, 3)
    m.check_status()
    flags, thr, tie = _flag_counts(rec)
    rms = yh_ref.pow(2).mean().sqrt().item()
    n_chunks = T // 128
    gone, unflagged, worst, compared = {}, 0, 0.0, 0
    for r in range(n_chunks):
        for c in range(n_seq * HKV):
            if c in gone:
                continue
            bi, h = divmod(c, HKV)
            g_ = got[bi, h * G:(h + 1) * G, r * 128:(r + 1) * 128]
            f_ = yh_ref[bi, h * G:(h + 1) * G, r * 128:(r + 1) * 128]
            err = (g_ - f_).abs()
            if (err > 2e-2 * f_.abs() + 2e-2 * rms).any():
                gone[c] = r
                unflagged += not any(bool(flags[j][c]) for j in range(0, r - 1))
                continue
            worst = max(worst, err.max().item() / rms)
            compared += 1
    steps = len(rec) * n_seq * HKV
    return {"sample": f"{n_seq} sequences x {T} tokens (configs[1] shape), oracle on the GPU's projections",
            "chain_steps": steps, "flagged_near_threshold": thr, "flagged_near_tie": tie, "flips": len(gone),
            "unflagged_deviations": unflagged, "flip_rate": len(gone) / max(steps, 1),
            "compared_chain_chunks": compared, "total_chain_chunks": n_chunks * n_seq * HKV,
            "max_err_rel_rms": worst, "tolerance": "rtol 2e-2, atol 2e-2 x RMS"}


def parity_decode(m, cfg, dev, n_seq: int = 4, prompt: int = DEC_PROMPT, steps: int = DEC_STEPS):
    """configs[2] check: n_seq sequences, a prompt of `prompt` tokens in C-token slices then
    `steps` one-token steps through Bolt3Decoder.layer_step, against the oracle's decoder run on the
    GPU's projections of every step. A sequence may deviate only after a consolidation of one of its
    chains whose decision rounding can change; it is then counted as a flip and left out."""
    from oracle import LayerDecoderOracle, Store
    from vsa_lm_b200 import Bolt3Decoder, Bolt3LayerState

    P, oc = _oracle_setup(m, cfg)
    g = torch.Generator(device=dev).manual_seed(200)
    hs = torch.randn(n_seq, prompt + steps, cfg["dim"], generator=g, device=dev).to(torch.bfloat16)
    st = Bolt3LayerState(m, n_seq, dev)
    m_res = torch.zeros(n_seq, m.HKV, m.HD, m.HD, device=dev)
    dec = LayerDecoderOracle(P, oc, n_seq, Store("bf16"))
    plan = [(s, 128) for s in range(0, prompt, 128)] + [(prompt + i, 1) for i in range(steps)]
    gone, unflagged, worst, compared = {}, 0, 0.0, 0
    for pos, n in plan:
        h = hs[:, pos:pos + n]
        proj = tuple(t.float().cpu() for t in m.step_projections(h, pos))
        out = Bolt3Decoder.layer_step(m, st, h, pos, m_res).float().cpu()
        ref = dec.step(h, pos, proj=proj)
        rms = ref.pow(2).mean().sqrt().item()
        for bi in range(n_seq):
            if bi in gone:
                continue
            err = (out[bi] - ref[bi]).abs()
            if (err > 2e-2 * ref[bi].abs() + 2e-2 * rms).any():
                gone[bi] = pos
                flags, _, _ = _flag_counts(dec.record)
                mine = range(bi * m.HKV, (bi + 1) * m.HKV)
                unflagged += not any(bool(f[c]) for f in flags for c in mine)
                continue
            worst = max(worst, err.max().item() / rms)
            compared += 1
    Bolt3Decoder.check_status([st])
    _, thr, tie = _flag_counts(dec.record)
    chain_steps = len(dec.record) * n_seq * m.HKV
    return {"sample": f"{n_seq} sequences, {prompt}-token prompt + {steps} one-token steps (configs[2] shape), "
                      f"oracle on the GPU's projections",
            "chain_steps": chain_steps, "flagged_near_threshold": thr, "flagged_near_tie": tie,
            "flips": len(gone), "unflagged_deviations": unflagged, "flip_rate": len(gone) * m.HKV / max(chain_steps, 1),
            "compared_sequence_steps": compared, "total_sequence_steps": len(plan) * n_seq,
            "max_err_rel_rms": worst, "tolerance": "rtol 2e-2, atol 2e-2 x RMS"}


def cpu_prefill_rate(seconds: float, T: int) -> dict:
    """The reference algorithm's prefill (the oracle port, fp32) on the host cores: forwards of
    1 x T tokens of the configs[1] shape for about `seconds`."""
    from oracle import Store, forward, oracle_cfg

    torch.set_num_threads(os.cpu_count() or 1)
    cfg = layer_cfg(SHAPE)
    P = make_params(cfg, 0)
    oc = oracle_cfg(cfg)
    x = make_input(1, T, cfg["dim"], dup=DUP, seed=1)
    t0 = time.perf_counter()
    n = 0
    while True:
        forward(P, oc, x, Store("fp32"))
        n += 1
        if time.perf_counter() - t0 > seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": n * T / dt, "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"configs[1] shape, 1 x {T} tokens, fp32, {n} forward(s) in {dt:.1f} s"}


def cpu_decode_rate(seconds: float, B: int = 8, prompt: int = 512) -> dict:
    """The reference algorithm's decode step (the oracle port of Bolt3Decoder.step for one Bolt-3
    layer, fp32) on the host cores: B sequences after a `prompt`-token prefill (untimed), then
    one-token steps for about `seconds`."""
    from oracle import LayerDecoderOracle, Store, oracle_cfg

    torch.set_num_threads(os.cpu_count() or 1)
    cfg = layer_cfg(SHAPE)
    P = make_params(cfg, 0)
    oc = oracle_cfg(cfg)
    g = torch.Generator().manual_seed(300)
    dec = LayerDecoderOracle(P, oc, B, Store("fp32"))
    for s in range(0, prompt, 128):
        dec.step(torch.randn(B, 128, cfg["dim"], generator=g), s)
    pos, n = prompt, 0
    t0 = time.perf_counter()
    while True:
        dec.step(torch.randn(B, 1, cfg["dim"], generator=g), pos)
        pos, n = pos + 1, n + 1
        if time.perf_counter() - t0 > seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": B * n / dt, "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"configs[2] shape, {B} sequences after a {prompt}-token prefill, {n} one-token steps "
                      f"of one Bolt-3 layer, fp32, in {dt:.1f} s"}


def cpu_baseline(args, m=None, cfg=None, dev=None):
    """The CPU leg (rank 0, one GPU, outside every timed region): the reference algorithm on the host
    cores (the oracle port, fp32), timed on bounded samples of the prefill and the decode step; and
    the same oracle as the checker of the GPU path's results on configs[1]- and configs[2]-shaped
    samples (parity and the merge/evict flip rate)."""
    out = {"prefill": cpu_prefill_rate(args.cpu_seconds, args.cpu_tokens),
           "decode": cpu_decode_rate(args.cpu_seconds / 2)}
    if m is not None and not args.no_parity:
        out["parity"] = {"configs[1]": parity_prefill(m, cfg, dev),
                         "configs[2]": parity_decode(m, cfg, dev, steps=args.parity_decode_steps)}
    return out


def run_reference(args, rank, world):
    """The reference arm: the reference algorithm (CPU oracle port, fp32) on the host cores, with
    all host threads, on configs[1]'s shape. Each of the --warmup untimed and --steps timed steps is
    one bounded sample: a forward of 1 x --cpu-tokens tokens. Rank 0 only."""
    if rank != 0:
        return None
    from oracle import Store, forward, oracle_cfg

    torch.set_num_threads(os.cpu_count() or 1)
    cfg = layer_cfg(SHAPE)
    P = make_params(cfg, 0)
    oc = oracle_cfg(cfg)
    T = args.cpu_tokens
    x = make_input(1, T, cfg["dim"], dup=DUP, seed=1)
    for _ in range(args.warmup):
        forward(P, oc, x, Store("fp32"))
    t0 = time.perf_counter()
    for _ in range(args.steps):
        forward(P, oc, x, Store("fp32"))
    dt = time.perf_counter() - t0
    value = args.steps * T / dt
    sample = f"configs[1] shape, 1 x {T} tokens per step, fp32, {args.steps} timed step(s) in {dt:.1f} s"
    decode = cpu_decode_rate(args.cpu_seconds / 2)
    return {"metric": METRIC, "impl": "reference", "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "configs[1]: Bolt3Attn prefill, Qwen3-4B shape (D2560 H32/8 HD128 theta1e6 "
                                   "qk_norm), 30% near-duplicates, seeded random weights; reference algorithm on "
                                   "the host cores, a bounded sample per step",
                       "global_batch": 1, "seq_len": T, "parallelism": "host threads"},
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "decode": {"value": decode["value"], "unit": "tok/s", "cpu_baseline": decode}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--cpu-tokens", type=int, default=2048)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--batch", type=int, default=PREFILL_B, help="prefill sequences per GPU (profiling cases)")
    ap.add_argument("--seq", type=int, default=PREFILL_T, help="prefill tokens per sequence (profiling cases)")
    ap.add_argument("--decode-only", action="store_true", help="only the configs[2] decode measurement (profiling)")
    ap.add_argument("--decode-steps", type=int, default=DEC_STEPS, help="timed decode steps")
    ap.add_argument("--long", action="store_true", help="only the configs[4] long-context prefill")
    ap.add_argument("--no-parity", action="store_true", help="skip the oracle check of the GPU results")
    ap.add_argument("--no-long", action="store_true", help="skip the configs[4] leg of the default line")
    ap.add_argument("--full-model", action="store_true", help="only the configs[3] whole-model leg")
    ap.add_argument("--no-full", action="store_true", help="skip the configs[3] leg of the default line")
    ap.add_argument("--full-new-tokens", type=int, default=FULL_NEW, help="greedy tokens of the configs[3] leg")
    ap.add_argument("--anchor-only", action="store_true",
                    help="only the configs[3] softmax anchors' one-token attention kernel (profiling)")
    ap.add_argument("--parity-decode-steps", type=int, default=DEC_STEPS,
                    help="one-token steps of the configs[2] parity sample")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        # the CPU reference runs on rank 0 only; the other ranks exit without work
        res = run_reference(args, rank, world)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    if world > 1:
        from datetime import timedelta

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    try:
        if args.long:
            dev = torch.device("cuda", local)
            torch.cuda.set_device(dev)
            res = {"long_context": run_long(args, rank, world, dev, peaks()[1])}
        elif args.full_model:
            dev = torch.device("cuda", local)
            torch.cuda.set_device(dev)
            res = {"full_model": run_full_model(args, rank, world, dev)}
        elif args.anchor_only:
            dev = torch.device("cuda", local)
            torch.cuda.set_device(dev)
            res = {"anchor_decode": run_anchor(args, dev, peaks()[0])}
        elif args.decode_only:
            dev = torch.device("cuda", local)
            torch.cuda.set_device(dev)
            cfg, m = build_layer(dev)
            res = {"decode": run_decode(args, rank, world, dev, m, cfg, peaks()[0])}
        else:
            res = run_native(args, rank, world, local)
        if rank == 0 and res is not None:
            print(json.dumps(res), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
