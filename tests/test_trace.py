"""NVTX ranges: the Python phases (kernels.traced) and the C-ABI entry points of libbolt3.so.

The C side is observed through a test-only NVTX injection library (tests/nvtx_probe.c) that NVTX
itself loads in a child process and that logs every push and pop; the entry points are called with
null arguments, which open and close their range and return an error before any CUDA call, so this
runs without a GPU. The GPU test checks the ranges of a real forward and of decode steps across a
second chunk boundary (position 256, the first consolidation).
"""
import os
import shutil
import subprocess
import sys

import pytest
import torch

from vsa_lm_b200 import kernels as K

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ENTRY_POINTS = ["bolt3_prep", "bolt3_consolidate", "bolt3_attend", "bolt3_prefill_fwd",
                "bolt3_prefill_fwd_noalloc", "bolt3_anchor_decode", "bolt3_rmsnorm", "bolt3_silu_mul"]


def _cuda_include() -> str:
    for cand in (os.environ.get("CUDA_HOME"), "/usr/local/cuda"):
        if cand and os.path.exists(os.path.join(cand, "include", "nvtx3", "nvToolsExt.h")):
            return os.path.join(cand, "include")
    nvcc = shutil.which("nvcc")
    if nvcc:
        inc = os.path.join(os.path.dirname(os.path.dirname(nvcc)), "include")
        if os.path.exists(os.path.join(inc, "nvtx3", "nvToolsExt.h")):
            return inc
    pytest.skip("the CUDA toolkit's NVTX3 headers are not here")


@pytest.fixture(scope="module")
def probe(tmp_path_factory):
    if shutil.which("gcc") is None:
        pytest.skip("gcc is not here")
    out = tmp_path_factory.mktemp("nvtx") / "nvtx_probe.so"
    subprocess.check_call(["gcc", "-shared", "-fPIC", "-O1", "-I", _cuda_include(),
                           os.path.join(ROOT, "tests", "nvtx_probe.c"), "-o", str(out)])
    return str(out)


def _run_probed(probe: str, code: str, log) -> list[str]:
    env = dict(os.environ, NVTX_INJECTION64_PATH=probe, NVTX_PROBE_LOG=str(log), PYTHONPATH=ROOT)
    subprocess.run([sys.executable, "-c", code], check=True, env=env, cwd=ROOT, timeout=300)
    return log.read_text().splitlines() if log.exists() else []


def _balanced(lines: list[str]) -> bool:
    depth = 0
    for ln in lines:
        depth += 1 if ln.startswith("push ") else -1
        if depth < 0:
            return False
    return depth == 0


def test_traced_pushes_and_pops_around_the_call(monkeypatch):
    calls = []
    monkeypatch.setattr(torch.cuda.nvtx, "range_push", lambda name: calls.append(("push", name)))
    monkeypatch.setattr(torch.cuda.nvtx, "range_pop", lambda: calls.append(("pop",)))

    @K.traced("phase")
    def ok(x, y=1):
        calls.append(("body", x, y))
        return x + y

    assert ok(2, y=3) == 5
    assert calls == [("push", "phase"), ("body", 2, 3), ("pop",)]
    assert ok.__name__ == "ok"


def test_traced_pops_when_the_call_raises(monkeypatch):
    calls = []
    monkeypatch.setattr(torch.cuda.nvtx, "range_push", lambda name: calls.append("push"))
    monkeypatch.setattr(torch.cuda.nvtx, "range_pop", lambda: calls.append("pop"))

    @K.traced("phase")
    def bad():
        raise ValueError("boom")

    with pytest.raises(ValueError):
        bad()
    assert calls == ["push", "pop"]


def test_host_phases_carry_ranges():
    from vsa_lm_b200 import bolt3, oversize
    for fn in (bolt3.Bolt3Attn._native_forward, bolt3.Bolt3Decoder.step, bolt3.Bolt3Decoder.layer_step,
               bolt3.Bolt3Decoder._consolidate_ring, bolt3._ChunkGraph._capture, bolt3._ChunkGraph._replay,
               oversize.layer_step):
        assert hasattr(fn, "__wrapped__"), fn


def test_entry_points_open_and_close_a_range_without_a_gpu(probe, tmp_path):
    names = ", ".join(repr(n) for n in ENTRY_POINTS)
    code = (
        "from vsa_lm_b200 import _lib, kernels as K\n"
        "lib = _lib.load(build_if_missing=False)\n"
        "@K.traced('outer')\n"
        "def run():\n"
        f"    for n in [{names}]:\n"
        "        assert getattr(lib, n)(None, None) == 1, n\n"
        "run()\n")
    lines = _run_probed(probe, code, tmp_path / "log.txt")
    i = lines.index("push outer")
    expect = ["push outer"] + [ln for n in ENTRY_POINTS for ln in (f"push {n}", "pop")] + ["pop"]
    assert lines[i:i + len(expect)] == expect
    assert _balanced(lines)


@pytest.mark.gpu
def test_forward_and_decode_ranges_nest(probe, tmp_path):
    code = (
        "import torch\n"
        "from vsa_lm_b200 import Bolt3Decoder\n"
        "from vsa_lm_b200.model import Bolt3LM\n"
        "from vsa_lm_b200.workloads import MODEL_SHAPES, make_model_params\n"
        "mcfg = dict(MODEL_SHAPES['small_lm'])\n"
        "model = Bolt3LM(**mcfg)\n"
        "model.load_state_dict(make_model_params(mcfg, 0), strict=True)\n"
        "model = model.to(device='cuda', dtype=torch.bfloat16).eval()\n"
        "g = torch.Generator().manual_seed(0)\n"
        "ids = torch.randint(0, mcfg['vocab_size'], (2, 40), generator=g).cuda()\n"
        "with torch.no_grad():\n"
        "    model(ids)\n"
        "dec = Bolt3Decoder(model, cuda_graphs=False)\n"
        "toks, _ = dec.generate_batch(ids, 220, temperature=0.0)\n"
        "torch.cuda.synchronize()\n")
    lines = _run_probed(probe, code, tmp_path / "log.txt")
    assert _balanced(lines)
    pushed = [ln[5:] for ln in lines if ln.startswith("push ")]
    for name in ("Bolt3Attn.forward", "bolt3_prep", "bolt3_attend", "Bolt3Decoder.step", "Bolt3Decoder.layer_step",
                 "Bolt3Decoder.consolidate", "bolt3_consolidate", "bolt3_rmsnorm"):
        assert name in pushed, name
    # every bolt3_prep of a decode step is inside a layer step
    stack = []
    for ln in lines:
        if ln.startswith("push "):
            stack.append(ln[5:])
            if ln[5:] == "bolt3_prep" and "Bolt3Attn.forward" not in stack:
                assert "Bolt3Decoder.layer_step" in stack
        else:
            stack.pop()
