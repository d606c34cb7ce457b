"""bench.py without a GPU: the clocks summary that goes into the bench line (median SM clock under
load, the maximum, the throttle reasons seen while the timed region ran), the PCI bus id that
selects the GPU for nvidia-smi, and the `--impl reference` arm end to end (one process, and two
ranks under torchrun, where rank 0 alone prints)."""
import types

import torch

import bench


def _clocks_from(text: str):
    """A Clocks whose sampler 'ran' and wrote `text` (nvidia-smi csv, noheader, nounits)."""
    import io

    c = bench.Clocks.__new__(bench.Clocks)
    c.bus_id = "00000000:1B:00.0"
    c.proc = object()
    c.out = io.StringIO(text)
    return c


def test_clock_summary_takes_the_median_and_every_reason_seen():
    rows = [
        "1965, 1965, 700.1, Not Active, Not Active, Not Active, Not Active",
        "1950, 1965, 980.4, Not Active, Not Active, Not Active, Active",
        "1900, 1965, 1001.0, Not Active, Not Active, Not Active, Active",
        "garbage line",
        "[N/A], 1965, 650.0, Not Active, Not Active, Not Active, Not Active",
    ]
    s = _clocks_from("\n".join(rows) + "\n").summary()
    assert s["sm_mhz"] == 1950.0 and s["sm_max_mhz"] == 1965.0 and s["samples"] == 3
    assert s["reasons"] == ["sw_power_cap"]
    assert s["gpu_pci_bus_id"] == "00000000:1B:00.0"


def test_clock_summary_reports_slowdowns():
    rows = ["1200, 1965, 500.0, Active, Not Active, Active, Not Active"]
    s = _clocks_from("\n".join(rows)).summary()
    assert s["reasons"] == ["hw_slowdown", "sw_thermal_slowdown"]
    assert s["sm_mhz"] == 1200.0


def test_clock_summary_without_a_sampler():
    c = bench.Clocks.__new__(bench.Clocks)
    c.bus_id, c.proc, c.out = "00000000:1B:00.0", None, None
    s = c.summary()
    assert s["sm_mhz"] is None and s["reasons"] == ["nvidia-smi unavailable"]


def test_pci_bus_id_in_nvidia_smi_form(monkeypatch):
    props = types.SimpleNamespace(pci_domain_id=0, pci_bus_id=0x1B, pci_device_id=0)
    monkeypatch.setattr(torch.cuda, "get_device_properties", lambda dev: props)
    assert bench.pci_bus_id(0) == "00000000:1B:00.0"


def _reference_arm(launcher=()):
    import json
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    cmd = [*launcher, os.path.join(root, "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "3",
           "--cpu-tokens", "256", "--cpu-seconds", "1"]
    if not launcher:
        cmd = [sys.executable, *cmd]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=240, cwd=root)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    return [json.loads(ln) for ln in lines]


def test_reference_arm_prints_one_line_with_the_contract_keys():
    (line,) = _reference_arm()
    assert line["impl"] == "reference" and line["unit"] == "tok/s" and line["value"] > 0
    assert line["warmup"] >= 3 and line["higher_is_better"] is True and line["n_gpus"] == 1
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["value"] == line["value"]
    assert line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"] == {"value": line["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert line["decode"]["value"] > 0 and line["config"]["workload"].startswith("configs[1]")


def test_reference_arm_under_torchrun_prints_from_rank_0_only():
    import os
    import sys

    launcher = (sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
                "--master-addr=127.0.0.1", f"--master-port={32700 + os.getpid() % 500}")
    lines = _reference_arm(launcher=launcher)
    assert len(lines) == 1 and lines[0]["n_gpus"] == 2
