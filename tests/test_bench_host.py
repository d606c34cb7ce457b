"""bench.py's host-side measurement helpers, without a GPU: the clocks summary that goes into the
bench line (median SM clock under load, the maximum, the throttle reasons seen while the timed
region ran) and the PCI bus id that selects the GPU for nvidia-smi."""
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
