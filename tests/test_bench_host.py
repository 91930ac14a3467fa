"""Host-side helpers of bench.py that need no GPU: the cpulist parser and
NUMA binding used by the multi-rank e2e leg, and the clock summary of the
timed region."""
import os
import types

import bench


def test_parse_cpulist():
    assert bench.parse_cpulist("0-3,8,10-11") == {0, 1, 2, 3, 8, 10, 11}
    assert bench.parse_cpulist("5") == {5}
    assert bench.parse_cpulist("0-31\n") == set(range(32))


def _fake_torch(dom=0, bus=0x1B, dev=0):
    props = types.SimpleNamespace(pci_domain_id=dom, pci_bus_id=bus, pci_device_id=dev)
    return types.SimpleNamespace(cuda=types.SimpleNamespace(get_device_properties=lambda i: props))


def test_bind_near_gpu_no_change_when_gpu_is_local_to_every_cpu(tmp_path):
    here = sorted(os.sched_getaffinity(0))
    d = tmp_path / "0000:1b:00.0"
    d.mkdir()
    (d / "local_cpulist").write_text(",".join(str(c) for c in here) + "\n")
    before = os.sched_getaffinity(0)
    assert bench.bind_near_gpu(_fake_torch(), 0, sysfs=str(tmp_path)) is None
    assert os.sched_getaffinity(0) == before


def test_bind_near_gpu_without_topology(tmp_path):
    before = os.sched_getaffinity(0)
    assert bench.bind_near_gpu(_fake_torch(), 0, sysfs=str(tmp_path)) is None  # no such device
    assert bench.bind_near_gpu(types.SimpleNamespace(cuda=None), 0) is None     # no properties
    assert os.sched_getaffinity(0) == before


def test_bind_near_gpu_narrows_to_the_local_cpus(tmp_path):
    here = sorted(os.sched_getaffinity(0))
    if len(here) < 2:
        return
    d = tmp_path / "0000:40:00.0"
    d.mkdir()
    (d / "local_cpulist").write_text(f"{here[0]}\n")
    before = os.sched_getaffinity(0)
    try:
        assert bench.bind_near_gpu(_fake_torch(bus=0x40), 0, sysfs=str(tmp_path)) == str(here[0])
        assert os.sched_getaffinity(0) == {here[0]}
    finally:
        os.sched_setaffinity(0, before)


def test_clock_summary_from_nvml_samples():
    c = bench.ClockSampler(0)
    c.source = "nvml, every 2 ms"
    c.max_mhz = 1965.0
    c.samples = [(1965.0, 0), (1920.0, 0x4), (1965.0, 0x4 | 0x1)]
    s = c.summary()
    assert s["sm_mhz"] == 1965.0 and s["sm_max_mhz"] == 1965.0 and s["samples"] == 3
    assert s["reasons"] == ["sw_power_cap"]  # the idle bit (0x1) is not a throttle reason
    c.samples = [(1500.0, 0x40)]
    assert c.summary()["reasons"] == ["hw_thermal_slowdown"]


def test_clock_summary_from_nvidia_smi_lines():
    c = bench.ClockSampler(0)
    c.source = "nvidia-smi, every 100 ms"
    c.out = ("0, 1965, 1965, 700.1, 0x4, Not Active, Not Active, Not Active, Active\n"
             "0, 1950, 1965, 900.0, 0x0, Not Active, Not Active, Not Active, Not Active\n")
    s = c.summary()
    assert s["samples"] == 2 and s["sm_max_mhz"] == 1965.0 and s["reasons"] == ["sw_power_cap"]


def test_clock_summary_without_samples():
    c = bench.ClockSampler(0)
    assert c.summary()["samples"] == 0


def test_pci_address():
    assert bench.pci_address(_fake_torch(dom=0, bus=0x1B, dev=0), 0) == "0000:1b:00.0"
    assert bench.pci_address(types.SimpleNamespace(cuda=None), 0) is None
