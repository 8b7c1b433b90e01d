"""bench.bind_host_cpus against a fake NVML (CPU only): the GPU's local CPU
mask is read by PCI bus id, intersected with the allowed CPUs and applied to
the process; without NVML the rank runs unbound."""
import os
import sys
import types

import bench


class _Props:
    pci_domain_id = 0
    pci_bus_id = 0x1B
    pci_device_id = 0


class _Cuda:
    @staticmethod
    def get_device_properties(i):
        return _Props()


class _Torch:
    cuda = _Cuda()


def _fake_nvml(masks, seen):
    m = types.ModuleType("pynvml")
    m.nvmlInit = lambda: seen.append("init")
    m.nvmlShutdown = lambda: seen.append("shutdown")

    def by_bus(bus):
        seen.append(bus)
        return "handle"

    def affinity(h, n):
        seen.append(("affinity", h, n))
        return masks

    m.nvmlDeviceGetHandleByPciBusId = by_bus
    m.nvmlDeviceGetCpuAffinity = affinity
    return m


def test_binds_to_the_gpu_local_cpus(monkeypatch):
    seen, applied = [], []
    allowed = set(range(8))
    monkeypatch.setitem(sys.modules, "pynvml", _fake_nvml([0b1111_0000 | (1 << 40)], seen))
    monkeypatch.setattr(os, "sched_getaffinity", lambda pid: allowed)
    monkeypatch.setattr(os, "sched_setaffinity", lambda pid, cpus: applied.append(set(cpus)))
    r = bench.bind_host_cpus(_Torch(), 0)
    assert r["bound"] and r["cpus"] == 4 and r["pci"] == "00000000:1b:00.0"
    assert applied == [{4, 5, 6, 7}]  # CPU 40 is local but not allowed
    assert seen[0] == "init" and seen[-1] == "shutdown"


def test_unbound_without_nvml_or_when_disabled(monkeypatch):
    applied = []
    monkeypatch.setattr(os, "sched_setaffinity", lambda pid, cpus: applied.append(cpus))
    broken = types.ModuleType("pynvml")

    def fail():
        raise RuntimeError("NVML unavailable")

    broken.nvmlInit = fail
    monkeypatch.setitem(sys.modules, "pynvml", broken)
    r = bench.bind_host_cpus(_Torch(), 0)
    assert not r["bound"] and "NVML unavailable" in r["why"]
    assert bench.bind_host_cpus(_Torch(), 0, enabled=False) == {"bound": False, "why": "--no-bind"}
    assert applied == []
