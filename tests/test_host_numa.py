"""CPU tests of the NUMA helpers of the host pipeline, against a fake NVML."""

import os
import sys
import types

import torch

from moe_dispatch import host_pipeline


class _Props:
    pci_domain_id, pci_bus_id, pci_device_id = 0, 0x18, 0


def _fake_nvml(mask_words, seen):
    fake = types.ModuleType("pynvml")
    fake.nvmlInit = lambda: seen.append("init")
    fake.nvmlShutdown = lambda: seen.append("shutdown")

    def by_bus(bus_id):
        seen.append(bus_id)
        return "handle"

    fake.nvmlDeviceGetHandleByPciBusId = by_bus
    fake.nvmlDeviceGetCpuAffinity = lambda handle, words: mask_words[:words]
    return fake


def test_device_local_cpus_decodes_nvml_masks(monkeypatch):
    seen = []
    # CPUs 0-3 in the first word and CPU 65 in the second
    monkeypatch.setitem(sys.modules, "pynvml", _fake_nvml([0b1111, 0b10], seen))
    monkeypatch.setattr(torch.cuda, "get_device_properties", lambda device: _Props())
    monkeypatch.setattr(os, "cpu_count", lambda: 128)
    assert host_pipeline.device_local_cpus("cuda:3") == {0, 1, 2, 3, 65}
    assert seen == ["init", "00000000:18:00.0", "shutdown"]


def test_device_local_cpus_is_none_without_nvml(monkeypatch):
    broken = types.ModuleType("pynvml")

    def fail():
        raise RuntimeError("no driver")

    broken.nvmlInit = fail
    monkeypatch.setitem(sys.modules, "pynvml", broken)
    monkeypatch.setattr(torch.cuda, "get_device_properties", lambda device: _Props())
    assert host_pipeline.device_local_cpus("cuda:0") is None


def test_pinned_on_device_node_restores_the_affinity(monkeypatch):
    calls = []
    monkeypatch.setattr(host_pipeline, "device_local_cpus", lambda device: {0})
    monkeypatch.setattr(os, "sched_getaffinity", lambda pid: {0, 1, 2})
    monkeypatch.setattr(os, "sched_setaffinity", lambda pid, cpus: calls.append(set(cpus)))
    monkeypatch.setattr(torch.Tensor, "pin_memory", lambda self: self.clone())
    out = host_pipeline.pinned_on_device_node([torch.ones(3), torch.zeros(2)], "cuda:0")
    assert [t.tolist() for t in out] == [[1.0, 1.0, 1.0], [0.0, 0.0]]
    assert calls == [{0}, {0, 1, 2}]  # bound to the GPU's CPUs, then restored
