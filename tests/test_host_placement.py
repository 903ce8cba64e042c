"""Host-buffer placement helper (no GPU needed): the GPU's local CPU list is
read from its PCI device's sysfs entry, intersected with the cores this
process may use, and the process affinity is restored after the block."""

from __future__ import annotations

import os
from types import SimpleNamespace

import torch

from aws_training_study_b200.pcp_attention import host


def _fake_props(monkeypatch):
    props = SimpleNamespace(pci_domain_id=0, pci_bus_id=0x1B, pci_device_id=0)
    monkeypatch.setattr(torch.cuda, "get_device_properties", lambda device: props)
    return "0000:1b:00.0"


def test_parse_cpulist():
    assert host._parse_cpulist("0-3,8,10-11\n") == {0, 1, 2, 3, 8, 10, 11}
    assert host._parse_cpulist("5") == {5}
    assert host._parse_cpulist("") == set()


def test_device_local_cpus_reads_sysfs(tmp_path, monkeypatch):
    bus = _fake_props(monkeypatch)
    allowed = sorted(os.sched_getaffinity(0))
    (tmp_path / bus).mkdir()
    (tmp_path / bus / "local_cpulist").write_text(f"{allowed[0]},{max(allowed) + 1000}\n")
    # only the allowed cores of the list
    assert host.device_local_cpus(0, sysfs=tmp_path) == {allowed[0]}
    # no entry: no placement information
    assert host.device_local_cpus(0, sysfs=tmp_path / "missing") is None


def test_near_device_restores_affinity(tmp_path, monkeypatch):
    bus = _fake_props(monkeypatch)
    before = os.sched_getaffinity(0)
    first = min(before)
    monkeypatch.setattr(host, "device_local_cpus", lambda device: {first})
    with host.near_device(0) as n:
        if len(before) > 1:
            assert n == 1 and os.sched_getaffinity(0) == {first}
        else:
            assert n is None
    assert os.sched_getaffinity(0) == before
    with host.near_device(0, enable=False) as n:
        assert n is None and os.sched_getaffinity(0) == before
    del bus
