"""NUMA placement of the pinned host pool (``pager_hf.host_pool``): sysfs lookup and thread affinity."""

import os
import types

import pytest
import torch

from pager_hf import host_pool as hp


def test_cpulist_parsing():
    assert hp.parse_cpulist("0-3,8,10-11\n") == {0, 1, 2, 3, 8, 10, 11}
    assert hp.parse_cpulist("5") == {5}
    assert hp.parse_cpulist("") == set()


def _fake_sysfs(tmp_path, bdf, node, cpulist):
    dev = tmp_path / "bus" / "pci" / "devices" / bdf
    dev.mkdir(parents=True)
    (dev / "numa_node").write_text(f"{node}\n")
    if node >= 0:
        nd = tmp_path / "devices" / "system" / "node" / f"node{node}"
        nd.mkdir(parents=True)
        (nd / "cpulist").write_text(cpulist + "\n")


def test_device_node_cpus_from_sysfs(tmp_path, monkeypatch):
    props = types.SimpleNamespace(pci_domain_id=0, pci_bus_id=0x9C, pci_device_id=0)
    monkeypatch.setattr(torch.cuda, "get_device_properties", lambda i: props)
    _fake_sysfs(tmp_path, "0000:9c:00.0", 1, "16-31,48-63")
    assert hp.device_numa_cpus(0, sysfs=str(tmp_path)) == set(range(16, 32)) | set(range(48, 64))


def test_unknown_node_places_nothing(tmp_path, monkeypatch):
    props = types.SimpleNamespace(pci_domain_id=0, pci_bus_id=0x9C, pci_device_id=0)
    monkeypatch.setattr(torch.cuda, "get_device_properties", lambda i: props)
    _fake_sysfs(tmp_path, "0000:9c:00.0", -1, "")
    assert hp.device_numa_cpus(0, sysfs=str(tmp_path)) is None
    assert hp.device_numa_cpus(0, sysfs=str(tmp_path / "missing")) is None


@pytest.mark.skipif(not hasattr(os, "sched_setaffinity") or len(os.sched_getaffinity(0)) < 2,
                    reason="needs two CPUs to restrict to one")
def test_affinity_is_restricted_inside_and_restored_after():
    before = os.sched_getaffinity(0)
    one = {min(before)}
    with hp.on_cpus(one):
        assert os.sched_getaffinity(0) == one
    assert os.sched_getaffinity(0) == before
    with hp.on_cpus({10 ** 6}):  # no usable CPU: affinity left alone
        assert os.sched_getaffinity(0) == before
    with pytest.raises(RuntimeError):
        with hp.on_cpus(one):
            raise RuntimeError("allocation failed")
    assert os.sched_getaffinity(0) == before
