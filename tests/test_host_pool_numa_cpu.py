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


def test_numa_pages_sums_the_mappings_over_a_range(tmp_path):
    from pager_hf.host_pool import numa_pages

    (tmp_path / "maps").write_text(
        "7f0000000000-7f0000200000 rw-s 00000000 00:05 1 /dev/nvidia0\n"
        "7f0000200000-7f0000400000 rw-s 00000000 00:05 1 /dev/nvidia0\n"
        "7f1000000000-7f1000001000 r--p 00000000 00:05 2 /lib/x.so\n")
    (tmp_path / "numa_maps").write_text(
        "7f0000000000 default file=/dev/nvidia0 dirty=512 N0=300 N1=212 kernelpagesize_kB=4\n"
        "7f0000200000 default file=/dev/nvidia0 dirty=512 N1=512 kernelpagesize_kB=4\n"
        "7f1000000000 default file=/lib/x.so mapped=1 N0=1 kernelpagesize_kB=4\n")
    assert numa_pages(0x7F0000000000, 0x400000, str(tmp_path)) == {0: 300, 1: 724}
    assert numa_pages(0x7F0000300000, 0x1000, str(tmp_path)) == {1: 512}
    assert numa_pages(0x7F0000000000, 16, str(tmp_path / "missing")) == {}
