"""Pinned, device-mapped host memory for the host tier of the KV pools.

Allocated by the C ABI (``pager_host_pool_alloc``: cudaHostAlloc with the
Portable and Mapped flags), so kernels on any device read it zero-copy
through the same address, and wrapped as a CPU torch tensor for host-side
copies.  The reference keeps CPU blocks as pageable tensors in a dict
(pager_hf/kv_block_store.py:45-46, :120-121); pinned mapped memory is what
lets the decode kernel read them without a per-step gather.
"""

from __future__ import annotations

import contextlib
import ctypes
import math
import os

import torch

from . import _lib as L

SYSFS = "/sys"


def parse_cpulist(text: str) -> set[int]:
    """CPUs of a sysfs cpulist such as ``"0-3,8,10-11"``."""
    cpus: set[int] = set()
    for part in text.strip().split(","):
        if not part:
            continue
        lo, _, hi = part.partition("-")
        cpus.update(range(int(lo), int(hi or lo) + 1))
    return cpus


def device_numa_cpus(device_index: int, sysfs: str | None = None) -> set[int] | None:
    """The host CPUs of the NUMA node a GPU's PCIe link attaches to, from sysfs; None when the system
    does not say (no such entry, or node -1 as virtual machines often report)."""
    sysfs = SYSFS if sysfs is None else sysfs
    try:
        p = torch.cuda.get_device_properties(device_index)
        bdf = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        with open(os.path.join(sysfs, "bus", "pci", "devices", bdf, "numa_node")) as f:
            node = int(f.read().strip())
        if node < 0:
            return None
        with open(os.path.join(sysfs, "devices", "system", "node", f"node{node}", "cpulist")) as f:
            return parse_cpulist(f.read())
    except (OSError, ValueError, RuntimeError, AssertionError):
        return None


def device_numa_node(device_index: int, sysfs: str | None = None) -> int | None:
    """The NUMA node of a GPU's PCIe link from sysfs, or None when the system does not say."""
    sysfs = SYSFS if sysfs is None else sysfs
    try:
        p = torch.cuda.get_device_properties(device_index)
        bdf = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        with open(os.path.join(sysfs, "bus", "pci", "devices", bdf, "numa_node")) as f:
            node = int(f.read().strip())
        return node if node >= 0 else None
    except (OSError, ValueError, RuntimeError, AssertionError):
        return None


def numa_pages(ptr: int, nbytes: int, proc: str = "/proc/self") -> dict[int, int]:
    """Resident pages per NUMA node of the memory mappings overlapping ``[ptr, ptr + nbytes)``, from
    the process's ``maps`` (address ranges) and ``numa_maps`` (``N<node>=<pages>`` per mapping);
    {} when the kernel does not report them."""
    try:
        with open(os.path.join(proc, "maps")) as f:
            ranges = []
            for line in f:
                lo, _, hi = line.split(" ", 1)[0].partition("-")
                ranges.append((int(lo, 16), int(hi, 16)))
        with open(os.path.join(proc, "numa_maps")) as f:
            nodes_at = {}
            for line in f:
                parts = line.split()
                if not parts:
                    continue
                counts = {}
                for field in parts[2:]:
                    if field.startswith("N") and "=" in field:
                        node, _, pages = field[1:].partition("=")
                        if node.isdigit():
                            counts[int(node)] = int(pages)
                nodes_at[int(parts[0], 16)] = counts
    except (OSError, ValueError):
        return {}
    out: dict[int, int] = {}
    for lo, hi in ranges:
        if hi > ptr and lo < ptr + nbytes:
            for node, pages in nodes_at.get(lo, {}).items():
                out[node] = out.get(node, 0) + pages
    return out


@contextlib.contextmanager
def on_cpus(cpus: set[int] | None):
    """Run the block with the calling thread restricted to ``cpus`` (those it may use at all), then
    restore its affinity.  Memory the block first touches lands on those CPUs' NUMA node under the
    default local-allocation policy."""
    old = None
    if cpus and hasattr(os, "sched_setaffinity"):
        allowed = os.sched_getaffinity(0)
        use = cpus & allowed
        if use and use != allowed:
            old = allowed
            os.sched_setaffinity(0, use)
    try:
        yield
    finally:
        if old is not None:
            os.sched_setaffinity(0, old)


class HostPool:
    """One pinned allocation viewed as a torch tensor of ``shape`` and ``dtype``.

    The pages are allocated on the NUMA node of the current CUDA device's PCIe link (the allocating
    thread runs on that node's CPUs meanwhile), so that on a multi-socket box each GPU reads its
    host tier from its own socket's memory; a single-node machine is unaffected."""

    def __init__(self, shape, dtype: torch.dtype):
        self.shape = tuple(int(s) for s in shape)
        self.dtype = dtype
        self.nbytes = math.prod(self.shape) * torch.tensor([], dtype=dtype).element_size()
        ptr = ctypes.c_void_p()
        cpus = device_numa_cpus(torch.cuda.current_device()) if self.nbytes and torch.cuda.is_available() else None
        with on_cpus(cpus):
            L.check(L.lib().pager_host_pool_alloc(self.nbytes, ctypes.byref(ptr)))
        self._ptr = ptr.value
        with torch.inference_mode(False):  # an ordinary tensor, updatable in and out of inference mode
            if self.nbytes:
                raw = (ctypes.c_uint8 * self.nbytes).from_address(self._ptr)
                self.tensor = torch.frombuffer(raw, dtype=torch.uint8).view(dtype).view(self.shape)
            else:
                self.tensor = torch.empty(self.shape, dtype=dtype)
        self._raw_ref = self.tensor

    @property
    def data_ptr(self) -> int:
        return self._ptr or 0

    def close(self) -> None:
        if self._ptr:
            self.tensor = None
            self._raw_ref = None
            L.check(L.lib().pager_host_pool_free(self._ptr))
            self._ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
