"""Pinned, device-mapped host memory for the host tier of the KV pools.

Allocated by the C ABI (``pager_host_pool_alloc``: cudaHostAlloc with the
Portable and Mapped flags), so kernels on any device read it zero-copy
through the same address, and wrapped as a CPU torch tensor for host-side
copies.  The reference keeps CPU blocks as pageable tensors in a dict
(pager_hf/kv_block_store.py:45-46, :120-121); pinned mapped memory is what
lets the decode kernel read them without a per-step gather.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _lib as L


class HostPool:
    """One pinned allocation viewed as a torch tensor of ``shape`` and ``dtype``."""

    def __init__(self, shape, dtype: torch.dtype):
        self.shape = tuple(int(s) for s in shape)
        self.dtype = dtype
        self.nbytes = math.prod(self.shape) * torch.tensor([], dtype=dtype).element_size()
        ptr = ctypes.c_void_p()
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
