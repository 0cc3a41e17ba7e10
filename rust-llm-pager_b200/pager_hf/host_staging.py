"""Staged reads of the host tier: copy engines move host blocks, the kernel reads HBM.

Host-pool blocks can reach the decode kernel two ways:

* zero-copy: the kernel's consumer warps load them straight from mapped pinned
  memory (``PAGER_HOST_SLOT_BIT`` entries);
* staged: before layer ``l``'s kernel, each host block's layer-``l`` chunk
  (``[2, kv_heads, tokens_per_block, head_dim]``, contiguous in the slot) is
  copied by the DMA engines into a device staging buffer; the block table names
  the staged copy (``PAGER_STAGE_SLOT_BIT``) and the kernel reads it with TMA.
  Copies for layer ``l+1`` run on a copy stream while layer ``l`` computes, into
  the other half of a double buffer.

Which one wins depends on the link and on how the host blocks lie in the pool:
``choose_host_read`` measures both reads on this device (pinned
``cudaMemcpyAsync`` against a zero-copy read kernel, 256 MiB) and picks staged
reads when copying a layer's blocks, one submission per run of consecutive
slots, is expected to beat reading them zero-copy.  The reference reads
host blocks with synchronous pageable copies per layer and group
(``pager_hf/paged_model.py:878-924``).
"""

from __future__ import annotations

import ctypes
import threading

import numpy as np
import torch

from . import _lib as L

HOST_SLOT_BIT = L.HOST_SLOT_BIT
STAGE_SLOT_BIT = L.STAGE_SLOT_BIT

_LINK: dict[int, dict] = {}
_LINK_LOCK = threading.Lock()


def plan_host_runs(block_table: torch.Tensor, tokens_per_block: int | None = None, num_blocks=None,
                   valid_lo=None, valid_hi=None, active=None):
    """Staging plan for a block table (int32 ``[batch, blocks]``).

    Only host blocks the kernel will read are staged: inside the row's
    ``num_blocks``, overlapping its ``[valid_lo, valid_hi)`` token range, in an
    active row (a sliding window or left padding leaves most of a long row's
    blocks unread).  Other host entries keep their host tag and stay readable
    zero-copy, so the plan never changes what the kernel computes.

    Returns ``(staged_table, host_slots, runs)``: the table with each staged
    entry replaced by ``stage_index | STAGE_SLOT_BIT``, the distinct staged host
    slots in staging order (ascending), and ``runs`` = int32 arrays
    ``(src, dst, len)`` of maximal runs of consecutive host slots (one 2D copy
    each)."""
    t = block_table.to("cpu", torch.int32)
    nb = t.shape[1]
    need = (t >= 0) & ((t & HOST_SLOT_BIT) != 0)
    cols = torch.arange(nb, dtype=torch.int64)[None, :]
    if num_blocks is not None:
        need &= cols < num_blocks.to("cpu", torch.int64)[:, None]
    if tokens_per_block is not None and valid_lo is not None:
        need &= (cols + 1) * tokens_per_block > valid_lo.to("cpu", torch.int64)[:, None]
    if tokens_per_block is not None and valid_hi is not None:
        need &= cols * tokens_per_block < valid_hi.to("cpu", torch.int64)[:, None]
    if active is not None:
        need &= active.to("cpu", torch.int64)[:, None] != 0
    slots = torch.unique(t[need] & (HOST_SLOT_BIT - 1)).to(torch.int64)  # sorted ascending
    staged = t.clone()
    if slots.numel():
        idx = torch.searchsorted(slots, (t[need] & (HOST_SLOT_BIT - 1)).to(torch.int64)).to(torch.int32)
        staged[need] = idx | STAGE_SLOT_BIT
    s = slots.numpy()
    if s.size:
        breaks = np.nonzero(np.diff(s) != 1)[0] + 1
        starts = np.concatenate(([0], breaks))
        ends = np.concatenate((breaks, [s.size]))
        runs = (s[starts].astype(np.int32), starts.astype(np.int32), (ends - starts).astype(np.int32))
    else:
        runs = (np.zeros(0, np.int32),) * 3
    return staged, slots, runs


def link_bandwidth(device) -> dict:
    """Measured host->device bandwidth of this device (GB/s): pinned copy and zero-copy read."""
    device = torch.device(device)
    idx = device.index if device.index is not None else torch.cuda.current_device()
    with _LINK_LOCK:
        if idx in _LINK:
            return _LINK[idx]
        from .host_pool import HostPool

        nbytes = 256 << 20
        with torch.cuda.device(idx):
            src = HostPool((nbytes,), torch.uint8)
            dst = torch.empty(nbytes, dtype=torch.uint8, device=f"cuda:{idx}")
            stream = torch.cuda.current_stream(idx).cuda_stream
            c, z = ctypes.c_double(), ctypes.c_double()
            lib = L.lib()
            L.check(lib.pager_probe_h2d_copy_gbs(src.data_ptr, dst.data_ptr(), nbytes, 3, stream, ctypes.byref(c)))
            L.check(lib.pager_probe_zero_copy_gbs(src.data_ptr, dst.data_ptr(), nbytes, 3, stream, ctypes.byref(z)))
            src.close()
            del dst
        _LINK[idx] = {"copy_gbs": c.value, "zero_copy_gbs": z.value}
        return _LINK[idx]


def record_link_bandwidth(device, copy_gbs: float, zero_copy_gbs: float) -> None:
    """Use an outside measurement of this device's link (e.g. taken with every GPU of the box copying
    at once) for later ``auto`` choices instead of probing it alone."""
    device = torch.device(device)
    idx = device.index if device.index is not None else torch.cuda.current_device()
    with _LINK_LOCK:
        _LINK[idx] = {"copy_gbs": float(copy_gbs), "zero_copy_gbs": float(zero_copy_gbs)}


# Host time to submit one 2D copy of a run (cudaMemcpy2DAsync), measured on B200 boxes: a
# left-padded 16-row batch whose host slots fell into ~570 runs per layer issued 99,616 copies
# in 8 decode steps for 774 ms of host time (~7.8 us each, command-buffer stalls included).
COPY_SUBMIT_S = 10e-6


def choose_host_read(device, bytes_per_layer: int | None = None, copies_per_layer: int = 1) -> str:
    """``"staged"`` when copying a layer's host blocks is expected to take less time than reading them
    zero-copy, else ``"zero_copy"``.  The copies of a layer are submitted while earlier work runs, so
    staged time = the longer of the copy engines' time (bytes / copy bandwidth) and the host's
    submissions (one per copy, ``COPY_SUBMIT_S``): a host tier scattered over many short runs of
    slots is submission-bound.  Without sizes, compares the two links."""
    bw = link_bandwidth(device)
    if bytes_per_layer is None:
        return "staged" if bw["copy_gbs"] > bw["zero_copy_gbs"] else "zero_copy"
    t_staged = max(bytes_per_layer / (bw["copy_gbs"] * 1e9), copies_per_layer * COPY_SUBMIT_S)
    t_zero_copy = bytes_per_layer / (bw["zero_copy_gbs"] * 1e9)
    return "staged" if t_staged < t_zero_copy else "zero_copy"


class HostStaging:
    """Double-buffered per-layer staging of a block table's host blocks.

    ``before_kernel(layer, stream)`` makes sure the layer's copies are issued
    (on the copy stream, after the kernel that last read that half of the
    buffer), issues the next layer's copies so they overlap this layer's
    kernel, and makes ``stream`` wait for this layer's copies;
    ``after_kernel(layer, stream)`` marks the buffer half as read.  With
    ``prefetch_next_step`` the last layer also prefetches layer 0 for the next
    ``run`` of the same plan (host blocks do not change while they are named by
    an unchanged table).
    """

    def __init__(self, block_table: torch.Tensor, host_pool: torch.Tensor, num_layers: int, device,
                 prefetch_next_step: bool = False, tokens_per_block: int | None = None, num_blocks=None,
                 valid_lo=None, valid_hi=None, active=None, plan=None):
        staged, slots, runs = plan if plan is not None else plan_host_runs(
            block_table, tokens_per_block, num_blocks, valid_lo, valid_hi, active)
        self.device = torch.device(device)
        self.table = staged.to(self.device)
        self.num_slots = int(slots.numel())
        self.runs = tuple(np.ascontiguousarray(r) for r in runs)
        self.num_layers = int(num_layers)
        _, L_, two, hkv, tpb, d = host_pool.shape
        if L_ != num_layers or two != 2:
            raise ValueError("host pool must be [slots, layers, 2, kv_heads, tokens_per_block, head_dim]")
        self.host_pool = host_pool
        elt = host_pool.element_size()
        self.chunk_bytes = 2 * hkv * tpb * d * elt
        self.slot_bytes = num_layers * self.chunk_bytes
        shape = (max(self.num_slots, 1), 2, hkv, tpb, d)
        self.buffers = [torch.empty(shape, dtype=host_pool.dtype, device=self.device) for _ in range(2)]
        self.copy_stream = torch.cuda.Stream(device=self.device)
        # copies start after everything already queued on the caller's stream (e.g. tier moves)
        self.copy_stream.wait_stream(torch.cuda.current_stream(self.device))
        self.copy_done = [torch.cuda.Event(), torch.cuda.Event()]
        self.read_done = [torch.cuda.Event(), torch.cuda.Event()]
        self.content = [None, None]  # (layer, generation) staged in each half
        self.generation = 0
        self.prefetch_next_step = prefetch_next_step
        self.bytes_per_layer = self.num_slots * self.chunk_bytes
        self._runs_ptr = tuple(r.ctypes.data for r in self.runs)
        self._lib = L.lib()

    def _issue(self, layer: int, generation: int) -> None:
        buf = layer % 2
        if self.content[buf] == (layer, generation):
            return
        s = self.copy_stream
        s.wait_event(self.read_done[buf])  # the kernel that last read this half has finished
        L.check(self._lib.pager_stage_host_blocks(
            self.buffers[buf].data_ptr(), self.host_pool.data_ptr(), self.slot_bytes, layer * self.chunk_bytes,
            self.chunk_bytes, self._runs_ptr[0], self._runs_ptr[1], self._runs_ptr[2], len(self.runs[0]),
            s.cuda_stream))
        self.copy_done[buf].record(s)
        self.content[buf] = (layer, generation)

    def _next(self, layer: int):
        """The (layer, generation) to prefetch after ``layer``, or None."""
        if layer + 1 < self.num_layers:
            return layer + 1, self.generation
        if self.prefetch_next_step:
            return 0, self.generation + 1
        return None

    def before_kernel(self, layer: int, stream: torch.cuda.Stream) -> torch.Tensor:
        if layer == 0:
            self.generation += 1
        self._issue(layer, self.generation)
        nxt = self._next(layer)
        if nxt is not None and nxt[0] % 2 != layer % 2:  # the other half: overlaps this kernel
            self._issue(*nxt)
        stream.wait_event(self.copy_done[layer % 2])
        return self.buffers[layer % 2]

    def after_kernel(self, layer: int, stream: torch.cuda.Stream) -> None:
        self.read_done[layer % 2].record(stream)
        nxt = self._next(layer)
        if nxt is not None and nxt[0] % 2 == layer % 2:  # same half: only after this kernel has read it
            self._issue(*nxt)

    def synchronize(self) -> None:
        self.copy_stream.synchronize()

    def invalidate(self) -> None:
        """Wait for pending copies and forget what the buffer halves hold: the next ``run`` of each
        layer copies it again (e.g. before a timed region, so that no copy done earlier counts)."""
        self.copy_stream.synchronize()
        self.content = [None, None]
