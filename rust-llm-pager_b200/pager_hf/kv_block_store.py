"""KV block store over a device pool and a pinned host pool.

Same API as the reference's ``pager_hf/kv_block_store.py:36-274``
(``KVBlockStore``: ``put_gpu``, ``offload_to_cpu``, ``load_to_gpu``,
``ensure_gpu/cpu``, ``apply_tiers``, ``reorder_batch_rows``, ``get_gpu``,
``get_any``, ``summary``, resident-byte accounting, the RAM budget with its
80 % warning and ``RuntimeError``), with the block storage the decode kernel
reads directly:

* a block of ``B`` batch rows occupies ``B`` consecutive *slots* (a slot
  group) of a pool ``[slots, layers, 2 (K,V), kv_heads, tokens_per_block,
  head_dim]``: the device pool in HBM (torch-allocated) or the pinned,
  device-mapped host pool (``HostPool``);
* a tier move is one contiguous ``cudaMemcpyAsync`` of the group on a copy
  stream (pinned memory, so it runs at link speed and overlaps the compute
  stream), instead of per-tensor synchronous ``.to()`` copies from pageable
  memory (``kv_block_store.py:114-156``);
* ``block_table()`` turns the store's residency into the int32 block table of
  ``paged_decode_attention`` (slot, or slot | host bit), so no gather runs.

``key``/``value`` tensors handed in and out keep the reference's layout
``[layers, batch, block_len, kv_heads, head_dim]``; what ``get_gpu`` /
``get_any`` return are views into the pools (same values, not contiguous).

Differences, all deliberate:
* every block has the geometry and dtype of the first one, and at most
  ``tokens_per_block`` tokens (a shorter block is stored padded and counted at
  its real size; ``block_table`` refuses short blocks, the kernel reads whole
  blocks); the reference stores arbitrary tensors;
* moves are stream-ordered: with ``sync=True`` (the default, the reference's
  behaviour) calls return after the copies finish; ``apply_tiers(...,
  sync=False)`` only orders the current stream after them;
* the pools grow by doubling when full (device groups are copied on the GPU,
  host groups into a new pinned pool), which changes their base pointers:
  ``version`` increments, and a ``PagedDecodePlan`` built before must be
  rebuilt.
"""

from __future__ import annotations

import logging
from collections.abc import Mapping
from dataclasses import dataclass

import numpy as np
import torch

from ._lib import HOST_SLOT_BIT
from .host_pool import HostPool

logger = logging.getLogger(__name__)

# kv_block_store.py:10-13: warn once CPU-resident bytes pass this fraction of ram_budget_bytes
_RAM_BUDGET_WARNING_THRESHOLD = 0.8


@dataclass
class KVBlockStoreStats:
    gpu_to_cpu_bytes: int = 0
    cpu_to_gpu_bytes: int = 0
    gpu_to_cpu_copies: int = 0
    cpu_to_gpu_copies: int = 0
    gpu_to_cpu_sec: float = 0.0
    cpu_to_gpu_sec: float = 0.0


def tensor_nbytes(tensor: torch.Tensor) -> int:
    """Return how many bytes a tensor occupies."""
    return tensor.numel() * tensor.element_size()


def kv_nbytes(key: torch.Tensor, value: torch.Tensor) -> int:
    """Return the combined byte size of a key/value tensor pair."""
    return tensor_nbytes(key) + tensor_nbytes(value)


class SlotGroups:
    """Free list of slot groups in one pool (group g = slots [g*batch, (g+1)*batch))."""

    def __init__(self, capacity: int = 0):
        self.capacity = 0
        self._free: list[int] = []
        self.grow(capacity)

    def grow(self, capacity: int) -> None:
        if capacity < self.capacity:
            raise ValueError("slot groups cannot shrink")
        # lowest group first: keep the free list sorted descending so pop() returns the lowest
        self._free = sorted(set(self._free) | set(range(self.capacity, capacity)), reverse=True)
        self.capacity = capacity

    def take(self) -> int | None:
        return self._free.pop() if self._free else None

    def give(self, group: int) -> None:
        if not 0 <= group < self.capacity or group in self._free:
            raise ValueError(f"slot group {group} is not in use")
        self._free.append(group)
        self._free.sort(reverse=True)

    @property
    def used(self) -> int:
        return self.capacity - len(self._free)


class _TierView(Mapping):
    """Read-only ``block_id -> (key, value)`` mapping of one tier, the reference's
    ``gpu_blocks`` / ``cpu_blocks`` dicts."""

    def __init__(self, store: "KVBlockStore", on_gpu: bool):
        self._s, self._gpu = store, on_gpu

    def _ids(self):
        return self._s._dev_group if self._gpu else self._s._host_group

    def __getitem__(self, block_id):
        ids = self._ids()
        if block_id not in ids:
            raise KeyError(block_id)
        return self._s._kv_view(block_id, self._gpu)

    def __iter__(self):
        return iter(list(self._ids()))

    def __len__(self):
        return len(self._ids())

    def __contains__(self, block_id):
        return block_id in self._ids()


class KVPools:
    """A device pool and a pinned host pool of KV slots, with their slot-group allocators.

    One store owns a private ``KVPools`` by default; decode sessions that are
    batched into one launch share one (``KVBlockStore(..., pools=shared)``), so
    that a single block table can name every session's blocks.  A slot group is
    ``rows_per_group`` consecutive slots (one per batch row of a block).
    Growing a pool (doubling) changes its base pointer and bumps ``version``.
    """

    def __init__(self, *, num_layers: int, kv_heads: int, head_dim: int, tokens_per_block: int,
                 dtype: torch.dtype, device, rows_per_group: int = 1, gpu_groups: int = 8, cpu_groups: int = 8):
        self.num_layers, self.kv_heads, self.head_dim = num_layers, kv_heads, head_dim
        self.tokens_per_block, self.dtype = tokens_per_block, dtype
        self.elt = torch.tensor([], dtype=dtype).element_size()
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("KVPools needs a CUDA device for its device pool.")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.rows_per_group = rows_per_group
        self.copy_stream = torch.cuda.Stream(device=self.device)
        self.version = 0
        self._alloc(max(1, gpu_groups), max(1, cpu_groups), rows_per_group)

    def slot_shape(self):
        return (self.num_layers, 2, self.kv_heads, self.tokens_per_block, self.head_dim)

    # Pool tensors are always created with inference mode off, so that code inside and outside
    # torch.inference_mode (generate() and a caller's own loop) can both update them in place.
    def _alloc(self, gpu_groups: int, cpu_groups: int, rows: int) -> None:
        with torch.inference_mode(False):
            self.dev_pool = torch.empty((gpu_groups * rows,) + self.slot_shape(), dtype=self.dtype,
                                        device=self.device)
            self.host_pool = HostPool((cpu_groups * rows,) + self.slot_shape(), self.dtype)
        self.dev_groups = SlotGroups(gpu_groups)
        self.host_groups = SlotGroups(cpu_groups)
        self.rows_per_group = rows
        self.version += 1

    def group_slots(self, group: int) -> slice:
        return slice(group * self.rows_per_group, (group + 1) * self.rows_per_group)

    def take_dev_group(self) -> int:
        g = self.dev_groups.take()
        if g is None:
            self.grow_dev(2 * self.dev_groups.capacity)
            g = self.dev_groups.take()
        return g

    def take_host_group(self) -> int:
        g = self.host_groups.take()
        if g is None:
            self.grow_host(2 * self.host_groups.capacity)
            g = self.host_groups.take()
        return g

    def grow_dev(self, groups: int) -> None:
        self.copy_stream.synchronize()
        with torch.inference_mode(False):
            new = torch.empty((groups * self.rows_per_group,) + self.slot_shape(), dtype=self.dtype,
                              device=self.device)
            new[: self.dev_pool.shape[0]].copy_(self.dev_pool)
        self.dev_pool = new
        self.dev_groups.grow(groups)
        self.version += 1

    def grow_host(self, groups: int) -> None:
        self.copy_stream.synchronize()
        with torch.inference_mode(False):
            new = HostPool((groups * self.rows_per_group,) + self.slot_shape(), self.dtype)
            new.tensor[: self.host_pool.shape[0]].copy_(self.host_pool.tensor)
        self.host_pool.close()
        self.host_pool = new
        self.host_groups.grow(groups)
        self.version += 1

    def close(self) -> None:
        self.copy_stream.synchronize()
        if self.host_pool is not None:
            self.host_pool.close()
            self.host_pool = None


class KVBlockStore:
    """Blocks of KV cache in a device pool and a pinned host pool, indexed by block id."""

    def __init__(self, tokens_per_block: int, ram_budget_bytes: int | None = None, *,
                 gpu_capacity_blocks: int = 8, cpu_capacity_blocks: int = 8, pools: KVPools | None = None):
        self.tokens_per_block = tokens_per_block
        self.ram_budget_bytes = ram_budget_bytes
        self._cap0 = (max(1, gpu_capacity_blocks), max(1, cpu_capacity_blocks))
        self.stats = KVBlockStoreStats()
        if pools is not None and pools.tokens_per_block != tokens_per_block:
            raise ValueError(f"shared pools hold {pools.tokens_per_block}-token blocks, not {tokens_per_block}")
        self.pools = pools
        self._owns_pools = pools is None
        self._dev_group: dict[int, int] = {}  # block id -> group in the device pool
        self._host_group: dict[int, int] = {}  # block id -> group in the host pool
        self._tokens: dict[int, int] = {}  # block id -> tokens stored (<= tokens_per_block)
        self._resident_gpu_bytes = 0
        self._resident_cpu_bytes = 0
        self._pending: list[tuple[str, torch.cuda.Event, torch.cuda.Event]] = []
        self.gpu_blocks = _TierView(self, True)
        self.cpu_blocks = _TierView(self, False)

    # ------------------------------------------------------------------ geometry and pools
    def _geo(self, name):
        return None if self.pools is None else getattr(self.pools, name)

    num_layers = property(lambda self: self._geo("num_layers"))
    kv_heads = property(lambda self: self._geo("kv_heads"))
    head_dim = property(lambda self: self._geo("head_dim"))
    dtype = property(lambda self: self._geo("dtype"))
    device = property(lambda self: self._geo("device"))
    batch = property(lambda self: self._geo("rows_per_group"))
    version = property(lambda self: 0 if self.pools is None else self.pools.version)
    dev_pool = property(lambda self: self._geo("dev_pool"))
    host_pool = property(lambda self: self._geo("host_pool"))

    def _block_bytes(self, tokens: int) -> int:
        p = self.pools
        return 2 * p.num_layers * p.rows_per_group * tokens * p.kv_heads * p.head_dim * p.elt

    def _check_block(self, key: torch.Tensor, value: torch.Tensor) -> int:
        if key.dim() != 5 or key.shape != value.shape:
            raise ValueError(f"expected key/value of shape [layers, batch, block_len, kv_heads, head_dim], got "
                             f"{tuple(key.shape)} and {tuple(value.shape)}")
        if key.dtype != value.dtype:
            raise ValueError("key and value must share a dtype")
        L, B, t, H, D = key.shape
        if self.pools is None:
            self.pools = KVPools(num_layers=L, kv_heads=H, head_dim=D, tokens_per_block=self.tokens_per_block,
                                 dtype=key.dtype, device=key.device, rows_per_group=B, gpu_groups=self._cap0[0],
                                 cpu_groups=self._cap0[1])
        if (L, B, H, D) != (self.num_layers, self.batch, self.kv_heads, self.head_dim) or key.dtype != self.dtype:
            raise ValueError(f"block geometry {(L, B, H, D)} {key.dtype} differs from the store's "
                             f"{(self.num_layers, self.batch, self.kv_heads, self.head_dim)} {self.dtype}")
        if key.device != self.device:
            raise ValueError(f"block on {key.device}, store on {self.device}")
        if not 0 < t <= self.tokens_per_block:
            raise ValueError(f"block of {t} tokens; this store holds blocks of 1..{self.tokens_per_block} tokens")
        return t

    def _group_slots(self, group: int) -> slice:
        return self.pools.group_slots(group)

    def _kv_view(self, block_id: int, on_gpu: bool):
        pool = self.dev_pool if on_gpu else self.host_pool.tensor
        g = (self._dev_group if on_gpu else self._host_group)[block_id]
        t = self._tokens[block_id]
        grp = pool[self._group_slots(g)]  # [B, L, 2, H, T, D]
        key = grp[:, :, 0, :, :t].permute(1, 0, 3, 2, 4)
        value = grp[:, :, 1, :, :t].permute(1, 0, 3, 2, 4)
        return key, value

    # ------------------------------------------------------------------ copy stream
    def _copy(self, dst: torch.Tensor, src: torch.Tensor, kind: str) -> None:
        s = self.pools.copy_stream
        s.wait_stream(torch.cuda.current_stream(self.device))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(s):
            e0.record(s)
            dst.copy_(src, non_blocking=True)
            e1.record(s)
        self._pending.append((kind, e0, e1))

    def _drain(self) -> None:
        """Wait for pending tier copies and add their device time to the stats."""
        if self.pools is None:
            return
        self.pools.copy_stream.synchronize()
        for kind, e0, e1 in self._pending:
            sec = e0.elapsed_time(e1) / 1000.0
            if kind == "d2h":
                self.stats.gpu_to_cpu_sec += sec
            else:
                self.stats.cpu_to_gpu_sec += sec
        self._pending.clear()

    def synchronize(self) -> None:
        """Block until every tier move issued so far has landed."""
        self._drain()

    def _order_after_copies(self) -> None:
        if self.pools is not None:
            torch.cuda.current_stream(self.device).wait_stream(self.pools.copy_stream)

    # ------------------------------------------------------------------ the reference API
    def put_gpu(self, block_id: int, key: torch.Tensor, value: torch.Tensor) -> None:
        """Register a block that already lives on the GPU (copied into a device slot group).

        Registering an id that is already on the GPU replaces that block (the
        reference replaces it too but counts its bytes twice)."""
        if not key.is_cuda or not value.is_cuda:
            raise ValueError("put_gpu expects CUDA tensors.")
        if block_id in self._host_group:
            raise ValueError(f"Block {block_id} already exists on CPU.")
        t = self._check_block(key, value)
        if block_id in self._dev_group:  # re-registering replaces the block in place
            self._resident_gpu_bytes -= self._block_bytes(self._tokens[block_id])
            g = self._dev_group[block_id]
        else:
            g = self.pools.take_dev_group()
        dst = self.dev_pool[self._group_slots(g)]
        dst[:, :, 0, :, :t].copy_(key.detach().permute(1, 0, 3, 2, 4))
        dst[:, :, 1, :, :t].copy_(value.detach().permute(1, 0, 3, 2, 4))
        self._dev_group[block_id] = g
        self._tokens[block_id] = t
        self._resident_gpu_bytes += kv_nbytes(key, value)

    def put_gpu_layers(self, block_id: int, keys, values) -> None:
        """Register a block from per-layer HF tensors ``[batch, kv_heads, block_len, head_dim]``.

        The layout of a slot holds exactly those tensors, so each layer is one
        contiguous copy; no ``torch.stack`` of the layers (``kv_utils.py:37-53``).
        """
        if len(keys) != len(values) or not keys:
            raise ValueError("need one key and one value tensor per layer")
        k0 = keys[0]
        B, H, t, D = k0.shape
        probe = k0.new_empty((len(keys), B, t, H, D)) if self.pools is None else None
        if probe is not None:
            self._check_block(probe, probe)
        if (len(keys), B, H, D) != (self.num_layers, self.batch, self.kv_heads, self.head_dim):
            raise ValueError("layer tensors do not match the store's geometry")
        if block_id in self._host_group:
            raise ValueError(f"Block {block_id} already exists on CPU.")
        if not 0 < t <= self.tokens_per_block:
            raise ValueError(f"block of {t} tokens; this store holds blocks of 1..{self.tokens_per_block} tokens")
        if block_id in self._dev_group:
            self._resident_gpu_bytes -= self._block_bytes(self._tokens[block_id])
            g = self._dev_group[block_id]
        else:
            g = self.pools.take_dev_group()
        dst = self.dev_pool[self._group_slots(g)]
        for layer, (k, v) in enumerate(zip(keys, values)):
            if k.device != self.device or k.dtype != self.dtype or tuple(k.shape) != (B, H, t, D):
                raise ValueError(f"layer {layer}: tensor does not match the store")
            dst[:, layer, 0, :, :t].copy_(k)
            dst[:, layer, 1, :, :t].copy_(v)
        self._dev_group[block_id] = g
        self._tokens[block_id] = t
        self._resident_gpu_bytes += self._block_bytes(t)

    def adopt_gpu_group(self, block_id: int, group: int) -> None:
        """Register a full block that already sits in device slot group ``group`` of the pools
        (a decode session's tail slot once it holds ``tokens_per_block`` tokens): no copy."""
        if self.pools is None:
            raise ValueError("adopt_gpu_group needs pools")
        if block_id in self._dev_group or block_id in self._host_group:
            raise ValueError(f"Block {block_id} already exists.")
        self._dev_group[block_id] = group
        self._tokens[block_id] = self.tokens_per_block
        self._resident_gpu_bytes += self._block_bytes(self.tokens_per_block)

    def adopt_host_group(self, block_id: int, group: int) -> None:
        """Register a full block whose data the caller already wrote into host slot group ``group``."""
        if self.pools is None:
            raise ValueError("adopt_host_group needs pools")
        if block_id in self._dev_group or block_id in self._host_group:
            raise ValueError(f"Block {block_id} already exists.")
        incoming = self._block_bytes(self.tokens_per_block)
        if self.ram_budget_bytes is not None and self._resident_cpu_bytes + incoming > self.ram_budget_bytes:
            raise RuntimeError(f"ram_budget exceeded: block {block_id} would need "
                               f"{(self._resident_cpu_bytes + incoming) / 1_000_000:.2f} MB, budget is "
                               f"{self.ram_budget_bytes / 1_000_000:.2f} MB.")
        self._host_group[block_id] = group
        self._tokens[block_id] = self.tokens_per_block
        self._resident_cpu_bytes += incoming

    def has_gpu(self, block_id: int) -> bool:
        return block_id in self._dev_group

    def has_cpu(self, block_id: int) -> bool:
        return block_id in self._host_group

    def _offload(self, block_id: int) -> None:
        if block_id not in self._dev_group:
            raise KeyError(f"Block {block_id} is not on GPU.")
        incoming = self._block_bytes(self._tokens[block_id])
        if self.ram_budget_bytes is not None:
            projected = self._resident_cpu_bytes + incoming
            if projected > self.ram_budget_bytes:
                logger.error("ram_budget exceeded: block %d would need %.2f MB, budget is %.2f MB.", block_id,
                             projected / 1_000_000, self.ram_budget_bytes / 1_000_000)
                raise RuntimeError(
                    f"ram_budget exceeded: moving block {block_id} to CPU would need {projected / 1_000_000:.2f} MB, "
                    f"budget is {self.ram_budget_bytes / 1_000_000:.2f} MB. There is no SSD tier yet, so overflow "
                    "can't be absorbed further; use a shorter context, a larger ram_budget, or a bigger "
                    "tokens_per_block.")
            if projected > _RAM_BUDGET_WARNING_THRESHOLD * self.ram_budget_bytes:
                logger.warning("ram_budget usage at %.0f%% after offloading block %d (%.2f MB of %.2f MB budget).",
                               100.0 * projected / self.ram_budget_bytes, block_id, projected / 1_000_000,
                               self.ram_budget_bytes / 1_000_000)
        hg = self.pools.take_host_group()
        dg = self._dev_group.pop(block_id)
        self._copy(self.host_pool.tensor[self._group_slots(hg)], self.dev_pool[self._group_slots(dg)], "d2h")
        self.pools.dev_groups.give(dg)
        self._host_group[block_id] = hg
        self._resident_gpu_bytes -= incoming
        self._resident_cpu_bytes += incoming
        self.stats.gpu_to_cpu_bytes += incoming
        self.stats.gpu_to_cpu_copies += 1

    def _load(self, block_id: int, device) -> None:
        if block_id not in self._host_group:
            raise KeyError(f"Block {block_id} is not on CPU.")
        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("load_to_gpu expects a CUDA device.")
        index = device.index if device.index is not None else torch.cuda.current_device()
        if index != self.device.index:
            raise ValueError(f"this store's device pool is on {self.device}, not {device}")
        incoming = self._block_bytes(self._tokens[block_id])
        dg = self.pools.take_dev_group()
        hg = self._host_group.pop(block_id)
        self._copy(self.dev_pool[self._group_slots(dg)], self.host_pool.tensor[self._group_slots(hg)], "h2d")
        self.pools.host_groups.give(hg)
        self._dev_group[block_id] = dg
        self._resident_cpu_bytes -= incoming
        self._resident_gpu_bytes += incoming
        self.stats.cpu_to_gpu_bytes += incoming
        self.stats.cpu_to_gpu_copies += 1

    def offload_to_cpu(self, block_id: int) -> None:
        """Move a block from GPU to CPU and record how long the copy took."""
        self._offload(block_id)
        self._drain()

    def load_to_gpu(self, block_id: int, device: torch.device | str) -> None:
        """Move a block from CPU to GPU and record how long the copy took."""
        self._load(block_id, device)
        self._drain()

    def ensure_gpu(self, block_id: int, device: torch.device | str) -> None:
        if self.has_gpu(block_id):
            return
        self.load_to_gpu(block_id, device)

    def ensure_cpu(self, block_id: int) -> None:
        if self.has_cpu(block_id):
            return
        self.offload_to_cpu(block_id)

    def resident_gpu_bytes(self) -> int:
        return self._resident_gpu_bytes

    def resident_cpu_bytes(self) -> int:
        return self._resident_cpu_bytes

    def gpu_block_ids(self) -> list[int]:
        return sorted(self._dev_group)

    def cpu_block_ids(self) -> list[int]:
        return sorted(self._host_group)

    def summary(self) -> dict:
        """Resident bytes and cumulative transfer stats as a plain dict (``kv_block_store.py:183-196``)."""
        self._drain()
        return {
            "gpu_blocks": len(self._dev_group),
            "cpu_blocks": len(self._host_group),
            "resident_gpu_bytes": self.resident_gpu_bytes(),
            "resident_cpu_bytes": self.resident_cpu_bytes(),
            "gpu_to_cpu_bytes": self.stats.gpu_to_cpu_bytes,
            "cpu_to_gpu_bytes": self.stats.cpu_to_gpu_bytes,
            "gpu_to_cpu_copies": self.stats.gpu_to_cpu_copies,
            "cpu_to_gpu_copies": self.stats.cpu_to_gpu_copies,
            "gpu_to_cpu_sec": self.stats.gpu_to_cpu_sec,
            "cpu_to_gpu_sec": self.stats.cpu_to_gpu_sec,
        }

    def apply_tiers(self, tiers: list[int], device: torch.device | str, sync: bool = True) -> dict[str, list[int]]:
        """Move each block to the tier the pager assigned it (0 GPU, anything else CPU;
        ids past the end of ``tiers`` go to CPU), in ascending block order like
        ``kv_block_store.py:198-227``.  All copies are queued on the copy stream;
        ``sync=True`` waits for them, ``sync=False`` orders the current stream after them.
        A RAM-budget error leaves the moves before it done (as in the reference).
        """
        device = torch.device(device)
        to_gpu: list[int] = []
        to_cpu: list[int] = []
        try:
            for block_id in sorted(set(self._dev_group) | set(self._host_group)):
                desired = tiers[block_id] if block_id < len(tiers) else 2
                if desired == 0:
                    if not self.has_gpu(block_id):
                        self._load(block_id, device)
                        to_gpu.append(block_id)
                elif not self.has_cpu(block_id):
                    self._offload(block_id)
                    to_cpu.append(block_id)
        except BaseException:
            self._drain()
            raise
        if sync:
            self._drain()
        else:
            self._order_after_copies()
        return {"to_gpu": to_gpu, "to_cpu": to_cpu}

    def reorder_batch_rows(self, new_row_indices: list[int]) -> None:
        """Reindex every block's batch rows on whichever tier it lives (``kv_block_store.py:229-254``):
        new row i takes old row ``new_row_indices[i]``; repeats duplicate, omissions drop.
        A new row count re-lays both pools for the new batch size (private pools only)."""
        idx = [int(i) for i in new_row_indices]
        if self.pools is None:
            return
        B = self.batch
        if any(not -B <= i < B for i in idx):
            raise IndexError(f"row index out of range for batch {B}: {new_row_indices}")
        idx = [i % B for i in idx]
        n = len(idx)
        p = self.pools
        if n != B and not self._owns_pools:
            raise ValueError("cannot change the row count of blocks that live in shared pools")
        self._drain()
        torch.cuda.current_stream(self.device).synchronize()
        old_dev, old_host = p.dev_pool, p.host_pool
        if n == B:
            new_dev, new_host = old_dev, old_host
        else:
            with torch.inference_mode(False):
                new_dev = torch.empty((p.dev_groups.capacity * n,) + p.slot_shape(), dtype=p.dtype, device=p.device)
                new_host = HostPool((p.host_groups.capacity * n,) + p.slot_shape(), p.dtype)
        for groups, old, new, dev in ((self._dev_group, old_dev, new_dev, True),
                                      (self._host_group, old_host.tensor, new_host.tensor, False)):
            if not groups:
                continue
            src = [g * B + i for g in groups.values() for i in idx]
            dst = [g * n + r for g in groups.values() for r in range(n)]
            where = self.device if dev else "cpu"
            rows = old.index_select(0, torch.tensor(src, dtype=torch.long, device=where))
            new.index_copy_(0, torch.tensor(dst, dtype=torch.long, device=where), rows)
        torch.cuda.current_stream(self.device).synchronize()
        if n != B:
            old_host.close()
            p.dev_pool, p.host_pool, p.rows_per_group = new_dev, new_host, n
            p.version += 1
            self._resident_gpu_bytes = self._resident_gpu_bytes // B * n
            self._resident_cpu_bytes = self._resident_cpu_bytes // B * n

    def get_gpu(self, block_id: int) -> tuple[torch.Tensor, torch.Tensor]:
        if block_id not in self._dev_group:
            raise KeyError(f"Block {block_id} is not on GPU.")
        return self._kv_view(block_id, True)

    def get_any(self, block_id: int) -> tuple[torch.Tensor, torch.Tensor]:
        """A block's (key, value) from whichever tier holds it, residency unchanged (``:256-274``)."""
        if block_id in self._dev_group:
            return self._kv_view(block_id, True)
        if block_id in self._host_group:
            self._drain()
            return self._kv_view(block_id, False)
        raise KeyError(f"Block {block_id} is not on GPU or CPU.")

    # ------------------------------------------------------------------ fused-op bridge
    def block_table(self, block_ids=None, device=None) -> torch.Tensor:
        """int32 ``[batch, len(block_ids)]`` table for ``paged_decode_attention``: row r of block j
        is ``slot`` (device pool) or ``slot | 0x40000000`` (host pool); absent blocks are -1.
        ``block_ids`` defaults to ``0 .. max id``."""
        if self.batch is None:
            raise ValueError("the store holds no blocks yet")
        if block_ids is None:
            known = set(self._dev_group) | set(self._host_group)
            block_ids = range(max(known) + 1) if known else range(0)
        ids = list(block_ids)
        dev = np.fromiter((self._dev_group.get(b, -1) for b in ids), dtype=np.int64, count=len(ids))
        host = np.fromiter((self._host_group.get(b, -1) for b in ids), dtype=np.int64, count=len(ids))
        short = [b for b in ids if b in self._tokens and self._tokens[b] != self.tokens_per_block]
        if short:
            b = short[0]
            raise ValueError(f"block {b} holds {self._tokens[b]} of {self.tokens_per_block} tokens; "
                             "the decode op reads whole blocks")
        B = self.batch
        rows = np.arange(B, dtype=np.int64)[:, None]
        table = np.full((B, len(ids)), -1, dtype=np.int64)
        on_dev = dev >= 0
        on_host = host >= 0
        table[:, on_dev] = dev[on_dev][None, :] * B + rows
        table[:, on_host] = (host[on_host][None, :] * B + rows) | HOST_SLOT_BIT
        return torch.from_numpy(table.astype(np.int32)).to(device if device is not None else self.device)

    def close(self) -> None:
        """Free this store's blocks; a store with private pools also frees its pinned host pool."""
        self._drain()
        if self.pools is None:
            return
        if self._owns_pools:
            self.pools.close()
        else:
            for g in self._dev_group.values():
                self.pools.dev_groups.give(g)
            for g in self._host_group.values():
                self.pools.host_groups.give(g)
        self._dev_group.clear()
        self._host_group.clear()
        self._tokens.clear()
        self._resident_gpu_bytes = self._resident_cpu_bytes = 0
