"""Request sharding across GPUs: one process per GPU, no exchange on the data path.

Decode attention shards by request: a row's attention reads only that row's KV
blocks, so each GPU holds its own device pool, pinned host pool and requests,
and the only cross-rank traffic is control (routing, a barrier, the timing
reduction).  Routing follows the reference's ``MultiGpuScheduler``
(``pager_hf/serving/multi_gpu.py:11-103``): one-shot requests go to the
least-loaded replica (``_by_load()[0]``, a stable sort on ``load()``, so ties go
to the lowest rank, ``:37-38``, ``:66-68``), where load is accepted-but-unfinished
requests (``scheduler.py:295-301``); a session stays on the rank that created
it (``:90-97``), and session creation falls back to the next-least-loaded rank
when a rank's session registry is full (``:70-88``).
"""

from __future__ import annotations

import threading


class SessionCapacityError(RuntimeError):
    """Every rank's session registry is full (``scheduler.py``'s SessionCapacityError)."""


class RequestRouter:
    """Least-load routing of requests and sessions over ``world`` ranks.

    Every rank can hold its own copy and reach the same decisions from the same
    inputs: routing is a deterministic function of the arrival order.
    """

    def __init__(self, world: int, session_capacity: int | None = None):
        if world < 1:
            raise ValueError("RequestRouter requires at least one rank")
        self.world = world
        self._load = [0] * world
        self._sessions = [0] * world
        self._capacity = session_capacity
        self._owner: dict[str, int] = {}
        self._next_session = 0
        self._lock = threading.Lock()

    def load(self, rank: int) -> int:
        return self._load[rank]

    def _by_load(self) -> list[int]:
        return sorted(range(self.world), key=lambda r: self._load[r])

    def submit(self, weight: int = 1) -> int:
        """Rank that serves a one-shot request (least loaded; ties to the lowest rank)."""
        with self._lock:
            rank = self._by_load()[0]
            self._load[rank] += weight
            return rank

    def finish(self, rank: int, weight: int = 1) -> None:
        with self._lock:
            if self._load[rank] < weight:
                raise ValueError(f"rank {rank} has load {self._load[rank]}, cannot finish {weight}")
            self._load[rank] -= weight

    def create_session(self) -> str:
        """New session on the least-loaded rank whose registry has room."""
        with self._lock:
            for rank in self._by_load():
                if self._capacity is not None and self._sessions[rank] >= self._capacity:
                    continue
                sid = f"rank{rank}:session:{self._next_session}"
                self._next_session += 1
                self._sessions[rank] += 1
                self._owner[sid] = rank
                return sid
        raise SessionCapacityError(f"all {self.world} ranks have {self._capacity} sessions")

    def owner(self, session_id: str) -> int:
        """Rank a session lives on; KeyError for an unknown session (``multi_gpu.py:90-95``)."""
        with self._lock:
            return self._owner[session_id]

    def delete_session(self, session_id: str) -> None:
        with self._lock:
            rank = self._owner.pop(session_id)
            self._sessions[rank] -= 1


def device_for_local_rank(local_rank: int, local_world: int, visible: int) -> int:
    """The GPU index a rank drives on its node.

    With as many GPUs visible as ranks on the node, rank r drives GPU r.  With more GPUs visible than
    ranks, the ranks spread evenly over them (rank r drives GPU r * (visible // local_world)) instead
    of taking the first ones: each rank reads its host tier over its own GPU's host link, and on
    8-GPU B200 boxes neighbouring GPUs share host-side IO -- measured with every GPU of a set copying
    from pinned memory at once, GPUs 0-3 got 29 GB/s each, GPUs 0, 2, 4, 6 got 53-55 GB/s each.
    """
    if local_world <= 0 or visible <= local_world or not 0 <= local_rank < local_world:
        return local_rank
    return local_rank * (visible // local_world)


def shard_requests(num_requests: int, world: int, weights=None) -> list[int]:
    """Owner rank of each request, routed in arrival order by least load.

    ``weights`` (e.g. KV tokens per request) makes the load the routed weight
    instead of the request count.
    """
    router = RequestRouter(world)
    w = [1] * num_requests if weights is None else list(weights)
    if len(w) != num_requests:
        raise ValueError("weights must have one entry per request")
    return [router.submit(x) for x in w]


def local_requests(owners: list[int], rank: int) -> list[int]:
    """Indices of the requests owned by ``rank``, in arrival order."""
    return [i for i, r in enumerate(owners) if r == rank]


def max_over_ranks(value: float, device=None) -> float:
    """Maximum of a per-rank value over the default process group (identity without one).

    Multi-GPU timings are the slowest rank's device time; every rank must call
    this at the same point.
    """
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def aggregate_rate(units_per_rank: list[float] | float, max_seconds: float, world: int = 1) -> float:
    """Whole-job rate: units processed by all ranks / the slowest rank's time."""
    total = sum(units_per_rank) if isinstance(units_per_rank, (list, tuple)) else world * float(units_per_rank)
    return total / max_seconds
