"""Cross-session batched decode attention: one launch per layer for many sessions.

The attention half of the reference's ``batched_decode_step``
(``pager_hf/batched_decode.py:32-348``): several single-row decode sessions,
each with its own block store and pager, advance by one token with one fused
``paged_decode_attention`` launch per layer instead of a per-row, per-block
Python gather (``:143-219``) and a group loop.  The model half (projections,
RoPE, MLP, the logits) belongs to the caller: ``layer()`` takes the layer's
query and new key/value rows and returns the attention output.

B200 layout: the sessions share one ``KVPools`` (device pool + pinned host
pool), so a single int32 block table names every session's blocks on either
tier.  A session's tail (tokens after its last full block) lives in a device
pool slot; each step's new K/V is written into it (``pager_append_tokens``)
and the decode op reads it as the row's last block with ``valid_hi`` marking
its real tokens.  When the tail reaches ``tokens_per_block`` tokens it already
is a full block in the pool: it is registered with the store without a copy
(the reference stacks and copies it, ``paged_model.py:1210-1233``).

Lifted restrictions of the reference (``batched_decode.py:80-108``): tails
need not have equal lengths, sessions may use sliding windows (per-row
``valid_lo``), and attention-scoring and uniform policies may share a launch.
After ``finish()``, each session's pager sees exactly what the reference's
post-step sequence gives it (``:320-338``): ``on_step(query_block, 0,
block_attention)``, ``force_rebalance`` when a block was added, then
``apply_tiers``.
"""

from __future__ import annotations

import torch

from . import _lib as L
from .kv_block_store import KVBlockStore, KVPools
from .streaming_attention import PagedDecodePlan

_SCORING_POLICIES = frozenset({"heavy_hitter", "sinks_heavy_hitter"})


class DecodeSession:
    """One single-row decode session over shared pools: blocks, tail slot, pager."""

    def __init__(self, pools: KVPools, *, pager_kwargs: dict | None = None, ram_budget_bytes: int | None = None,
                 sliding_window: int | None = None, needs_attention: bool | None = None):
        if pools.rows_per_group != 1:
            raise ValueError("decode sessions are single-row: the shared pools must have rows_per_group=1")
        self.pools = pools
        self.store = KVBlockStore(pools.tokens_per_block, ram_budget_bytes, pools=pools)
        self.pager = None
        if pager_kwargs is not None:
            import pager as _pager

            self.pager = _pager.PyPager(**pager_kwargs)
        policy = (pager_kwargs or {}).get("policy", "heavy_hitter")
        self.needs_attention = (policy in _SCORING_POLICIES) if needs_attention is None else bool(needs_attention)
        self.sliding_window = sliding_window
        self.num_blocks = 0
        self.tail_len = 0
        self.tail_group = pools.take_dev_group()
        self.mass_accum: torch.Tensor | None = None

    @property
    def tail_slot(self) -> int:
        return self.tail_group

    @property
    def num_tokens(self) -> int:
        return self.num_blocks * self.pools.tokens_per_block + self.tail_len

    def prefill(self, keys, values) -> None:
        """Load a prompt's KV: per layer ``[1, kv_heads, T, head_dim]`` (the HF cache layout).
        Full blocks go to the device pool as blocks 0.., the rest into the tail slot."""
        p = self.pools
        if len(keys) != p.num_layers or len(values) != p.num_layers:
            raise ValueError(f"need {p.num_layers} key and value tensors")
        T = keys[0].shape[2]
        tpb = p.tokens_per_block
        full = T // tpb
        for j in range(full):
            self.store.put_gpu_layers(self.num_blocks, [k[:, :, j * tpb:(j + 1) * tpb] for k in keys],
                                      [v[:, :, j * tpb:(j + 1) * tpb] for v in values])
            self.num_blocks += 1
        rem = T - full * tpb
        for layer, (k, v) in enumerate(zip(keys, values)):
            p.dev_pool[self.tail_slot, layer, 0, :, :rem].copy_(k[0, :, full * tpb:])
            p.dev_pool[self.tail_slot, layer, 1, :, :rem].copy_(v[0, :, full * tpb:])
        self.tail_len = rem

    def block_attention(self, num_layers: int) -> list[float]:
        """``PagedModel._finalize_streaming_block_attention`` (``paged_model.py:865-876``)."""
        n = self.num_blocks
        if n == 0 or self.mass_accum is None:
            return [1.0 / n] * n if n else []
        averaged = (self.mass_accum / num_layers).tolist()
        total = sum(averaged)
        if total <= 0:
            return [1.0 / n] * n
        return [x / total for x in averaged]

    def close(self) -> None:
        self.store.close()
        self.pools.dev_groups.give(self.tail_group)


class BatchedDecodeAttention:
    """One decode step of attention for ``sessions``: ``layer()`` per layer, then ``finish()``.

    ``rounding`` (``paged_decode_attention``): "reference" rounds p as the reference's cross-session
    path does -- its two-pass sequence when any session scores blocks, its one-pass sequence
    otherwise (batched_decode.py:236-285), each session sitting as far into the reference's combined
    block numbering as it has fewer blocks than the longest (``:185-234``), in groups of
    ``group_size_blocks`` blocks; "one_pass" is the one-pass kernel."""

    def __init__(self, sessions: list[DecodeSession], num_query_heads: int, *, scale: float | None = None,
                 softcap: float | None = None, rounding: str = "reference", group_size_blocks: int = 64):
        if not sessions:
            raise ValueError("batched decode needs at least one session")
        pools = sessions[0].pools
        for s in sessions:
            if s.pools is not pools:
                raise ValueError("batched decode requires every session to share the same KVPools")
        self.sessions, self.pools = list(sessions), pools
        S, tpb = len(sessions), pools.tokens_per_block
        self.device = pools.device
        width = max(s.num_blocks for s in sessions) + 1  # + the tail slot
        table = torch.full((S, width), -1, dtype=torch.int32)
        nblk, lo, hi, slots, pos = [], [], [], [], []
        any_window = False
        for r, s in enumerate(sessions):
            if s.num_blocks:
                table[r, :s.num_blocks] = s.store.block_table(range(s.num_blocks), device="cpu")[0]
            table[r, s.num_blocks] = s.tail_slot
            nblk.append(s.num_blocks + 1)
            total = s.num_tokens + 1  # with this step's token
            hi.append(total)
            if s.sliding_window is not None:
                any_window = True
                lo.append(max(0, total - int(s.sliding_window)))  # keeps positions > pos - window
            else:
                lo.append(0)
            slots.append(s.tail_slot)
            pos.append(s.tail_len)
        i32 = dict(dtype=torch.int32, device=self.device)
        self.table = table.to(self.device)
        self.num_blocks = torch.tensor(nblk, **i32)
        self.valid_hi = torch.tensor(hi, **i32)
        self.valid_lo = torch.tensor(lo, **i32) if any_window else None
        self.slots = torch.tensor(slots, **i32)
        self.positions = torch.tensor(pos, **i32)
        self.needs_attention = any(s.needs_attention for s in sessions)
        self.mass = torch.zeros(S, width, dtype=torch.float32, device=self.device) if self.needs_attention else None
        from .paged_model import step_rounding

        max_nb = width - 1
        self.plan = PagedDecodePlan(
            batch=S, num_query_heads=num_query_heads, dev_pool=pools.dev_pool, host_pool=pools.host_pool.tensor,
            num_layers=pools.num_layers, tokens_per_block=tpb, block_table=self.table, num_blocks=self.num_blocks,
            max_row_tokens=width * tpb, valid_lo=self.valid_lo, valid_hi=self.valid_hi, scale=scale,
            softcap=softcap, mass_accum=self.mass, mass_mode="row_mean" if self.needs_attention else "none",
            rounding=step_rounding(rounding, self.needs_attention, pools.dtype, pools.head_dim, tpb),
            ref_group_tokens=group_size_blocks * tpb,
            ref_shift=torch.tensor([(max_nb - s.num_blocks) * tpb for s in sessions], **i32),
            ref_tail_start=torch.tensor([s.num_blocks * tpb for s in sessions], **i32))
        self._layers_done = 0
        self._lib = L.lib()

    def layer(self, layer: int, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
              out: torch.Tensor | None = None) -> torch.Tensor:
        """Attention of one layer: q ``[S, Hq, D]``; k_new / v_new ``[S, Hkv, D]`` (or ``[S, Hkv, 1, D]``)
        in the pools' dtype.  Writes the new token into each tail slot, then runs the fused op."""
        p = self.pools
        S = len(self.sessions)
        k_new = k_new.reshape(S, p.kv_heads, p.head_dim).contiguous()
        v_new = v_new.reshape(S, p.kv_heads, p.head_dim).contiguous()
        if k_new.dtype != p.dtype or v_new.dtype != p.dtype or k_new.device != self.device:
            raise ValueError("k_new / v_new must be on the pools' device in the pools' dtype")
        if p.dev_pool.data_ptr() != self.plan.dev_pool.data_ptr():
            raise RuntimeError("the shared pools grew after this step was planned; plan the step again")
        stream = torch.cuda.current_stream(self.device).cuda_stream
        L.check(self._lib.pager_append_tokens(
            p.dev_pool.data_ptr(), L.DTYPE_CODE[p.dtype], p.dev_pool.shape[0], p.num_layers, layer, p.kv_heads,
            p.tokens_per_block, p.head_dim, self.slots.data_ptr(), self.positions.data_ptr(), k_new.data_ptr(),
            v_new.data_ptr(), S, stream))
        if out is None:
            out = torch.empty(q.shape, dtype=q.dtype, device=self.device)
        self.plan.run(q.contiguous(), layer, out)
        self._layers_done += 1
        return out

    def finish(self, apply_tiers: bool = True) -> list[list[float]]:
        """Advance every session by the decoded token (``batched_decode.py:320-338``): roll a full
        tail into a block, hand the step's block attention to the pager, move blocks to the tiers
        it picks.  Returns each session's block attention list.  Raises ``DeviceStatusError`` (before
        any session changes) when the step's kernels flagged a timed-out wait or a slot outside its
        pool."""
        p = self.pools
        tpb = p.tokens_per_block
        L.watch_for(self.device).sync_and_check("batched decode attention step")
        mass = self.mass.cpu() if self.mass is not None else None
        result = []
        for r, s in enumerate(self.sessions):
            old_nb = s.num_blocks
            s.mass_accum = mass[r, :old_nb].clone() if (mass is not None and s.needs_attention) else None
            s.tail_len += 1
            added = []
            if s.tail_len == tpb:  # the tail slot now holds a full block: adopt it, take a fresh slot
                s.store.adopt_gpu_group(s.num_blocks, s.tail_group)
                added.append(s.num_blocks)
                s.num_blocks += 1
                s.tail_group = p.take_dev_group()
                s.tail_len = 0
            if s.num_blocks == 0:
                result.append([])
                continue
            if s.needs_attention:
                attention = s.block_attention(p.num_layers)
            else:
                attention = [1.0 / s.num_blocks] * s.num_blocks
            result.append(attention)
            if s.pager is not None:
                query_block = s.num_blocks - 1
                s.pager.on_step(query_block, 0, attention)
                if added:
                    s.pager.force_rebalance(query_block)
                if apply_tiers:
                    s.store.apply_tiers(s.pager.tiers(), self.device, sync=False)
        return result


def _validate_sessions(sessions: list, next_input_ids: list[int]) -> None:
    """The reference's checks (``batched_decode.py:72-108``) that still apply; all run before any device
    work.  Lifted: equal tail lengths, equal ``streaming_group_size_blocks`` (one launch per layer
    covers any number of blocks), one kind of policy, sliding-window models."""
    first = sessions[0]
    for s in sessions:
        if s.model is not first.model:
            raise ValueError("batched_decode_step requires every session to share the same underlying model.")
        if not s.use_streaming_attention:
            raise ValueError("batched_decode_step only supports use_streaming_attention=True sessions.")
        if s._store is None:
            raise ValueError("batched_decode_step requires every session to already have an active generate() session.")
        if s.tokens_per_block != first.tokens_per_block:
            raise ValueError("batched_decode_step requires every session to share the same tokens_per_block.")
        tail = s._tail_past
        if not tail or tail[0][0].shape[0] != 1:  # the session's row count, as the reference reads it
            raise ValueError("batched_decode_step only supports single-row (batch_size==1) sessions.")
    if len({id(s) for s in sessions}) != len(sessions):
        raise ValueError("batched_decode_step got the same session twice.")
    if len(next_input_ids) != len(sessions):
        raise ValueError("batched_decode_step needs one next input id per session.")


def _group_rounding(group: list, arch: dict) -> str:
    """The rounding of p for a set of sessions decoded in one launch: the reference's batched path
    runs its two-pass sequence when the sessions score blocks and its one-pass sequence otherwise
    (batched_decode.py:236-285); with mixed policies (which the reference rejects) the two-pass one."""
    from .paged_model import step_rounding

    first = group[0]
    return step_rounding(getattr(first, "attention_rounding", "reference"), any(s._needs_attention for s in group), first.model.dtype,
                         arch["d"], first.tokens_per_block)


def _group_plan(group: list, arch: dict, pools: KVPools, device: torch.device, max_nb: int):
    """The fused op's plans for single-row sessions that share ``pools`` (one per distinct sliding
    window of the model): one block-table row per session (its blocks on either tier, then its tail
    slot), per-row valid ranges (left padding, sliding window), and the per-row block-mass output
    when any session scores blocks.  For the reference rounding of p each row sits
    ``(max_nb - blocks) * tokens_per_block`` tokens into the reference's combined block numbering
    (sessions with fewer blocks are padded in front, ``max_nb`` being the most blocks of any session
    in the step, batched_decode.py:185-234)."""
    from .paged_model import window_lo

    S, tpb = len(group), pools.tokens_per_block
    width = max(s._num_blocks for s in group) + 1
    table = torch.full((S, width), -1, dtype=torch.int32)
    los, hi, slots, positions = [[] for _ in arch["windows"]], [], [], []
    for r, s in enumerate(group):
        nb = s._num_blocks
        if nb:
            table[r, :nb] = s._store.block_table(range(nb), device="cpu")[0]
        table[r, nb] = s._tail_group  # single-row groups: the group is the slot
        total = s._total + 1  # columns including this step's token
        pad = int(s._pad[0])
        for lo, w in zip(los, arch["windows"]):
            lo.append(window_lo(pad, total, w))
        hi.append(total)
        slots.append(s._tail_group)
        positions.append(s._tail_len)
    i32 = dict(dtype=torch.int32, device=device)
    needs = any(s._needs_attention for s in group)
    mass = torch.zeros(S, width, dtype=torch.float32, device=device) if needs else None
    table_dev = table.to(device)
    num_blocks = torch.tensor([s._num_blocks + 1 for s in group], **i32)
    valid_hi = torch.tensor(hi, **i32)
    shift = torch.tensor([(max_nb - s._num_blocks) * tpb for s in group], **i32)
    tail_start = torch.tensor([s._num_blocks * tpb for s in group], **i32)
    plans = [PagedDecodePlan(
        batch=S, num_query_heads=arch["hq"], dev_pool=pools.dev_pool, host_pool=pools.host_pool.tensor,
        num_layers=arch["layers"], tokens_per_block=tpb, block_table=table_dev, num_blocks=num_blocks,
        max_row_tokens=width * tpb, valid_lo=torch.tensor(lo, **i32) if any(lo) else None, valid_hi=valid_hi,
        scale=arch["scale"], softcap=arch["softcap"], mass_accum=mass, mass_mode="row_mean" if needs else "none",
        host_read=group[0].host_read, rounding=_group_rounding(group, arch),
        ref_group_tokens=group[0].streaming_group_size_blocks * tpb, ref_shift=shift, ref_tail_start=tail_start)
        for lo in los]
    return plans, mass, torch.tensor(slots, **i32), torch.tensor(positions, **i32)


def _group_ints(group: list, arch: dict, width: int, max_nb: int) -> torch.Tensor:
    """The per-step int32 inputs of one pools group, packed as a captured step reads them: the block
    table ``[rows, width]`` (each row's blocks, its tail slot, then absent columns), then per row the
    block count (blocks + tail), range end, tail slot, tail position, offset into the reference's
    combined block numbering, first tail token (``_group_plan``) and the first attended column for
    each distinct sliding window."""
    from .paged_model import window_lo

    S, nw = len(group), len(arch["windows"])
    tpb = group[0].tokens_per_block
    table = torch.full((S, width), -1, dtype=torch.int32)
    cols = torch.zeros(6 + nw, S, dtype=torch.int32)
    for r, s in enumerate(group):
        nb = s._num_blocks
        if nb:
            table[r, :nb] = s._store.block_table(range(nb), device="cpu")[0]
        table[r, nb] = s._tail_group
        total = s._total + 1
        pad = int(s._pad[0])
        cols[0, r] = nb + 1
        cols[1, r] = total
        cols[2, r] = s._tail_group
        cols[3, r] = s._tail_len
        cols[4, r] = (max_nb - nb) * tpb
        cols[5, r] = nb * tpb
        for i, w in enumerate(arch["windows"]):
            cols[6 + i, r] = window_lo(pad, total, w)
    return torch.cat([table.reshape(-1), cols.reshape(-1)])


class _BatchedGraph:
    """``batched_decode_step`` for one ordered set of sessions captured as a CUDA graph (see
    ``paged_model._DecodeGraph``): per pools group a packed int32 input buffer (``_group_ints``) and a
    mass buffer, the token and position ids of all rows, one plan per group with zero-copy host reads.
    The key -- the sessions, and per group the pools, their version and the table width (blocks plus
    tail, rounded up to ``_DecodeGraph.WIDTH_STEP``) -- changes when a session joins or leaves, a pool
    grows, or a session's blocks cross a width step."""

    def __init__(self, key, sessions, by_pools, arch, widths, device):
        from .paged_model import AttentionGroup

        self.key, self.arch = key, arch
        self.model = sessions[0].model
        S = len(sessions)
        self.input_ids = torch.zeros(S, 1, dtype=torch.long, device=device)
        self.position_ids = torch.zeros(S, 1, dtype=torch.long, device=device)
        self.groups, self.buffers = [], []
        for (rows, width) in zip(by_pools, widths):
            members = [sessions[r] for r in rows]
            pools = members[0]._pools
            n, nw = len(rows), len(arch["windows"])
            ints = torch.zeros(n * width + (6 + nw) * n, dtype=torch.int32, device=device)
            table = ints[: n * width].view(n, width)
            cols = ints[n * width:].view(6 + nw, n).unbind(0)
            nbs, hi, slots, positions, shift, tail_start = cols[:6]
            needs = any(s._needs_attention for s in members)
            mass = torch.zeros(n, width, dtype=torch.float32, device=device) if needs else None
            plans = [PagedDecodePlan(
                batch=n, num_query_heads=arch["hq"], dev_pool=pools.dev_pool, host_pool=pools.host_pool.tensor,
                num_layers=arch["layers"], tokens_per_block=pools.tokens_per_block, block_table=table, num_blocks=nbs,
                max_row_tokens=width * pools.tokens_per_block, valid_lo=lo, valid_hi=hi, scale=arch["scale"],
                softcap=arch["softcap"], mass_accum=mass, mass_mode="row_mean" if needs else "none",
                host_read="zero_copy", rounding=_group_rounding(members, arch),
                ref_group_tokens=members[0].streaming_group_size_blocks * pools.tokens_per_block, ref_shift=shift,
                ref_tail_start=tail_start) for lo in cols[6:]]
            index = None if len(by_pools) == 1 else torch.tensor(rows, dtype=torch.long, device=device)
            self.groups.append(AttentionGroup(pools, plans, slots, positions, index))
            self.buffers.append((rows, width, ints, mass))
        self.device = torch.device(device)
        self.graph = None
        self.logits = None

    def _run(self):
        from .paged_model import run_decoder_step

        for _, _, _, mass in self.buffers:
            if mass is not None:
                mass.zero_()
        return run_decoder_step(self.model, self.arch, self.groups, self.input_ids, self.position_ids)

    def step(self, sessions, next_input_ids, pos_ids):
        max_nb = max(s._num_blocks for s in sessions)
        for rows, width, ints, _ in self.buffers:
            ints.copy_(_group_ints([sessions[r] for r in rows], self.arch, width, max_nb))
        self.input_ids.copy_(torch.tensor(next_input_ids, dtype=torch.long)[:, None])
        self.position_ids.copy_(torch.tensor(pos_ids, dtype=torch.long)[:, None])
        with torch.cuda.device(self.device):
            if self.graph is None:
                cur = torch.cuda.current_stream()
                side = torch.cuda.Stream()
                side.wait_stream(cur)
                with torch.cuda.stream(side):
                    self._run()
                cur.wait_stream(side)
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, capture_error_mode="thread_local"):
                    self.logits = self._run()
                self.graph = graph
            self.graph.replay()
        return self.logits


# The last captured batched step per device (one at a time per device: each holds its own memory;
# per device, so that scheduler threads driving different GPUs keep their own).  A cached graph keeps
# its sessions' pools referenced until a batched step of another composition on that device
# replaces it.
_BATCHED_GRAPH: dict = {}


def _batched_graph_for(sessions, by_pools, arch, device):
    from .paged_model import _DecodeGraph

    groups = list(by_pools.values())
    widths = [_DecodeGraph.width_for(max(sessions[r]._num_blocks for r in rows)) for rows in groups]
    # a cached graph references its model and pools, so their ids cannot be reused while it is cached
    key = (id(sessions[0].model), tuple(id(s) for s in sessions),
           tuple((id(sessions[rows[0]]._pools), sessions[rows[0]]._pools.version, w,
                  any(sessions[r]._needs_attention for r in rows)) for rows, w in zip(groups, widths)))
    dev = torch.device(device).index
    cached = _BATCHED_GRAPH.get(dev)
    if cached is not None and cached.key == key:
        return cached
    _BATCHED_GRAPH.pop(dev, None)  # release the previous graph's memory before capturing the next
    g = _BatchedGraph(key, sessions, groups, arch, widths, device)
    _BATCHED_GRAPH[dev] = g
    return g


@torch.inference_mode()
def batched_decode_step(sessions: list, next_input_ids: list[int], device) -> list[torch.Tensor]:
    """Advance single-row ``PagedModel`` sessions by one token each in one model forward
    (``batched_decode.py:32-348``); returns each session's last-position logits in order.

    The sessions must share one model and ``tokens_per_block`` and each must have an active session
    (a ``generate`` call made).  Projections, RoPE, MLP and logits run once over all rows.  Attention
    runs as one fused paged launch per layer for each set of sessions that share a ``KVPools``: one
    launch for sessions created with ``PagedModel(..., pools=shared)``, one per session for sessions
    that allocated their own pools (as the reference's serving scheduler creates them).  Rows of
    different lengths, tails of different lengths, per-row sliding windows and mixed policies are
    fine (the reference requires equal tails and one kind of policy and rejects windows, ``:80-108``).
    Afterwards each session gets the reference's post-step calls (``:320-338``) on its own pager and
    store, through ``PagedModel._finish_token``, and its primed prefix grows by the token fed, so a
    later ``generate`` call on it continues from here.
    """
    from .paged_model import AttentionGroup, run_decoder_step

    if not sessions:
        return []
    _validate_sessions(sessions, next_input_ids)
    device = torch.device(device)
    if device.type == "cuda" and device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    by_pools: dict[int, list[int]] = {}
    for r, s in enumerate(sessions):
        if s._pools.device != device:
            raise ValueError(f"batched_decode_step: a session's KV lives on {s._pools.device}, not on {device}.")
        by_pools.setdefault(id(s._pools), []).append(r)
    first = sessions[0]
    a = first._arch()
    S = len(sessions)
    pos_ids = [s._total - int(s._pad[0]) for s in sessions]  # RoPE position of the new token
    if all(getattr(s, "decode_graphs", False) for s in sessions):
        g = _batched_graph_for(sessions, by_pools, a, device)
        logits = g.step(sessions, next_input_ids, pos_ids)
        L.watch_for(device).sync_and_check("batched_decode_step")
        for rows, _, _, mass in g.buffers:
            for i, r in enumerate(rows):
                s = sessions[r]
                s._finish_token(mass[i, :s._num_blocks] if (mass is not None and s._needs_attention) else None)
                s._note_fed_token(int(next_input_ids[r]))
                s.last_host_read = "zero_copy"
        # the graph's logits buffer is overwritten by the next replay: hand out a copy, as the eager
        # path (and the reference) hand out fresh tensors
        last = logits[:, -1, :].clone()
        return [last[r] for r in range(S)]
    groups, masses = [], []
    max_nb = max(s._num_blocks for s in sessions)
    for rows in by_pools.values():
        members = [sessions[r] for r in rows]
        plans, mass, slots, positions = _group_plan(members, a, members[0]._pools, device, max_nb)
        index = None if len(by_pools) == 1 else torch.tensor(rows, dtype=torch.long, device=device)
        groups.append(AttentionGroup(members[0]._pools, plans, slots, positions, index))
        masses.append((rows, mass))
    input_ids = torch.tensor(next_input_ids, dtype=torch.long, device=device)[:, None]
    position_ids = torch.tensor(pos_ids, dtype=torch.long, device=device)[:, None]
    logits = run_decoder_step(first.model, a, groups, input_ids, position_ids)
    L.watch_for(device).sync_and_check("batched_decode_step")
    for rows, mass in masses:
        for i, r in enumerate(rows):
            s = sessions[r]
            s._finish_token(mass[i, :s._num_blocks] if (mass is not None and s._needs_attention) else None)
            s._note_fed_token(int(next_input_ids[r]))
    return [logits[r, -1, :] for r in range(S)]
