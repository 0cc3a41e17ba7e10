"""Request-sharded serving sweep of decode attention (the reference's serving config 5).

Continuous batching of long-context decode attention on N GPUs, one process
per GPU, the way the reference's serving stack shards independent requests
across replicas (``pager_hf/serving/multi_gpu.py``; no collective on the data
path):

* requests arrive as a Poisson process (default 256 at 8 req/s) with prompt
  lengths log-uniform in [1024, 65536] tokens and 256 output tokens each;
* every rank computes the same routing from the same seeded arrival list
  (least load first by prompt tokens, ``request_shard.RequestRouter``) and
  serves its share;
* a rank admits an arrived request when its pools have room for the request's
  whole life (KV blocks of prompt + output, a per-GPU HBM budget, the overflow
  in the pinned host pool), prefills its KV (seeded synthetic data: this
  harness times attention, not a model), and from then on decodes every active
  session together: one ``pager_append_tokens`` and one fused paged launch per
  layer (``batched_decode.BatchedDecodeAttention``), then each session's pager
  moves blocks between the tiers;
* a session leaves after its output tokens; its slots return to the pools.

Reported: decode tokens/s (all ranks' tokens over the slowest rank's wall
time), effective KV GB/s (attended KV bytes over the same time), per-request
latency from arrival to last token, mean step time.  The query, key and value
rows of each step are synthetic; the model half of a serving step
(projections, MLP, sampling) is not part of this hot path.

    PYTHONPATH=rust-llm-pager_b200 python -m pager_hf.serving_sweep [--requests 256 --rate 8 ...]
    PYTHONPATH=rust-llm-pager_b200 torchrun --nproc-per-node 8 -m pager_hf.serving_sweep ...
"""

from __future__ import annotations

import argparse
import json
import math
import os
import time
from collections import deque
from dataclasses import dataclass, field

import numpy as np
import torch

from ._lib import DeviceStatusError
from .batched_decode import BatchedDecodeAttention, DecodeSession
from .kv_block_store import KVPools
from .request_shard import device_for_local_rank, local_requests, shard_requests

LLAMA3_8B = dict(layers=32, hq=32, hkv=8, d=128)  # attention geometry of the reference's serving config
PAGER_BLOCK_BYTES = 16 * 1024 * 1024  # the pager's budget unit (pager/src/core.rs:6)


@dataclass
class Request:
    rid: int
    arrival: float  # seconds after the start of the sweep
    prompt_tokens: int
    out_tokens: int


def poisson_requests(n: int = 256, rate: float = 8.0, min_tokens: int = 1024, max_tokens: int = 65536,
                     out_tokens: int = 256, seed: int = 0) -> list[Request]:
    """Seeded Poisson arrivals (first at t=0) with log-uniform prompt lengths."""
    rng = np.random.default_rng(seed)
    gaps = rng.exponential(1.0 / rate, n)
    arrivals = np.concatenate(([0.0], np.cumsum(gaps[1:]))) if n else np.zeros(0)
    lengths = np.exp(rng.uniform(math.log(min_tokens), math.log(max_tokens), n)).astype(np.int64)
    lengths = np.clip(lengths, min_tokens, max_tokens)
    return [Request(i, float(a), int(ln), int(out_tokens)) for i, (a, ln) in enumerate(zip(arrivals, lengths))]


def route(requests: list[Request], world: int) -> list[int]:
    """Owner rank per request: least load first in arrival order, load = prompt tokens routed."""
    return shard_requests(len(requests), world, weights=[r.prompt_tokens for r in requests])


@dataclass
class _Active:
    req: Request
    session: DecodeSession
    generated: int = 0


@dataclass
class ShardStats:
    rank: int = 0
    requests: int = 0
    tokens: int = 0
    steps: int = 0
    wall_s: float = 0.0
    step_s: float = 0.0
    kv_bytes: int = 0
    host_bytes: int = 0  # of kv_bytes, those read from the pinned host tier
    link_gbs: float = 0.0  # this rank's measured host->device bandwidth (the faster of copy and zero-copy)
    latencies: list = field(default_factory=list)
    waits: list = field(default_factory=list)
    peak_sessions: int = 0
    host_blocks_peak: int = 0
    errors: list = field(default_factory=list)  # {"rid", "error"} per request failed by a faulted step


class ShardRunner:
    """One GPU's share of the sweep: admission, continuous batched decode, completion."""

    def __init__(self, device, *, geometry: dict = LLAMA3_8B, tokens_per_block: int = 64,
                 hbm_budget_bytes: float = 40e9, host_budget_bytes: float = 96e9, max_sessions: int = 16,
                 policy: str = "recent_only", dtype: torch.dtype = torch.bfloat16, seed: int = 0,
                 rounding: str = "reference"):
        self.device = torch.device(device)
        self.g = dict(geometry)
        self.tpb = tokens_per_block
        self.max_sessions = max_sessions
        self.policy = policy
        self.rounding = rounding  # of p before P.V: the reference's, or the one-pass kernel's
        L, hkv, d = self.g["layers"], self.g["hkv"], self.g["d"]
        elt = torch.tensor([], dtype=dtype).element_size()
        self.slot_bytes = 2 * L * hkv * tokens_per_block * d * elt
        self.token_bytes = self.slot_bytes // tokens_per_block  # K+V of one token, all layers
        hbm_blocks = int(hbm_budget_bytes // self.slot_bytes)
        self.resident = max(1, hbm_blocks // max_sessions)  # device blocks per session (its pager budget)
        gpu_groups = max_sessions * (self.resident + 2)  # + tail slot + the block a tail roll adds
        cpu_groups = max(1, int(host_budget_bytes // self.slot_bytes))
        self.pools = KVPools(num_layers=L, kv_heads=hkv, head_dim=d, tokens_per_block=tokens_per_block, dtype=dtype,
                             device=self.device, gpu_groups=gpu_groups, cpu_groups=cpu_groups)
        gen = torch.Generator(device=self.device).manual_seed(seed)
        self.template = torch.empty(self.pools.slot_shape(), dtype=dtype, device=self.device)
        self.template.normal_(generator=gen)  # the KV content of every synthetic block
        S = max_sessions
        self.q = torch.randn(L, S, self.g["hq"], d, generator=gen, device=self.device).to(dtype)
        self.kn = torch.randn(L, S, hkv, d, generator=gen, device=self.device).to(dtype)
        self.vn = torch.randn(L, S, hkv, d, generator=gen, device=self.device).to(dtype)
        self.dev_free0 = self.pools.dev_groups.capacity - self.pools.dev_groups.used
        self.host_free0 = self.pools.host_groups.capacity - self.pools.host_groups.used

    # ------------------------------------------------------------------ admission
    def _needs(self, req: Request):
        final_blocks = (req.prompt_tokens + req.out_tokens) // self.tpb
        resident = min(final_blocks, self.resident)
        return resident + 2, max(0, final_blocks - resident)

    def fits_ever(self, req: Request) -> bool:
        dev, host = self._needs(req)
        return dev <= self.pools.dev_groups.capacity and host <= self.pools.host_groups.capacity

    def _free(self):
        p = self.pools
        return p.dev_groups.capacity - p.dev_groups.used, p.host_groups.capacity - p.host_groups.used

    def _reserved(self, active):
        dev = host = 0
        for a in active:
            d, h = self._needs(a.req)
            s = a.session
            dev += max(0, d - (len(s.store.gpu_block_ids()) + 1))
            host += max(0, h - len(s.store.cpu_block_ids()))
        return dev, host

    def admit(self, req: Request, active) -> DecodeSession | None:
        """A session for ``req`` with its prompt's KV in place, or None while the pools lack room."""
        need_dev, need_host = self._needs(req)
        free_dev, free_host = self._free()
        res_dev, res_host = self._reserved(active)  # room the active sessions will still take
        if need_dev > free_dev - res_dev or need_host > free_host - res_host:
            return None
        p = self.pools
        kw = dict(vram=self.resident * PAGER_BLOCK_BYTES, ram=10 ** 15, recent=max(self.resident - 1, 0),
                  rebalance_interval=4, promote_margin=0.05, ram_promote_margin=0.20, policy=self.policy)
        s = DecodeSession(p, pager_kwargs=kw)
        nb = req.prompt_tokens // self.tpb
        on_dev_from = nb - min(nb, self.resident)  # the newest blocks start in HBM, as the pager will keep them
        host_view = p.host_pool.tensor
        for j in range(nb):
            if j >= on_dev_from:
                g = p.take_dev_group()
                p.dev_pool[g].copy_(self.template)
                s.store.adopt_gpu_group(j, g)
            else:
                g = p.take_host_group()
                host_view[g].copy_(self.template, non_blocking=True)
                s.store.adopt_host_group(j, g)
        p.dev_pool[s.tail_slot].copy_(self.template)
        s.num_blocks = nb
        s.tail_len = req.prompt_tokens - nb * self.tpb
        return s

    # ------------------------------------------------------------------ the serving loop
    def run(self, requests: list[Request], rank: int = 0) -> ShardStats:
        from .host_staging import link_bandwidth

        st = ShardStats(rank=rank, requests=len(requests))
        bw = link_bandwidth(self.device)
        st.link_gbs = max(bw["copy_gbs"], bw["zero_copy_gbs"])
        for r in requests:
            if not self.fits_ever(r):
                raise ValueError(f"request {r.rid} ({r.prompt_tokens} tokens) can never fit this rank's pools")
        pending = deque(sorted(requests, key=lambda r: r.arrival))
        active: list[_Active] = []
        torch.cuda.synchronize(self.device)
        t0 = time.perf_counter()
        step_time = 0.0
        while pending or active:
            now = time.perf_counter() - t0
            while pending and pending[0].arrival <= now and len(active) < self.max_sessions:
                s = self.admit(pending[0], active)
                if s is None:
                    break
                st.waits.append(now - pending[0].arrival)
                active.append(_Active(pending.popleft(), s))
            if not active:
                if pending:
                    time.sleep(max(0.0, pending[0].arrival - (time.perf_counter() - t0)))
                continue
            st.peak_sessions = max(st.peak_sessions, len(active))
            S = len(active)
            host_tokens = sum(len(a.session.store.cpu_block_ids()) for a in active) * self.tpb
            ts = time.perf_counter()
            plan = BatchedDecodeAttention([a.session for a in active], self.g["hq"], rounding=self.rounding)
            for layer in range(self.g["layers"]):
                plan.layer(layer, self.q[layer, :S], self.kn[layer, :S], self.vn[layer, :S])
            try:
                plan.finish()
            except DeviceStatusError as e:
                # a faulted step fails the requests it served, each with the reason, as the reference's
                # scheduler sets req.error and finishes a request whose step raised (scheduler.py:520-524)
                for a in active:
                    st.errors.append({"rid": a.req.rid, "error": str(e)})
                    a.session.close()
                active = []
                step_time += time.perf_counter() - ts
                continue
            torch.cuda.synchronize(self.device)
            step_time += time.perf_counter() - ts
            st.steps += 1
            st.tokens += S
            st.kv_bytes += sum(a.session.num_tokens for a in active) * self.token_bytes  # after finish():
            # num_tokens now counts this step's token too, i.e. what the step attended
            st.host_bytes += host_tokens * self.token_bytes
            st.host_blocks_peak = max(st.host_blocks_peak, self.pools.host_groups.used)
            done_at = time.perf_counter() - t0
            keep = []
            for a in active:
                a.generated += 1
                if a.generated >= a.req.out_tokens:
                    st.latencies.append(done_at - a.req.arrival)
                    a.session.close()
                else:
                    keep.append(a)
            active = keep
        torch.cuda.synchronize(self.device)
        st.wall_s = time.perf_counter() - t0
        st.step_s = step_time
        return st

    def close(self):
        self.pools.close()


def summarize(stats: list[ShardStats], hbm_gbs: float = 6553.3) -> dict:
    """The sweep's figures over all ranks.  ``roofline``: each rank's decode steps against the
    combined floor of its attended bytes -- the HBM-resident ones at ``hbm_gbs`` (a measured B200
    copy bandwidth by default) plus the host-resident ones at the rank's measured link bandwidth --
    as the floor's share of the time spent in decode steps (``frac_steps``) and of the rank's wall
    time, admission and prefill included (``frac_wall``); the slowest rank's figures."""
    wall = max(s.wall_s for s in stats) if stats else 0.0
    lat = sorted(x for s in stats for x in s.latencies)
    tokens = sum(s.tokens for s in stats)
    kv = sum(s.kv_bytes for s in stats)
    pct = (lambda q: lat[min(len(lat) - 1, int(q * len(lat)))] if lat else None)
    return {"ranks": len(stats), "requests": sum(s.requests for s in stats), "tokens": tokens, "wall_s": wall,
            "decode_tokens_per_s": tokens / wall if wall else None, "kv_gbs": kv / wall / 1e9 if wall else None,
            "latency_s": {"mean": sum(lat) / len(lat) if lat else None, "p50": pct(0.5), "p90": pct(0.9)},
            "mean_step_ms": 1000 * sum(s.step_s for s in stats) / max(1, sum(s.steps for s in stats)),
            "errors": [e for s in stats for e in s.errors],
            "roofline": _roofline(stats, hbm_gbs),
            "per_rank": [{"rank": s.rank, "requests": s.requests, "tokens": s.tokens, "wall_s": s.wall_s,
                          "step_s": s.step_s, "kv_gb": s.kv_bytes / 1e9, "host_gb": s.host_bytes / 1e9,
                          "link_gbs": s.link_gbs, "peak_sessions": s.peak_sessions,
                          "host_blocks_peak": s.host_blocks_peak}
                         for s in stats]}


def _roofline(stats: list[ShardStats], hbm_gbs: float) -> dict | None:
    rows = []
    for s in stats:
        if not s.step_s or not s.link_gbs:
            continue
        t_hbm = (s.kv_bytes - s.host_bytes) / (hbm_gbs * 1e9)
        t_host = s.host_bytes / (s.link_gbs * 1e9)
        floor = t_hbm + t_host
        rows.append({"rank": s.rank, "wall_s": s.wall_s, "floor_s": floor, "hbm_s": t_hbm, "host_link_s": t_host, "frac_steps": floor / s.step_s,
                     "frac_wall": floor / s.wall_s, "bound": "host link" if t_host > t_hbm else "hbm"})
    if not rows:
        return None
    return {"hbm_gbs": hbm_gbs, **max(rows, key=lambda r: r["wall_s"])}


def main(argv=None):
    ap = argparse.ArgumentParser(description="request-sharded decode-attention serving sweep")
    ap.add_argument("--requests", type=int, default=256)
    ap.add_argument("--rate", type=float, default=8.0)
    ap.add_argument("--min-tokens", type=int, default=1024)
    ap.add_argument("--max-tokens", type=int, default=65536)
    ap.add_argument("--out-tokens", type=int, default=256)
    ap.add_argument("--hbm-budget-gb", type=float, default=40.0)
    ap.add_argument("--host-budget-gb", type=float, default=96.0)
    ap.add_argument("--max-sessions", type=int, default=16)
    ap.add_argument("--policy", default="recent_only")
    ap.add_argument("--tokens-per-block", type=int, default=64)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--rounding", default="reference", choices=["reference", "one_pass"])
    ap.add_argument("--hbm-gbs", type=float, default=6553.3, help="HBM bandwidth of the roofline (GB/s)")
    a = ap.parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = device_for_local_rank(int(os.environ.get("LOCAL_RANK", "0")),
                                  int(os.environ.get("LOCAL_WORLD_SIZE", str(world))), torch.cuda.device_count())
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta

        dist.init_process_group("gloo", init_method="env://", timeout=timedelta(seconds=3600))
    reqs = poisson_requests(a.requests, a.rate, a.min_tokens, a.max_tokens, a.out_tokens, a.seed)
    mine = [reqs[i] for i in local_requests(route(reqs, world), rank)]
    runner = ShardRunner(f"cuda:{local}", tokens_per_block=a.tokens_per_block, hbm_budget_bytes=a.hbm_budget_gb * 1e9,
                         host_budget_bytes=a.host_budget_gb * 1e9, max_sessions=a.max_sessions, policy=a.policy,
                         seed=a.seed + rank, rounding=a.rounding)
    try:
        if world > 1:
            dist.barrier()
        st = runner.run(mine, rank)
    finally:
        runner.close()
    stats = [st]
    if world > 1:
        gathered = [None] * world
        dist.all_gather_object(gathered, st)
        stats = gathered
        dist.destroy_process_group()
    if rank == 0:
        out = summarize(stats, a.hbm_gbs)
        out["config"] = vars(a) | {"world": world}
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
