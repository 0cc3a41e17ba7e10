"""Host logic of the serving sweep (``pager_hf/serving_sweep.py``): arrivals, routing, summary."""

import math

import numpy as np

from pager_hf.serving_sweep import ShardStats, poisson_requests, route, summarize


def test_poisson_arrivals_and_log_uniform_lengths_are_seeded():
    a = poisson_requests(2000, rate=8.0, min_tokens=1024, max_tokens=65536, out_tokens=256, seed=3)
    b = poisson_requests(2000, rate=8.0, min_tokens=1024, max_tokens=65536, out_tokens=256, seed=3)
    assert [(r.arrival, r.prompt_tokens) for r in a] == [(r.arrival, r.prompt_tokens) for r in b]
    arr = np.array([r.arrival for r in a])
    assert arr[0] == 0.0 and np.all(np.diff(arr) >= 0)
    assert abs(np.mean(np.diff(arr)) - 1 / 8.0) < 0.012          # mean gap 1/rate
    lens = np.array([r.prompt_tokens for r in a])
    assert lens.min() >= 1024 and lens.max() <= 65536
    assert abs(np.median(np.log(lens)) - 0.5 * (math.log(1024) + math.log(65536))) < 0.2  # log-uniform
    assert all(r.out_tokens == 256 for r in a)


def test_routing_is_deterministic_and_balances_prompt_tokens():
    reqs = poisson_requests(256, seed=0)
    owners = route(reqs, 8)
    assert owners == route(reqs, 8)
    load = np.zeros(8)
    for r, o in zip(reqs, owners):
        load[o] += r.prompt_tokens
    assert load.max() - load.min() <= max(r.prompt_tokens for r in reqs)
    assert route(reqs, 1) == [0] * 256


def test_summary_aggregates_over_ranks():
    s0 = ShardStats(rank=0, requests=2, tokens=10, steps=5, wall_s=2.0, step_s=1.0, kv_bytes=4 * 10**9,
                    latencies=[1.0, 2.0])
    s1 = ShardStats(rank=1, requests=1, tokens=6, steps=6, wall_s=4.0, step_s=2.0, kv_bytes=4 * 10**9,
                    latencies=[3.0])
    out = summarize([s0, s1])
    assert out["tokens"] == 16 and out["wall_s"] == 4.0
    assert out["decode_tokens_per_s"] == 4.0 and out["kv_gbs"] == 2.0
    assert out["latency_s"]["mean"] == 2.0 and out["latency_s"]["p50"] == 2.0
    assert abs(out["mean_step_ms"] - 1000 * 3.0 / 11) < 1e-9


def test_roofline_is_the_slowest_ranks_combined_floor():
    # rank 0: 3 GB from HBM at 6000 GB/s (0.5 ms) + 1 GB from the host at 50 GB/s (20 ms) in 25 ms of steps
    s0 = ShardStats(rank=0, requests=1, tokens=4, steps=4, wall_s=0.05, step_s=0.025, kv_bytes=4 * 10**9,
                    host_bytes=10**9, link_gbs=50.0)
    # rank 1 (the faster one): HBM only, 6 GB (1 ms) in 4 ms of steps
    s1 = ShardStats(rank=1, requests=1, tokens=4, steps=4, wall_s=0.004, step_s=0.004, kv_bytes=6 * 10**9,
                    host_bytes=0, link_gbs=50.0)
    r = summarize([s0, s1], hbm_gbs=6000.0)["roofline"]
    assert r["bound"] == "host link"
    assert abs(r["floor_s"] - 0.0205) < 1e-12
    assert abs(r["frac_steps"] - 0.0205 / 0.025) < 1e-9 and abs(r["frac_wall"] - 0.0205 / 0.05) < 1e-9
    assert summarize([s1], hbm_gbs=6000.0)["roofline"]["bound"] == "hbm"
    assert summarize([ShardStats()])["roofline"] is None
