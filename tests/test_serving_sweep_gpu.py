"""A small serving sweep on one GPU: every request finishes with all its tokens, blocks move to the
host tier along the way, and every slot returns to the pools at the end."""

import pytest

pytestmark = pytest.mark.gpu


def test_small_sweep_completes_and_frees_the_pools():
    from pager_hf import _lib
    from pager_hf.serving_sweep import ShardRunner, poisson_requests, summarize

    geometry = dict(layers=2, hq=8, hkv=2, d=64)
    slot = 2 * 2 * 2 * 16 * 64 * 2  # bytes of one 16-token block, all layers, bf16
    reqs = poisson_requests(7, rate=200.0, min_tokens=40, max_tokens=400, out_tokens=24, seed=5)
    runner = ShardRunner("cuda", geometry=geometry, tokens_per_block=16, hbm_budget_bytes=3 * 6 * slot,
                         host_budget_bytes=400 * slot, max_sessions=3, policy="recent_only", seed=1)
    try:
        st = runner.run(reqs)
        assert st.tokens == sum(r.out_tokens for r in reqs)
        assert len(st.latencies) == len(reqs)
        assert st.peak_sessions <= 3 and st.host_blocks_peak > 0
        p = runner.pools
        assert p.dev_groups.capacity - p.dev_groups.used == runner.dev_free0
        assert p.host_groups.capacity - p.host_groups.used == runner.host_free0
        out = summarize([st])
        assert out["decode_tokens_per_s"] > 0 and out["kv_gbs"] > 0
        assert _lib.device_status(0) == 0
    finally:
        runner.close()
