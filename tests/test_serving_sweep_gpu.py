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


@pytest.mark.parametrize("policy,rule", [("recent_only", "running"), ("sinks_heavy_hitter", "final")])
def test_sweep_attention_matches_the_reference_algorithm(monkeypatch, policy, rule):
    """What the sweep computes, not just that it finishes: during a small sweep (sessions joining and
    leaving, blocks moving between tiers, tails rolling into blocks), every layer of every fifth step
    is recomputed with the reference's algorithm on the KV gathered from the pools by the step's own
    block table -- its cross-session one-pass sequence for recent_only, its two-pass one for the
    heavy-hitter policy (batched_decode.py:236-285) -- and the outputs (within 2e-3 or one output
    ulp, at most 6 % different after rounding) and the per-row block mass (1e-4 relative) must agree."""
    import torch
    from model_parity import reference_attention

    from pager_hf import batched_decode as bd
    from pager_hf.serving_sweep import ShardRunner, poisson_requests

    orig = bd.BatchedDecodeAttention.layer
    seen = {"step": 0, "checks": []}

    def layer(self, layer_idx, q, k_new, v_new, out=None):
        before = None if self.mass is None else self.mass.clone()
        res = orig(self, layer_idx, q, k_new, v_new, out)
        if layer_idx == 0:
            seen["step"] += 1
        if seen["step"] % 5 != 1:
            return res
        torch.cuda.synchronize()
        ref, mass = reference_attention(self.plan, q.contiguous(), layer_idx, rule)
        got, want = res.float(), ref.float()
        units = float(((got - want).abs() / torch.clamp(torch.finfo(res.dtype).eps * want.abs(), min=2e-3)).max())
        differ = float((got != want).float().mean())
        mass_err = 0.0
        if before is not None:
            delta = self.mass - before
            ref_delta = mass.mean(dim=1)[:, : delta.shape[1]]
            mass_err = float(((delta - ref_delta).abs() / ref_delta.abs().max().clamp(min=1e-30)).max())
        seen["checks"].append((units, differ, mass_err, len(self.sessions)))
        return res

    monkeypatch.setattr(bd.BatchedDecodeAttention, "layer", layer)
    geometry = dict(layers=2, hq=8, hkv=2, d=64)
    slot = 2 * 2 * 2 * 16 * 64 * 2
    reqs = poisson_requests(6, rate=100.0, min_tokens=60, max_tokens=500, out_tokens=30, seed=9)
    runner = ShardRunner("cuda", geometry=geometry, tokens_per_block=16, hbm_budget_bytes=3 * 6 * slot,
                         host_budget_bytes=400 * slot, max_sessions=3, policy=policy, seed=2, dtype=torch.bfloat16)
    try:
        st = runner.run(reqs)
    finally:
        runner.close()
    assert st.tokens == sum(r.out_tokens for r in reqs) and not st.errors
    assert len(seen["checks"]) >= 8 and max(c[3] for c in seen["checks"]) > 1
    print(f"{policy}: {len(seen['checks'])} layer calls checked; worst {max(c[0] for c in seen['checks']):.2f} x "
          f"max(2e-3, 1 ulp), worst differing fraction {max(c[1] for c in seen['checks']):.4f}, "
          f"mass rel {max(c[2] for c in seen['checks']):.2e}")
    assert max(c[0] for c in seen["checks"]) <= 1.0
    assert max(c[1] for c in seen["checks"]) <= 0.06
    assert max(c[2] for c in seen["checks"]) <= 1e-4
