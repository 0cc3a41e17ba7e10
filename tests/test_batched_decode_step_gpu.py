"""``batched_decode_step``: PagedModel sessions of different lengths, on shared or private pools,
advanced together by one model forward per token, give each session the tokens it gets decoded alone.

The reference (``batched_decode.py``) requires equal tail lengths and rejects sliding windows; here
three sessions with different prompt lengths (different tails) decode together, most blocks in the
host tier, heavy-hitter and recency policies mixed.  Each session's greedy tokens must match
unpaged HF greedy decoding of its own prompt (tie-aware at fp16 output precision, as for
PagedModel.generate)."""

import pytest
import torch

pytestmark = pytest.mark.gpu

BLOCK = 16 * 1024 * 1024


@pytest.mark.parametrize("kind", ["qwen2", "mistral"])
def test_batched_sessions_match_their_solo_decoding(kind):
    from test_paged_model_gpu import _assert_greedy_match, _hf_greedy, _model

    from pager_hf.batched_decode import batched_decode_step
    from pager_hf.kv_block_store import KVPools
    from pager_hf.paged_model import PagedModel

    model = _model(kind)
    cfg = model.config
    pools = KVPools(num_layers=cfg.num_hidden_layers, kv_heads=cfg.num_key_value_heads, head_dim=64,
                    tokens_per_block=16, dtype=torch.float16, device="cuda", gpu_groups=8, cpu_groups=8)
    g = torch.Generator().manual_seed(9)
    prompts = [torch.randint(0, 2000, (1, n), generator=g).cuda() for n in (150, 97, 33)]
    policies = ["sinks_heavy_hitter", "recent_only", "heavy_hitter"]
    steps = 24
    sessions, tokens = [], []
    for ids, pol in zip(prompts, policies):
        pm = PagedModel(model, vram_budget=2 * BLOCK, ram_budget=1000 * BLOCK, recent_window=1, policy=pol,
                        tokens_per_block=16, pools=pools)
        tokens.append(pm.generate(ids, torch.ones_like(ids), 1))  # prefill + first token
        sessions.append(pm)
    for _ in range(steps):
        logits = batched_decode_step(sessions, [t[-1] for t in tokens], "cuda")
        for t, lg in zip(tokens, logits):
            t.append(int(lg.argmax()))
    for ids, t, s in zip(prompts, tokens, sessions):
        want, ref_logits = _hf_greedy(model, ids, torch.ones_like(ids), steps + 1)
        _assert_greedy_match(t, want[0], ref_logits)
    assert any(s._store.cpu_block_ids() for s in sessions), "no block reached the host tier"
    for s in sessions:
        s.reset()
    pools.close()


def test_scheduler_style_private_pool_sessions_with_a_generate_fallback():
    """Sessions as the reference's serving scheduler makes them (``PagedModel(model, vram_budget=...,
    ram_budget=..., **kwargs)``, each with its own pools), mixed with two sessions on shared pools, all
    advanced by one forward per token (one attention launch per layer per pool); midway one session
    falls back to ``generate(full_sequence, mask, 1)`` for a token, as the scheduler's ``_step_single``
    does, and then rejoins the batch.  Every session's tokens match its solo HF greedy decoding."""
    from test_paged_model_gpu import _assert_greedy_match, _hf_greedy, _model

    from pager_hf.batched_decode import batched_decode_step
    from pager_hf.kv_block_store import KVPools
    from pager_hf.paged_model import PagedModel

    model = _model("qwen2")
    cfg = model.config
    shared = KVPools(num_layers=cfg.num_hidden_layers, kv_heads=cfg.num_key_value_heads, head_dim=64,
                     tokens_per_block=16, dtype=torch.float16, device="cuda", gpu_groups=4, cpu_groups=4)
    g = torch.Generator().manual_seed(11)
    prompts = [torch.randint(0, 2000, (1, n), generator=g).cuda() for n in (121, 64, 90, 47)]
    policies = ["sinks_heavy_hitter", "heavy_hitter", "recent_only", "sinks_heavy_hitter"]
    pools_of = [shared, None, shared, None]
    steps, fallback_step, fallback_row = 22, 9, 1
    sessions, tokens = [], []
    for ids, pol, pools in zip(prompts, policies, pools_of):
        pm = PagedModel(model, vram_budget=2 * BLOCK, ram_budget=1000 * BLOCK, recent_window=1, policy=pol,
                        tokens_per_block=16, pools=pools)
        tokens.append(pm.generate(ids, torch.ones_like(ids), 1))
        sessions.append(pm)
    for step in range(steps):
        rows = list(range(len(sessions)))
        if step == fallback_step:
            seq = torch.cat([prompts[fallback_row], torch.tensor([tokens[fallback_row]], device="cuda")], dim=1)
            tokens[fallback_row] += sessions[fallback_row].generate(seq, torch.ones_like(seq), 1)
            rows.remove(fallback_row)
        logits = batched_decode_step([sessions[r] for r in rows], [tokens[r][-1] for r in rows], "cuda")
        for r, lg in zip(rows, logits):
            tokens[r].append(int(lg.argmax()))
    for ids, t, s in zip(prompts, tokens, sessions):
        want, ref_logits = _hf_greedy(model, ids, torch.ones_like(ids), steps + 1)
        _assert_greedy_match(t, want[0], ref_logits)
        fed = ids.shape[1] + len(t) - 1  # every token but the last generated one is in the cache
        assert s._primed_tokens == fed
        key, value = s._tail_past[0]
        assert key.shape == (1, cfg.num_key_value_heads, fed % 16, 64) and value.shape == key.shape
        assert s._num_blocks == fed // 16
    assert any(s._store.cpu_block_ids() for s in sessions), "no block reached the host tier"
    for s in sessions:
        s.reset()
    shared.close()
    assert batched_decode_step([], [], "cuda") == []


def test_captured_batched_steps_match_eager_batched_steps():
    """Batched steps replayed from a CUDA graph (sessions created with the default ``decode_graphs``)
    give the same tokens and tiers as eager batched steps: two pool groups (three sessions sharing
    pools, one on its own), mixed policies, and a session leaving mid-way (a new capture)."""
    from test_paged_model_gpu import _model

    from pager_hf.batched_decode import batched_decode_step
    from pager_hf.kv_block_store import KVPools
    from pager_hf.paged_model import PagedModel

    model = _model("qwen2")
    cfg = model.config
    g = torch.Generator().manual_seed(21)
    prompts = [torch.randint(0, 2000, (1, n), generator=g).cuda() for n in (120, 61, 35, 90)]
    policies = ["sinks_heavy_hitter", "recent_only", "heavy_hitter", "sinks_heavy_hitter"]
    runs = {}
    for graphs in (False, True):
        pools = KVPools(num_layers=cfg.num_hidden_layers, kv_heads=cfg.num_key_value_heads, head_dim=64,
                        tokens_per_block=16, dtype=torch.float16, device="cuda", gpu_groups=16, cpu_groups=16)
        sessions, tokens = [], []
        for i, (ids, pol) in enumerate(zip(prompts, policies)):
            pm = PagedModel(model, vram_budget=2 * BLOCK, ram_budget=1000 * BLOCK, recent_window=1, policy=pol,
                            tokens_per_block=16, pools=pools if i < 3 else None, decode_graphs=graphs)
            tokens.append(pm.generate(ids, torch.ones_like(ids), 1))
            sessions.append(pm)
        live = list(range(4))
        for step in range(20):
            if step == 12:
                live.remove(1)  # a session leaves the batch
            logits = batched_decode_step([sessions[r] for r in live], [tokens[r][-1] for r in live], "cuda")
            for r, lg in zip(live, logits):
                tokens[r].append(int(lg.argmax()))
        runs[graphs] = (tokens, [sorted(s._store.gpu_block_ids()) for s in sessions])
        for s in sessions:
            s.reset()
        pools.close()
    assert runs[True] == runs[False]
