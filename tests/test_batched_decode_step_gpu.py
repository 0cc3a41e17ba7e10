"""``batched_decode_step``: PagedModel sessions of different lengths, on shared pools, advanced
together by one model forward per token, give each session the tokens it gets decoded alone.

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


def test_batched_decode_step_rejects_sessions_without_shared_pools():
    from test_paged_model_gpu import _model

    from pager_hf.batched_decode import batched_decode_step
    from pager_hf.paged_model import PagedModel

    model = _model("qwen2")
    ids = torch.randint(0, 2000, (1, 40)).cuda()
    pm = PagedModel(model, vram_budget=BLOCK, ram_budget=100 * BLOCK, tokens_per_block=16)
    pm.generate(ids, torch.ones_like(ids), 1)
    with pytest.raises(ValueError, match="pools"):
        batched_decode_step([pm], [1], "cuda")
    assert batched_decode_step([], [], "cuda") == []
