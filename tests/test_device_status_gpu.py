"""A decode step whose kernels flag a fault raises instead of handing out tokens.

The decode kernels never dereference a block-table entry that names a slot outside its pool: they
skip the block and set the device status word to 6 (a timed-out bounded wait sets 5).  The product
paths read that word once per step, at the synchronisation the step already has, and raise
``DeviceStatusError``: ``PagedModel.generate`` (captured and eager steps), ``batched_decode_step``,
``BatchedDecodeAttention.finish`` and, per request, the serving sweep (as the reference's scheduler
fails a request whose step raised, ``pager_hf/serving/scheduler.py:520-524``).

The fault is planted on the host: a live session's block map is pointed at a slot past the end of
its pool.  The kernels' own bounds checks turn it into status 6, so no GPU access goes out of bounds.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

BLOCK = 16 * 1024 * 1024


def _model():
    from transformers import Qwen2Config, Qwen2ForCausalLM

    torch.manual_seed(0)
    cfg = Qwen2Config(hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=64, vocab_size=1000, max_position_embeddings=4096,
                      rope_theta=1e6, initializer_range=0.02)
    return Qwen2ForCausalLM(cfg).to(device="cuda", dtype=torch.float16).eval()


@pytest.mark.parametrize("graphs", [True, False])
def test_generate_raises_on_a_block_outside_the_pool(graphs):
    from pager_hf import _lib
    from pager_hf.paged_model import PagedModel

    model = _model()
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, 1000, (1, 100), generator=g).cuda()
    pm = PagedModel(model, vram_budget=64 * BLOCK, ram_budget=64 * BLOCK, recent_window=63, policy="recent_only",
                    tokens_per_block=16, decode_graphs=graphs)
    first = pm.generate(ids, torch.ones_like(ids), 4)
    _lib.device_status(0)
    store = pm._store
    good = store._dev_group[0]
    store._dev_group[0] = pm._pools.dev_groups.capacity + 7  # a slot past the device pool's end
    try:
        ids2 = torch.cat([ids, torch.tensor([first], device="cuda")], dim=1)
        with pytest.raises(_lib.DeviceStatusError) as err:
            pm.generate(ids2, torch.ones_like(ids2), 3)
        assert err.value.code == _lib.STATUS_BAD_SLOT
    finally:
        store._dev_group[0] = good
    assert _lib.device_status(0) == 0  # the step's snapshot already cleared the word
    pm.reset()
    assert len(pm.generate(ids, torch.ones_like(ids), 3)) == 3  # the context stays usable


def test_batched_decode_step_raises_on_a_block_outside_the_pool():
    from pager_hf import _lib
    from pager_hf import batched_decode as bd
    from pager_hf.batched_decode import batched_decode_step
    from pager_hf.kv_block_store import KVPools
    from pager_hf.paged_model import PagedModel

    model = _model()
    a = model.config
    pools = KVPools(num_layers=a.num_hidden_layers, kv_heads=a.num_key_value_heads, head_dim=64, tokens_per_block=16,
                    dtype=torch.float16, device=torch.device("cuda", 0), gpu_groups=32, cpu_groups=32)
    g = torch.Generator().manual_seed(1)
    sessions, nxt = [], []
    for n in (70, 90):
        pm = PagedModel(model, vram_budget=64 * BLOCK, ram_budget=64 * BLOCK, recent_window=63, policy="recent_only",
                        tokens_per_block=16, pools=pools)
        ids = torch.randint(0, 1000, (1, n), generator=g).cuda()
        nxt.append(pm.generate(ids, torch.ones_like(ids), 1)[0])
        sessions.append(pm)
    _lib.device_status(0)
    store = sessions[1]._store
    good = store._dev_group[1]
    store._dev_group[1] = pools.dev_groups.capacity + 3
    try:
        with pytest.raises(_lib.DeviceStatusError) as err:
            batched_decode_step(sessions, nxt, "cuda")
        assert err.value.code == _lib.STATUS_BAD_SLOT
    finally:
        store._dev_group[1] = good
    out = batched_decode_step(sessions, nxt, "cuda")  # a clean step goes through
    assert len(out) == 2
    for s in sessions:
        s.reset()
    bd._BATCHED_GRAPH.clear()  # the cached step graph references the pools
    pools.close()


def test_serving_sweep_fails_the_requests_of_a_faulted_step(monkeypatch):
    """A step whose kernels flagged a fault ends the requests it served with an error (the
    reference's ``req.error``), and the sweep goes on with the next arrivals.  The fault is the
    host-side error of a faked ``finish``: nothing is planted on the GPU."""
    from pager_hf import _lib
    from pager_hf import batched_decode as bd
    from pager_hf.serving_sweep import Request, ShardRunner

    real_finish = bd.BatchedDecodeAttention.finish
    calls = {"n": 0}

    def finish(self, apply_tiers=True):
        calls["n"] += 1
        if calls["n"] == 3:
            torch.cuda.synchronize()
            raise _lib.DeviceStatusError(_lib.STATUS_TIMEOUT, "batched decode attention step")
        return real_finish(self, apply_tiers)

    monkeypatch.setattr(bd.BatchedDecodeAttention, "finish", finish)
    geo = dict(layers=2, hq=8, hkv=2, d=64)
    runner = ShardRunner("cuda:0", geometry=geo, tokens_per_block=16, hbm_budget_bytes=64e6, host_budget_bytes=64e6,
                         max_sessions=4, dtype=torch.float16)
    try:
        # request 2 arrives long after the faulted third step of requests 0 and 1
        reqs = [Request(0, 0.0, 100, 6), Request(1, 0.0, 70, 6), Request(2, 4.0, 90, 4)]
        st = runner.run(reqs)
        assert runner.pools.dev_groups.used == 0  # every session, failed or finished, gave its slots back
    finally:
        runner.close()
    failed = sorted(e["rid"] for e in st.errors)
    assert failed == [0, 1], st.errors
    assert all("device status 5" in e["error"] for e in st.errors)
    assert len(st.latencies) == 1  # request 2 arrived later and completed
