"""The pool-backed ``KVBlockStore`` on the GPU.

The first tests are the reference's own (``tests/test_kv_block_store.py``):
RAM budget error / warning / no-budget, resident-byte accounting across moves,
and the row-tagged beam reorder on both tiers.  The rest check what the pools
add: tier moves preserve data, pool growth keeps every block, the block table
drives ``paged_decode_attention`` to the oracle's result with the tiers a
``pager.PyPager`` picked, and per-layer registration equals ``put_gpu``.
"""

import logging

import numpy as np
import pytest
import torch

from oracle import streaming_attention_oracle as orc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def kvs():
    from pager_hf import kv_block_store

    return kv_block_store


def make_block(*, num_layers=2, batch=1, tokens_per_block=16, kv_heads=2, head_dim=64):
    shape = (num_layers, batch, tokens_per_block, kv_heads, head_dim)
    return (torch.zeros(shape, dtype=torch.float16, device="cuda"),
            torch.zeros(shape, dtype=torch.float16, device="cuda"))


def test_offload_to_cpu_raises_when_ram_budget_would_be_exceeded(kvs):
    store = kvs.KVBlockStore(tokens_per_block=16, ram_budget_bytes=1000)
    store.put_gpu(0, *make_block())
    with pytest.raises(RuntimeError, match="ram_budget exceeded"):
        store.ensure_cpu(0)
    assert store.has_gpu(0)
    assert not store.has_cpu(0)
    assert store.resident_cpu_bytes() == 0
    store.close()


def test_offload_to_cpu_succeeds_within_ram_budget(kvs):
    store = kvs.KVBlockStore(tokens_per_block=16, ram_budget_bytes=1_000_000_000)
    store.put_gpu(0, *make_block())
    store.ensure_cpu(0)
    assert store.has_cpu(0)
    assert not store.has_gpu(0)
    store.close()


def test_offload_to_cpu_logs_error_when_ram_budget_exceeded(kvs, caplog):
    store = kvs.KVBlockStore(tokens_per_block=16, ram_budget_bytes=1000)
    store.put_gpu(0, *make_block())
    with caplog.at_level(logging.ERROR, logger="pager_hf.kv_block_store"):
        with pytest.raises(RuntimeError, match="ram_budget exceeded"):
            store.ensure_cpu(0)
    assert any(r.levelno == logging.ERROR and "ram_budget exceeded" in r.message for r in caplog.records)
    store.close()


def test_offload_to_cpu_warns_when_approaching_ram_budget(kvs, caplog):
    key, value = make_block()
    store = kvs.KVBlockStore(tokens_per_block=16, ram_budget_bytes=int(kvs.kv_nbytes(key, value) / 0.82))
    store.put_gpu(0, key, value)
    with caplog.at_level(logging.WARNING, logger="pager_hf.kv_block_store"):
        store.ensure_cpu(0)
    assert store.has_cpu(0)
    assert any(r.levelno == logging.WARNING and "ram_budget usage" in r.message for r in caplog.records)
    store.close()


def test_offload_to_cpu_ignores_ram_budget_when_unset(kvs):
    store = kvs.KVBlockStore(tokens_per_block=16)
    store.put_gpu(0, *make_block())
    store.ensure_cpu(0)
    assert store.has_cpu(0)
    store.close()


def test_resident_bytes_stay_correct_across_many_moves(kvs):
    """Blocks of different lengths (here 8..16 tokens: the pool holds at most tokens_per_block)."""
    store = kvs.KVBlockStore(tokens_per_block=16, gpu_capacity_blocks=2, cpu_capacity_blocks=1)
    for block_id in range(10):
        store.put_gpu(block_id, *make_block(tokens_per_block=8 + block_id % 9))
    for block_id in range(0, 10, 2):
        store.offload_to_cpu(block_id)
    for block_id in range(0, 10, 4):
        store.load_to_gpu(block_id, torch.device("cuda"))
    gpu = sum(kvs.kv_nbytes(k, v) for k, v in store.gpu_blocks.values())
    cpu = sum(kvs.kv_nbytes(k, v) for k, v in store.cpu_blocks.values())
    assert store.resident_gpu_bytes() == gpu
    assert store.resident_cpu_bytes() == cpu
    s = store.summary()
    assert s["gpu_to_cpu_copies"] == 5 and s["cpu_to_gpu_copies"] == 3
    assert s["gpu_to_cpu_sec"] > 0 and s["cpu_to_gpu_sec"] > 0
    store.close()


def make_row_tagged_block(*, num_layers=2, batch=4, tokens_per_block=16, kv_heads=2, head_dim=8):
    shape = (num_layers, batch, tokens_per_block, kv_heads, head_dim)
    key = torch.zeros(shape, dtype=torch.float16, device="cuda")
    value = torch.zeros(shape, dtype=torch.float16, device="cuda")
    for row in range(batch):
        key[:, row] = row
        value[:, row] = row + 1000
    return key, value


def test_reorder_batch_rows_reorders_duplicates_and_drops_on_both_tiers(kvs):
    store = kvs.KVBlockStore(tokens_per_block=16)
    store.put_gpu(0, *make_row_tagged_block())
    store.put_gpu(1, *make_row_tagged_block())
    store.offload_to_cpu(1)
    new_rows = [2, 2, 1, 3]
    store.reorder_batch_rows(new_rows)
    k, v = store.get_gpu(0)
    assert store.has_gpu(0)
    for new, old in enumerate(new_rows):
        assert torch.all(k[:, new] == old) and torch.all(v[:, new] == old + 1000)
    assert store.has_cpu(1)
    k, v = store.cpu_blocks[1]
    for new, old in enumerate(new_rows):
        assert torch.all(k[:, new] == old) and torch.all(v[:, new] == old + 1000)
    store.close()


def test_reorder_to_a_different_row_count_relays_both_pools(kvs):
    store = kvs.KVBlockStore(tokens_per_block=16)
    store.put_gpu(0, *make_row_tagged_block())
    store.put_gpu(1, *make_row_tagged_block())
    store.offload_to_cpu(0)
    before = store.resident_gpu_bytes() + store.resident_cpu_bytes()
    store.reorder_batch_rows([3, 0])
    assert store.batch == 2
    for bid in (0, 1):
        k, v = store.get_any(bid)
        assert k.shape[1] == 2
        assert torch.all(k[:, 0] == 3) and torch.all(k[:, 1] == 0) and torch.all(v[:, 0] == 1003)
    assert store.resident_gpu_bytes() + store.resident_cpu_bytes() == before // 2
    store.close()


def _rand_block(g, L, B, t, H, D, dtype):
    return (torch.randn(L, B, t, H, D, generator=g).to(dtype).cuda(),
            torch.randn(L, B, t, H, D, generator=g).to(dtype).cuda())


def test_moves_and_growth_preserve_every_block(kvs):
    g = torch.Generator().manual_seed(5)
    store = kvs.KVBlockStore(tokens_per_block=16, gpu_capacity_blocks=1, cpu_capacity_blocks=1)
    blocks = {i: _rand_block(g, 3, 2, 16, 2, 32, torch.bfloat16) for i in range(9)}
    for i, (k, v) in blocks.items():
        store.put_gpu(i, k, v)
    v0 = store.version
    moved = store.apply_tiers([0, 1, 1, 0, 2, 1, 0, 1], "cuda")  # block 8 past the end -> CPU
    assert moved == {"to_gpu": [], "to_cpu": [1, 2, 4, 5, 7, 8]}
    assert store.version > v0  # the host pool grew
    moved = store.apply_tiers([1, 0, 0, 0, 0, 0, 0, 0, 0], "cuda", sync=False)
    assert moved == {"to_gpu": [1, 2, 4, 5, 7, 8], "to_cpu": [0]}
    store.synchronize()
    for i, (k, v) in blocks.items():
        gk, gv = store.get_any(i)
        assert torch.equal(gk.cpu(), k.cpu()) and torch.equal(gv.cpu(), v.cpu()), i
    store.close()


def test_put_gpu_layers_equals_put_gpu(kvs):
    g = torch.Generator().manual_seed(6)
    k, v = _rand_block(g, 4, 3, 16, 2, 64, torch.float16)
    a = kvs.KVBlockStore(tokens_per_block=16)
    b = kvs.KVBlockStore(tokens_per_block=16)
    a.put_gpu(7, k, v)
    # HF per-layer layout [batch, kv_heads, block_len, head_dim]
    b.put_gpu_layers(7, [k[i].permute(0, 2, 1, 3) for i in range(4)], [v[i].permute(0, 2, 1, 3) for i in range(4)])
    assert torch.equal(a.dev_pool[:3], b.dev_pool[:3])
    assert a.resident_gpu_bytes() == b.resident_gpu_bytes()
    a.close()
    b.close()


@pytest.mark.parametrize("policy", ["sinks_heavy_hitter", "recent_only"])
def test_block_table_drives_the_decode_op_to_the_oracle(kvs, policy):
    """Blocks placed by a PyPager decision, decoded straight from the two pools."""
    import pager
    from pager_hf import streaming_attention as sa

    g = torch.Generator().manual_seed(7)
    L, B, Hq, Hkv, D, tpb, nb, tail = 2, 3, 16, 4, 64, 16, 11, 5
    dt = torch.float16
    store = kvs.KVBlockStore(tokens_per_block=tpb)
    blocks = [_rand_block(g, L, B, tpb, Hkv, D, dt) for _ in range(nb)]
    for i, (k, v) in enumerate(blocks):
        store.put_gpu(i, k, v)
    pg = pager.PyPager(4 * 16 * 1024 * 1024, 100 * 16 * 1024 * 1024, 2, 1, 0.05, 0.2, policy)
    rng = np.random.default_rng(0)
    for _ in range(3):
        pg.on_step(nb - 1, 0, rng.dirichlet(np.ones(nb)).tolist())
    store.apply_tiers(pg.tiers(), "cuda")
    assert 0 < len(store.gpu_block_ids()) < nb and store.cpu_block_ids()
    table = store.block_table(range(nb))
    assert int((table & 0x40000000).ne(0).sum()) == B * len(store.cpu_block_ids())

    q = torch.randn(B, Hq, D, generator=g).to(dt).cuda()
    tk = torch.randn(B, Hkv, tail, D, generator=g).to(dt).cuda()
    tv = torch.randn(B, Hkv, tail, D, generator=g).to(dt).cuda()
    layer = 1
    mass = torch.zeros(B, nb, device="cuda")
    out = sa.paged_decode_attention(
        q, table, torch.full((B,), nb, dtype=torch.int32, device="cuda"), dev_pool=store.dev_pool,
        host_pool=store.host_pool.tensor, num_layers=L, layer=layer, tokens_per_block=tpb,
        max_row_tokens=nb * tpb + tail, tail_k=tk, tail_v=tv,
        tail_len=torch.full((B,), tail, dtype=torch.int32, device="cuda"), mass_accum=mass, mass_mode="row_mean")
    torch.cuda.synchronize()
    for b in range(B):
        k = torch.cat([blk[0][layer, b].permute(1, 0, 2) for blk in blocks], dim=1)[None].float().cpu().numpy()
        v = torch.cat([blk[1][layer, b].permute(1, 0, 2) for blk in blocks], dim=1)[None].float().cpu().numpy()
        ref_out, ref_mass, _, _ = orc.two_pass_decode(
            q[b:b + 1].float().cpu().numpy(), k, v, tk[b:b + 1].float().cpu().numpy(),
            tv[b:b + 1].float().cpu().numpy(), nb, tpb, nb, v_dtype="f16", out_dtype="f16")
        np.testing.assert_allclose(out[b].float().cpu().numpy(), ref_out[0], rtol=0, atol=2e-3)
        np.testing.assert_allclose(mass[b].cpu().numpy(), ref_mass[0].mean(0), rtol=1e-4, atol=1e-6)
    store.close()


def test_reference_kv_utils_round_trip_through_the_pool_store(kvs):
    """kv_utils.real_past_to_blocks -> pool-backed store (through the host tier and back) ->
    kv_utils.reconstruct_past_from_store gives the cache back exactly."""
    from pager_hf.kv_utils import real_past_to_blocks, reconstruct_past_from_store, split_full_blocks_and_tail

    g = torch.Generator().manual_seed(8)
    past = [(torch.randn(2, 4, 70, 32, generator=g).half().cuda(), torch.randn(2, 4, 70, 32, generator=g).half().cuda())
            for _ in range(3)]
    full, tail, n = split_full_blocks_and_tail(past, tokens_per_block=16)
    store = kvs.KVBlockStore(tokens_per_block=16, gpu_capacity_blocks=2, cpu_capacity_blocks=2)
    for j, (k, v) in enumerate(real_past_to_blocks(full, tokens_per_block=16)):
        store.put_gpu(j, k, v)
    store.apply_tiers([1, 0, 1, 0], "cuda")
    store.apply_tiers([0, 0, 0, 0], "cuda")
    rec = reconstruct_past_from_store(store=store, num_layers=3, num_blocks=n // 16, tail_past=tail)
    for layer in range(3):
        assert torch.equal(rec[layer][0], past[layer][0]) and torch.equal(rec[layer][1], past[layer][1])
    store.close()
