"""``pager_hf.kv_utils``: the reference's own tests (``tests/test_kv_utils.py``), ported, plus the
block-attention reduction and the installed transformers' cache form."""

import pytest
import torch

from pager_hf.kv_utils import (extract_single_block_from_past, get_legacy_past_key_values, real_past_to_blocks,
                               reconstruct_past_from_store, split_full_blocks_and_tail, token_attention_to_blocks)


class FakeBlockStore:
    """What reconstruct_past_from_store needs of a store: get_gpu(block_id) -> (key, value)."""

    def __init__(self):
        self._blocks = {}

    def put(self, block_id, key, value):
        self._blocks[block_id] = (key, value)

    def get_gpu(self, block_id):
        return self._blocks[block_id]


def make_fake_past(*, num_layers, batch, kv_heads, seq_len, head_dim, seed=0):
    g = torch.Generator().manual_seed(seed)
    return [(torch.randn(batch, kv_heads, seq_len, head_dim, generator=g),
             torch.randn(batch, kv_heads, seq_len, head_dim, generator=g)) for _ in range(num_layers)]


def test_split_full_blocks_and_tail_splits_at_block_boundary():
    past = make_fake_past(num_layers=2, batch=1, kv_heads=2, seq_len=35, head_dim=4)
    full_past, tail_past, full_tokens = split_full_blocks_and_tail(past, tokens_per_block=16)
    assert full_tokens == 32
    assert full_past[0][0].shape[2] == 32
    assert tail_past[0][0].shape[2] == 3


def test_split_full_blocks_and_tail_handles_exact_multiple():
    past = make_fake_past(num_layers=1, batch=1, kv_heads=1, seq_len=32, head_dim=2)
    full_past, tail_past, full_tokens = split_full_blocks_and_tail(past, tokens_per_block=16)
    assert full_tokens == 32
    assert tail_past[0][0].shape[2] == 0


@pytest.mark.parametrize("batch", [1, 3])
def test_extract_and_reconstruct_round_trip(batch):
    num_layers, kv_heads, head_dim, tpb = 3, 2, 4, 16
    past = make_fake_past(num_layers=num_layers, batch=batch, kv_heads=kv_heads, seq_len=4 * tpb, head_dim=head_dim)
    blocks = real_past_to_blocks(past, tokens_per_block=tpb)
    assert len(blocks) == 4
    for key, value in blocks:
        assert key.shape == value.shape == (num_layers, batch, tpb, kv_heads, head_dim)
    store = FakeBlockStore()
    for j, (k, v) in enumerate(blocks):
        store.put(j, k, v)
    rec = reconstruct_past_from_store(store=store, num_layers=num_layers, num_blocks=4)
    assert len(rec) == num_layers
    for layer in range(num_layers):
        assert torch.equal(rec[layer][0], past[layer][0]) and torch.equal(rec[layer][1], past[layer][1])


def test_extract_single_block_from_past_selects_the_right_token_range():
    past = make_fake_past(num_layers=1, batch=1, kv_heads=1, seq_len=32, head_dim=2)
    key, value = extract_single_block_from_past(past, block_id=1, tokens_per_block=16)
    assert torch.equal(key[0], past[0][0][:, :, 16:32, :].permute(0, 2, 1, 3))
    assert torch.equal(value[0], past[0][1][:, :, 16:32, :].permute(0, 2, 1, 3))


def test_reconstruct_past_from_store_appends_tail_past():
    num_layers, kv_heads, head_dim, tpb = 2, 2, 4, 16
    past = make_fake_past(num_layers=num_layers, batch=1, kv_heads=kv_heads, seq_len=2 * tpb, head_dim=head_dim)
    store = FakeBlockStore()
    for j, (k, v) in enumerate(real_past_to_blocks(past, tokens_per_block=tpb)):
        store.put(j, k, v)
    tail = [(torch.ones(1, kv_heads, 3, head_dim), torch.ones(1, kv_heads, 3, head_dim)) for _ in range(num_layers)]
    rec = reconstruct_past_from_store(store=store, num_layers=num_layers, num_blocks=2, tail_past=tail)
    for layer in range(num_layers):
        assert rec[layer][0].shape == (1, kv_heads, 2 * tpb + 3, head_dim)
        assert torch.equal(rec[layer][0][:, :, :2 * tpb], past[layer][0])
        assert torch.equal(rec[layer][0][:, :, 2 * tpb:], tail[layer][0])
        assert torch.equal(rec[layer][1][:, :, 2 * tpb:], tail[layer][1])


def test_reconstruct_past_from_store_with_zero_blocks_uses_tail_only():
    tail = [(torch.randn(1, 2, 5, 4), torch.randn(1, 2, 5, 4)) for _ in range(2)]
    rec = reconstruct_past_from_store(store=FakeBlockStore(), num_layers=2, num_blocks=0, tail_past=tail)
    for layer in range(2):
        assert torch.equal(rec[layer][0], tail[layer][0]) and torch.equal(rec[layer][1], tail[layer][1])


def test_reconstruct_past_from_store_with_zero_blocks_and_no_tail_raises():
    with pytest.raises(ValueError, match="no blocks and no tail"):
        reconstruct_past_from_store(store=FakeBlockStore(), num_layers=1, num_blocks=0, tail_past=None)


class _Outputs:
    def __init__(self, past):
        self.past_key_values = past


class _FakeCache:
    def __init__(self, past):
        self.key_cache = [k for k, _ in past]
        self.value_cache = [v for _, v in past]


def test_get_legacy_past_key_values_accepts_the_tuple_and_cache_object_forms():
    past = make_fake_past(num_layers=2, batch=1, kv_heads=1, seq_len=4, head_dim=2)
    for outputs in (_Outputs(tuple(past)), _Outputs(_FakeCache(past))):
        result = get_legacy_past_key_values(outputs)
        assert len(result) == 2 and torch.equal(result[0][0], past[0][0]) and torch.equal(result[1][1], past[1][1])


def test_get_legacy_past_key_values_accepts_the_installed_dynamic_cache():
    from transformers import DynamicCache

    past = make_fake_past(num_layers=2, batch=1, kv_heads=2, seq_len=6, head_dim=4)
    cache = DynamicCache()
    for layer, (k, v) in enumerate(past):
        cache.update(k, v, layer)
    result = get_legacy_past_key_values(_Outputs(cache))
    assert len(result) == 2 and torch.equal(result[1][0], past[1][0]) and torch.equal(result[0][1], past[0][1])


def test_get_legacy_past_key_values_rejects_missing_cache():
    with pytest.raises(RuntimeError):
        get_legacy_past_key_values(_Outputs(None))


def test_token_attention_to_blocks_sums_per_block_and_normalises():
    attn = torch.tensor([0.1, 0.2, 0.3, 0.4, 0.0, 0.0], dtype=torch.float32)
    out = token_attention_to_blocks(attn, tokens_per_block=2, num_blocks=3)
    ref = [0.0, 0.0, 0.0]
    for t in range(6):  # the reference's own loop, in double precision
        ref[t // 2] += float(attn[t].item())
    total = sum(ref)
    assert out == [x / total for x in ref]
    assert token_attention_to_blocks(torch.zeros(4), tokens_per_block=2, num_blocks=2) == [0.5, 0.5]
    with pytest.raises(IndexError):
        token_attention_to_blocks(torch.ones(3), tokens_per_block=2, num_blocks=2)
