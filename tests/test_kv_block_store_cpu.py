"""Host-side logic of the pool-backed ``KVBlockStore`` (no GPU needed)."""

import pytest
import torch

from pager_hf.kv_block_store import KVBlockStore, SlotGroups, kv_nbytes, tensor_nbytes


def test_slot_groups_hand_out_the_lowest_free_group_and_grow():
    s = SlotGroups(3)
    assert [s.take(), s.take()] == [0, 1]
    s.give(0)
    assert s.take() == 0
    assert s.take() == 2
    assert s.take() is None
    s.grow(5)
    assert [s.take(), s.take(), s.take()] == [3, 4, None]
    assert s.used == 5
    with pytest.raises(ValueError):
        s.give(7)
    s.give(4)
    with pytest.raises(ValueError):
        s.give(4)
    with pytest.raises(ValueError):
        s.grow(2)


def test_put_gpu_rejects_host_tensors_like_the_reference():
    store = KVBlockStore(tokens_per_block=16)
    k = torch.zeros(2, 1, 16, 2, 8)
    with pytest.raises(ValueError, match="put_gpu expects CUDA tensors"):
        store.put_gpu(0, k, k)


def test_empty_store_queries():
    store = KVBlockStore(tokens_per_block=16)
    assert store.gpu_block_ids() == [] and store.cpu_block_ids() == []
    assert not store.has_gpu(0) and not store.has_cpu(0)
    assert len(store.gpu_blocks) == 0 and 0 not in store.cpu_blocks
    with pytest.raises(KeyError):
        store.get_any(0)
    with pytest.raises(KeyError):
        store.get_gpu(0)
    with pytest.raises(KeyError):
        store.offload_to_cpu(0)
    with pytest.raises(KeyError):
        store.load_to_gpu(0, "cuda")
    with pytest.raises(ValueError):
        store.block_table()
    assert store.summary()["gpu_blocks"] == 0
    assert store.apply_tiers([0, 1], "cuda") == {"to_gpu": [], "to_cpu": []}


def test_byte_helpers():
    k = torch.zeros(2, 3, 4, dtype=torch.float16)
    assert tensor_nbytes(k) == 48
    assert kv_nbytes(k, k) == 96
