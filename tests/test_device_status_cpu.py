"""Host side of the per-step device status check (no GPU needed): the watch raises
``DeviceStatusError`` with the code and its meaning, and clears the word it read."""

import pytest
import torch


def test_status_watch_raises_once_and_clears():
    from pager_hf import _lib

    w = _lib.StatusWatch.__new__(_lib.StatusWatch)  # host buffer only; enqueue needs a GPU
    w.host = torch.zeros(1, dtype=torch.int32)
    w.check()
    w.host[0] = _lib.STATUS_BAD_SLOT
    with pytest.raises(_lib.DeviceStatusError) as err:
        w.check("PagedModel decode step")
    assert err.value.code == 6
    assert "outside its pool" in str(err.value) and "PagedModel decode step" in str(err.value)
    w.check()  # the code was consumed
    w.host[0] = _lib.STATUS_TIMEOUT
    with pytest.raises(RuntimeError, match="bounded wait"):
        w.check()


def test_status_snapshot_is_exported():
    from pager_hf import _lib

    assert "pager_status_snapshot_async" in _lib.declared_symbols()
    assert hasattr(_lib.load_library(), "pager_status_snapshot_async")
