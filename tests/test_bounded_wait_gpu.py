"""Failure detection without a GPU fault: a wait that nothing satisfies gives up and reports.

Every wait in the decode kernels is bounded; on expiry the kernel sets the
device status word (5, timeout), stops and returns, so a stuck copy cannot hang
the GPU.  Here one thread waits on an mbarrier that nothing ever arrives on,
with a 2 ms limit: the call returns, the host reads status 5 (and reading it
clears it), the wait took at least the limit, and the context stays usable for
a regular decode call afterwards.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_expired_wait_reports_timeout_and_the_context_stays_usable():
    from oracle import streaming_attention_oracle as orc
    from pager_hf import _lib
    from pager_hf import streaming_attention as sa

    lib = _lib.lib()
    _lib.device_status(0)  # clear whatever an earlier test left
    waited = ctypes.c_ulonglong()
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.pager_selftest_bounded_wait(2_000_000, ctypes.byref(waited), stream) == 0
    assert _lib.device_status(0) == 5
    assert _lib.device_status(0) == 0  # reading the status clears it
    assert 2_000_000 <= waited.value < 1_000_000_000
    with pytest.raises(ValueError):
        _lib.check(lib.pager_selftest_bounded_wait(10**9, None, stream))  # above the 100 ms cap

    g = torch.Generator().manual_seed(3)
    q = torch.randn(2, 8, 64, generator=g).half()
    k = torch.randn(2, 2, 96, 64, generator=g).half()
    v = torch.randn(2, 2, 96, 64, generator=g).half()
    m, l, acc = sa.streaming_attention_state_init(2, 8, 64, "cuda")
    sa.streaming_attention_step(q.cuda(), k.cuda(), v.cuda(), m, l, acc)
    out = sa.streaming_attention_finalize(acc, l, torch.float16)
    mo, lo, ao = orc.state_init(2, 8, 64)
    orc.step(q.float().numpy(), k.float().numpy(), v.float().numpy(), mo, lo, ao, v_dtype="f16")
    np.testing.assert_allclose(out.float().cpu().numpy(), orc.finalize(ao, lo, "f16"), rtol=0, atol=2e-3)
    assert _lib.device_status(0) == 0
