"""Property-based differential test of the C++ block pager against the oracle.

Hypothesis draws the constructor arguments (any of the four policy names or an
unknown one, byte budgets that need not be whole 16 MiB blocks, recent window,
rebalance interval, non-negative margins) and a sequence of ``on_step`` /
``force_rebalance`` calls with token indices that may jump or go back and
attention vectors of any length (shorter or longer than the block list, ties,
zeros).  After every call both implementations must agree on tiers, VRAM ids,
f32 scores and metrics -- the state ``pager/src/core.rs:56-555`` defines.

Negative margins and NaN attention stay out: with them the reference's
hysteresis loops (``core.rs:368-400``, ``:450-477``) need not end, which the
C++ library bounds on purpose.
"""

import numpy as np
import pytest

hyp = pytest.importorskip("hypothesis")
from hypothesis import given, settings, strategies as st  # noqa: E402

import pager  # noqa: E402
from oracle import pager_core_oracle as orc  # noqa: E402

BLOCK = 16 * 1024 * 1024

_policy = st.sampled_from(["recent_only", "sinks_recent", "heavy_hitter", "sinks_heavy_hitter", "bogus"])
_budget = st.one_of(st.integers(0, 12).map(lambda n: n * BLOCK), st.integers(0, 12 * BLOCK))
_margin = st.one_of(st.just(0.0), st.floats(0.0, 1.0, width=32))
_value = st.one_of(st.sampled_from([0.0, 0.25, 0.5, 1.0]), st.floats(0.0, 1e3, width=32, allow_nan=False))
_call = st.one_of(
    st.tuples(st.just("step"), st.integers(0, 48), st.integers(0, 2**32 - 1), st.lists(_value, max_size=40)),
    st.tuples(st.just("rebalance"), st.integers(0, 48)),
)


def _metrics(p):
    if isinstance(p, orc.Pager):
        return dict(p.m)
    m = p.metrics()
    return {k: getattr(m, k) for k in ("tokens", "vram_peak", "ram_peak", "swap_vram_ram", "swap_ram_ssd",
                                       "attention_mass_total", "attention_mass_vram")}


@settings(max_examples=300, deadline=None, derandomize=True)
@given(policy=_policy, vram=_budget, ram=_budget, recent=st.integers(0, 10), interval=st.integers(1, 6),
       pm=_margin, rm=_margin, calls=st.lists(_call, max_size=50))
def test_cpp_matches_oracle_on_random_call_sequences(policy, vram, ram, recent, interval, pm, rm, calls):
    cpp = pager.PyPager(vram, ram, recent, interval, pm, rm, policy)
    ref = orc.Pager(vram, ram, recent, interval, pm, rm, policy)
    for i, call in enumerate(calls):
        if call[0] == "step":
            _, tok, layer, att = call
            cpp.on_step(tok, layer, att)
            ref.on_step(tok, layer, att)
        else:
            cpp.force_rebalance(call[1])
            ref.force_rebalance(call[1])
        assert cpp.tiers() == ref.tiers(), (i, call)
        assert cpp.vram_block_ids() == ref.vram_block_ids(), (i, call)
        assert np.array_equal(np.array(cpp.scores(), np.float32), np.array(ref.scores(), np.float32)), (i, call)
        assert _metrics(cpp) == _metrics(ref), (i, call)
        assert len(cpp.vram_block_ids()) <= vram // BLOCK
