"""The block-placement pager (``libpager_core.so`` via the ``pager`` module).

* the reference's own unit tests (``pager/src/core.rs:559-705``), ported, run
  against both the C++ library and the Python oracle;
* the reference's CI smoke call (``.github/workflows/ci.yml:81``);
* pyo3-style argument errors of ``PyPager`` (``lib.rs:16-46``);
* seeded differential runs: identical call sequences must give identical tiers,
  VRAM ids, metrics and f32 scores in the C++ library and the oracle, for every
  policy, budget and margin mix below.
"""

import numpy as np
import pytest

import pager
from oracle import pager_core_oracle as orc

BLOCK = 16 * 1024 * 1024
POLICIES = ["recent_only", "sinks_recent", "heavy_hitter", "sinks_heavy_hitter"]


def _make(kind, vram_blocks, ram_blocks, recent, policy, interval=4):
    # core.rs:565-575 make_pager: promote_margin 0.05, ram_promote_margin 0.20
    cls = pager.PyPager if kind == "cpp" else orc.Pager
    return cls(vram_blocks * BLOCK, ram_blocks * BLOCK, recent, interval, 0.05, 0.20, policy)


def _drive(p, count):
    # core.rs:577-582 drive_blocks
    for i in range(count):
        p.on_step(i, 0, [1.0] * (i + 1))
        p.force_rebalance(i)


def _metrics(p):
    if isinstance(p, orc.Pager):
        return dict(p.m)
    m = p.metrics()
    return {k: getattr(m, k) for k in ("tokens", "vram_peak", "ram_peak", "swap_vram_ram", "swap_ram_ssd",
                                       "attention_mass_total", "attention_mass_vram")}


KINDS = ["cpp", "oracle"]


def test_unknown_policy_name_falls_back_to_heavy_hitter():
    assert orc.policy_from_name("not_a_real_policy") == "heavy_hitter"
    codes = {n: pager.lib().pager_core_policy_code(n.encode()) for n in POLICIES + ["not_a_real_policy"]}
    assert codes["not_a_real_policy"] == codes["heavy_hitter"]
    assert len({codes[n] for n in POLICIES}) == 4
    for n in POLICIES:
        assert orc.policy_from_name(n) == n


@pytest.mark.parametrize("kind", KINDS)
def test_recent_only_respects_vram_budget(kind):
    p = _make(kind, 2, 100, 1, "recent_only")
    _drive(p, 5)
    assert len(p.vram_block_ids()) == 2


@pytest.mark.parametrize("kind", KINDS)
def test_recent_only_keeps_the_most_recent_blocks(kind):
    p = _make(kind, 2, 100, 1, "recent_only")
    _drive(p, 5)
    ids = p.vram_block_ids()
    assert 3 in ids and 4 in ids, ids


@pytest.mark.parametrize("kind", KINDS)
def test_sinks_recent_keeps_a_sink_block_resident_even_when_old(kind):
    p = _make(kind, 3, 100, 1, "sinks_recent")
    _drive(p, 10)
    assert any(i < 4 for i in p.vram_block_ids())


@pytest.mark.parametrize("kind", KINDS)
def test_recent_only_ignores_attention_scores_for_placement(kind):
    p = _make(kind, 2, 100, 1, "recent_only")
    p.on_step(0, 0, [1000.0])
    p.force_rebalance(0)
    _drive(p, 6)
    assert 0 not in p.vram_block_ids()


@pytest.mark.parametrize("kind", KINDS)
def test_ensure_blocks_grows_monotonically_and_assigns_sequential_ids(kind):
    p = _make(kind, 10, 10, 4, "recent_only")
    p.on_step(0, 0, [1.0, 1.0, 1.0])
    assert len(p.tiers()) == 3


@pytest.mark.parametrize("kind", KINDS)
def test_metrics_tokens_counts_on_step_calls(kind):
    p = _make(kind, 5, 100, 10, "recent_only")
    assert _metrics(p)["tokens"] == 0
    p.on_step(0, 0, [1.0])
    p.on_step(1, 0, [1.0, 1.0])
    p.on_step(2, 0, [1.0, 1.0, 1.0])
    assert _metrics(p)["tokens"] == 3


@pytest.mark.parametrize("kind", KINDS)
def test_metrics_vram_peak_never_exceeds_budget(kind):
    p = _make(kind, 2, 100, 1, "sinks_heavy_hitter")
    _drive(p, 20)
    assert _metrics(p)["vram_peak"] <= 2 * BLOCK


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("policy", POLICIES)
def test_tiers_never_reports_more_vram_blocks_than_the_budget_allows(kind, policy):
    p = _make(kind, 3, 100, 2, policy)
    _drive(p, 15)
    assert len(p.vram_block_ids()) <= 3


@pytest.mark.parametrize("kind", KINDS)
def test_force_rebalance_is_idempotent(kind):
    p = _make(kind, 2, 100, 1, "recent_only")
    _drive(p, 5)
    before = p.vram_block_ids()
    p.force_rebalance(4)
    assert p.vram_block_ids() == before


def test_ci_smoke_constructor():
    p = pager.PyPager(128_000_000, 2_000_000_000, 64, 4, 0.05, 0.20, "recent_only")
    assert p.tiers() == [] and p.vram_block_ids() == []
    m = p.metrics()
    assert (m.tokens, m.vram_peak, m.swap_vram_ram) == (0, 0, 0)


def test_defaults_and_argument_errors():
    p = pager.PyPager(BLOCK, BLOCK, 1)  # rebalance_interval 32, margins 0.10/0.20, heavy_hitter
    p.on_step(0, 0, [0.5, 0.5])
    assert len(p.tiers()) == 2
    with pytest.raises(OverflowError):
        pager.PyPager(-1, 0, 0)
    with pytest.raises(TypeError):
        pager.PyPager(1.5, 0, 0)
    with pytest.raises(TypeError):
        pager.PyPager(0, 0, 0, policy=3)
    with pytest.raises(OverflowError):
        p.on_step(0, 1 << 32, [1.0])
    with pytest.raises(TypeError):
        p.on_step(0, 0, "abc")
    with pytest.raises(AttributeError):
        p.metrics().tokens = 3


def test_zero_rebalance_interval_panics_on_second_step_like_the_reference():
    p = pager.PyPager(BLOCK, BLOCK, 1, 0)
    p.on_step(0, 0, [1.0])  # tokens == 1 short-circuits the modulo
    with pytest.raises(pager.PanicException):
        p.on_step(1, 0, [1.0, 1.0])
    o = orc.Pager(BLOCK, BLOCK, 1, 0)
    o.on_step(0, 0, [1.0])
    with pytest.raises(ZeroDivisionError):
        o.on_step(1, 0, [1.0, 1.0])


def test_empty_attention_and_tier_codes():
    p = pager.PyPager(2 * BLOCK, 1 * BLOCK, 1, 1, policy="recent_only")
    p.on_step(0, 0, [])
    assert p.tiers() == [0]  # force_rebalance(0) creates block 0 and places it in VRAM
    _drive(p, 4)
    t = p.tiers()
    assert t.count(0) == 2 and t.count(1) == 1 and t.count(2) == 1
    assert set(t) <= {0, 1, 2}


def _attention(rng, n, style):
    if style in ("uniform", "flat"):
        return [1.0 / n] * n
    if style == "classes":
        k = int(rng.integers(0, 3))  # which class is hot this step
        a = np.array([1.0 + 4.0 * (((i * 7) % 3) == k) for i in range(n)], np.float32)
        return (a / a.sum()).tolist()
    if style == "ties":
        return (rng.integers(0, 3, n) / 4.0).astype(np.float32).tolist()
    a = rng.gamma(0.3, 1.0, n).astype(np.float32)
    if style == "heavy":
        a[rng.integers(0, n)] += 5.0
    return (a / a.sum()).tolist()


CASES = [
    # policy, vram blocks, ram blocks, recent, interval, promote margin, ram margin, steps, style
    ("recent_only", 3, 5, 2, 4, 0.05, 0.20, 60, "random"),
    ("sinks_recent", 4, 3, 1, 1, 0.05, 0.20, 50, "random"),
    ("heavy_hitter", 5, 6, 2, 3, 0.01, 0.02, 80, "heavy"),
    ("heavy_hitter", 2, 0, 0, 2, 0.0, 0.0, 40, "ties"),
    ("heavy_hitter", 6, 4, 3, 5, 0.10, 0.20, 90, "random"),
    ("sinks_heavy_hitter", 6, 4, 3, 4, 0.05, 0.20, 80, "heavy"),
    ("sinks_heavy_hitter", 1, 2, 5, 2, 0.05, 0.20, 40, "ties"),
    ("sinks_heavy_hitter", 0, 3, 2, 3, 0.05, 0.20, 30, "random"),
    ("heavy_hitter", 8, 8, 4, 1, 0.001, 0.001, 70, "uniform"),
    ("not_a_policy", 4, 4, 2, 4, 0.05, 0.20, 50, "heavy"),
    # every block present from the first step with equal attention: scores tie, so the
    # first-minimum / last-maximum picks and the stable sorts decide the placement
    ("heavy_hitter", 6, 3, 1, 2, 0.0, 0.0, 30, "flat"),
    ("sinks_heavy_hitter", 7, 5, 2, 3, 0.0, 0.0, 30, "flat"),
    # blocks in three classes of equal attention that change rank over time: swaps have a
    # real gain and several tied candidates
    ("heavy_hitter", 7, 4, 1, 1, 0.0, 0.0, 40, "classes"),
    ("heavy_hitter", 5, 6, 2, 2, 0.001, 0.0, 40, "classes"),
]


@pytest.mark.parametrize("case", CASES, ids=[f"{c[0]}-{c[1]}v{c[2]}r-{c[8]}" for c in CASES])
def test_cpp_matches_oracle_call_by_call(case):
    policy, mv, mr, recent, interval, pm, rm, steps, style = case
    rng = np.random.default_rng(1000 + CASES.index(case))
    cpp = pager.PyPager(mv * BLOCK, mr * BLOCK, recent, interval, pm, rm, policy)
    ref = orc.Pager(mv * BLOCK, mr * BLOCK, recent, interval, pm, rm, policy)
    nblocks = 24 if style in ("flat", "classes") else 1
    for step in range(steps):
        if rng.random() < (0.05 if style in ("flat", "classes") else 0.4):
            nblocks += 1
        att = _attention(rng, nblocks, style)
        qb = nblocks - 1
        cpp.on_step(qb, 0, att)
        ref.on_step(qb, 0, att)
        if rng.random() < 0.3:
            cpp.force_rebalance(qb)
            ref.force_rebalance(qb)
        assert cpp.tiers() == ref.tiers(), step
        assert cpp.vram_block_ids() == ref.vram_block_ids(), step
        assert np.array_equal(np.array(cpp.scores(), np.float32), np.array(ref.scores(), np.float32)), step
        assert _metrics(cpp) == _metrics(ref), step
    assert len(cpp.vram_block_ids()) <= mv


def test_library_exports_every_declared_symbol():
    import os
    import re

    hdr = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "pager_core.h")
    names = re.findall(r"\b(pager_core_\w+)\s*\(", open(hdr).read())
    assert len(set(names)) == 11
    lib = pager.lib()
    for n in set(names):
        assert hasattr(lib, n), n
