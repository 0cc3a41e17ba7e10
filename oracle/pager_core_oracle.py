"""Test oracle: CPU restatement of the reference's Rust block pager.

TEST INFRASTRUCTURE ONLY -- imported by ``tests/`` to check the C++ pager
(``libpager_core.so``); nothing in the product calls it.

Follows ``pager/src/core.rs`` of rust-llm-pager step by step (line numbers
below).  Scores are numpy float32 scalars so that every EMA operation rounds
to f32 like Rust's ``f32`` arithmetic; the attention mass totals are Python
floats (f64).  Sorts are Python's stable ``sorted``; ``min_by`` returns the
first of equal minima and ``max_by`` the last of equal maxima, as Rust's
iterator methods do.  Comparisons treat unordered pairs (NaN) as equal
(``compare_scores``, core.rs:555-557).

Parity pin: the Rust crate cannot be built here (no Rust toolchain); this
restatement and the C++ library are pinned by the reference's own unit tests
(core.rs:559-705, ported in tests/test_pager_core_cpu.py) and its CI smoke call
(.github/workflows/ci.yml:81).  Its only third-party dependencies are binding
glue (pyo3 0.21.2, serde 1.0.228); no arithmetic lives there.
"""

from __future__ import annotations

import numpy as np

BLOCK_SIZE_BYTES = 16 * 1024 * 1024  # core.rs:6
SINK_BLOCKS = 4  # core.rs:7
VRAM, RAM, SSD = 0, 1, 2  # core.rs:9-14, tiers() codes core.rs:111-119
POLICIES = ("recent_only", "sinks_recent", "heavy_hitter", "sinks_heavy_hitter")  # core.rs:16-22
F32 = np.float32


def policy_from_name(name: str) -> str:
    """core.rs:24-33: unknown names fall back to heavy_hitter."""
    return name if name in POLICIES else "heavy_hitter"


def compare(a, b) -> int:
    """core.rs:555-557: partial_cmp with unordered -> Equal."""
    if a < b:
        return -1
    if a > b:
        return 1
    return 0


def _key(cmp):
    import functools

    return functools.cmp_to_key(cmp)


class Block:
    __slots__ = ("id", "size", "score", "tier", "pinned")

    def __init__(self, bid):
        self.id, self.size, self.score, self.tier, self.pinned = bid, BLOCK_SIZE_BYTES, F32(0.0), RAM, False


class Pager:
    """core.rs:56-84 ``Pager::new`` and the methods below it."""

    def __init__(self, vram, ram, recent_window, rebalance_interval=32, promote_margin=0.10,
                 ram_promote_margin=0.20, policy="heavy_hitter"):
        self.vram, self.ram, self.recent_window = vram, ram, recent_window
        self.rebalance_interval = rebalance_interval
        self.promote_margin, self.ram_promote_margin = F32(promote_margin), F32(ram_promote_margin)
        self.policy = policy_from_name(policy)
        self.m = dict(tokens=0, vram_peak=0, ram_peak=0, swap_vram_ram=0, swap_ram_ssd=0,
                      attention_mass_total=0.0, attention_mass_vram=0.0)
        self.blocks: list[Block] = []

    # core.rs:86-98
    def on_step(self, token_idx, layer, attention):
        att = [F32(a) for a in attention]
        self.m["tokens"] += 1
        self.ensure_blocks(len(att))
        self.update_scores(att)
        self.update_attention_quality(att)
        self.pin_blocks(token_idx)
        t = self.m["tokens"]
        if t == 1 or t % self.rebalance_interval == 0:  # ZeroDivisionError where Rust panics
            self.force_rebalance(token_idx)

    # core.rs:100-107
    def force_rebalance(self, token_idx):
        self.ensure_blocks(token_idx + 1)
        self.pin_blocks(token_idx)
        self.place_blocks()
        self.update_memory_peaks()

    def tiers(self):
        return [b.tier for b in self.blocks]

    def vram_block_ids(self):
        return [b.id for b in self.blocks if b.tier == VRAM]

    def scores(self):
        return [float(b.score) for b in self.blocks]

    # core.rs:133-142
    def ensure_blocks(self, count):
        while len(self.blocks) < count:
            self.blocks.append(Block(len(self.blocks)))

    # core.rs:144-148
    def update_scores(self, att):
        for blk, a in zip(self.blocks, att):
            blk.score = F32(blk.score * F32(0.90)) + F32(a * F32(0.10))

    # core.rs:150-164
    def update_attention_quality(self, att):
        total = vram = 0.0
        for blk, a in zip(self.blocks, att):
            total += float(a)
            if blk.tier == VRAM:
                vram += float(a)
        self.m["attention_mass_total"] += total
        self.m["attention_mass_vram"] += vram

    # core.rs:166-177
    def pin_blocks(self, token_idx):
        start = max(0, token_idx - self.recent_window)
        for blk in self.blocks:
            recent = blk.id >= start
            sink = blk.id < SINK_BLOCKS
            blk.pinned = recent if self.policy == "recent_only" else (recent or sink)

    # core.rs:179-195
    def place_blocks(self):
        old = [b.tier for b in self.blocks]
        mv, mr = self.vram // BLOCK_SIZE_BYTES, self.ram // BLOCK_SIZE_BYTES
        if self.policy in ("recent_only", "sinks_recent"):
            self.place_baseline_blocks(mv, mr)
        elif self.policy == "heavy_hitter":
            self.place_heavy_hitter(mv, mr)
        else:
            self.place_sinks_heavy_hitter(mv, mr)
        self.count_tier_changes(old)

    def _pinned_then(self, then):
        def cmp(a, b):
            pa, pb = self.blocks[a].pinned, self.blocks[b].pinned
            if pa != pb:
                return -1 if pa else 1
            return then(a, b)
        return cmp

    # core.rs:197-216
    def place_baseline_blocks(self, mv, mr):
        order = sorted(range(len(self.blocks)),
                       key=_key(self._pinned_then(lambda a, b: compare(self.blocks[a].id, self.blocks[b].id))))
        for b in self.blocks:
            b.tier = SSD
        self.assign_ranked_blocks(order, mv, mr)

    # core.rs:218-250
    def place_heavy_hitter(self, mv, mr):
        if not any(b.tier == VRAM for b in self.blocks):
            order = sorted(range(len(self.blocks)), key=_key(
                self._pinned_then(lambda a, b: compare(self.blocks[b].score, self.blocks[a].score))))
            self.assign_ranked_blocks(order, mv, mr)
            return
        for b in self.blocks:
            if b.pinned:
                b.tier = VRAM
        self.enforce_vram_budget_keep_best(mv)
        self.promote_vram_with_hysteresis(mv)
        self.fill_ram(mr)
        self.promote_ram_with_hysteresis(mr)

    # core.rs:252-313
    def place_sinks_heavy_hitter(self, mv, mr):
        for b in self.blocks:
            b.tier = SSD
        if mv == 0:
            return
        sel = set()
        for b in self.blocks[:SINK_BLOCKS]:
            if len(sel) >= mv:
                break
            sel.add(b.id)
        remaining = max(0, mv - len(sel))
        budget = min(self.recent_window, max(mv // 2, 1), remaining)
        start = max(0, len(self.blocks) - budget)
        for b in self.blocks[start:]:
            if len(sel) >= mv:
                break
            sel.add(b.id)
        scored = [(b.id, b.score) for b in self.blocks if b.id not in sel]
        scored = sorted(scored, key=_key(lambda x, y: compare(y[1], x[1])))
        for bid, _ in scored:
            if len(sel) >= mv:
                break
            sel.add(bid)
        for b in self.blocks:
            if b.id in sel:
                b.tier = VRAM
        self.fill_ram(mr)

    # core.rs:315-328
    def assign_ranked_blocks(self, order, mv, mr):
        for rank, i in enumerate(order):
            self.blocks[i].tier = VRAM if rank < mv else (RAM if rank < mv + mr else SSD)

    # core.rs:336-354
    def enforce_vram_budget_keep_best(self, mv):
        ids = [i for i, b in enumerate(self.blocks) if b.tier == VRAM]
        if len(ids) <= mv:
            return
        ids = sorted(ids, key=_key(self._pinned_then(lambda a, b: compare(self.blocks[b].score, self.blocks[a].score))))
        for i in ids[mv:]:
            self.blocks[i].tier = RAM

    def _min_by(self, pred):
        best = None
        for i, b in enumerate(self.blocks):
            if pred(b) and (best is None or compare(self.blocks[best].score, b.score) > 0):
                best = i
        return best

    def _max_by(self, pred):
        best = None
        for i, b in enumerate(self.blocks):
            if pred(b) and (best is None or compare(self.blocks[best].score, b.score) <= 0):
                best = i
        return best

    # core.rs:356-387
    def promote_vram_with_hysteresis(self, mv):
        while True:
            count = sum(b.tier == VRAM for b in self.blocks)
            if count < mv:
                best = self._max_by(lambda b: b.tier != VRAM)
                if best is not None:
                    self.blocks[best].tier = VRAM
                    continue
                break
            worst = self._min_by(lambda b: b.tier == VRAM and not b.pinned)
            if worst is None:
                break
            best = self._max_by(lambda b: b.tier != VRAM)
            if best is None:
                break
            if F32(self.blocks[best].score - self.blocks[worst].score) <= self.promote_margin:
                break
            prev = self.blocks[best].tier
            self.blocks[best].tier = VRAM
            self.blocks[worst].tier = prev

    # core.rs:389-427
    def fill_ram(self, mr):
        cur = sum(b.tier == RAM for b in self.blocks)
        if cur >= mr:
            self.trim_ram(mr)
            return
        cand = [i for i, b in enumerate(self.blocks) if b.tier == SSD]
        cand = sorted(cand, key=_key(lambda a, b: compare(self.blocks[b].score, self.blocks[a].score)))
        for i in cand[:mr - cur]:
            self.blocks[i].tier = RAM

    # core.rs:429-448
    def trim_ram(self, mr):
        ids = [i for i, b in enumerate(self.blocks) if b.tier == RAM]
        if len(ids) <= mr:
            return
        ids = sorted(ids, key=_key(lambda a, b: compare(self.blocks[a].score, self.blocks[b].score)))
        for i in ids[:len(ids) - mr]:
            self.blocks[i].tier = SSD

    # core.rs:450-477
    def promote_ram_with_hysteresis(self, mr):
        while True:
            if sum(b.tier == RAM for b in self.blocks) < mr:
                break
            worst = self._min_by(lambda b: b.tier == RAM)
            if worst is None:
                break
            best = self._max_by(lambda b: b.tier == SSD)
            if best is None:
                break
            if F32(self.blocks[best].score - self.blocks[worst].score) <= self.ram_promote_margin:
                break
            self.blocks[best].tier = RAM
            self.blocks[worst].tier = SSD

    # core.rs:511-529
    def count_tier_changes(self, old):
        for b, o in zip(self.blocks, old):
            pair = {o, b.tier}
            if o == b.tier:
                continue
            if pair == {VRAM, RAM}:
                self.m["swap_vram_ram"] += b.size
            elif pair == {RAM, SSD}:
                self.m["swap_ram_ssd"] += b.size
            else:
                self.m["swap_vram_ram"] += b.size
                self.m["swap_ram_ssd"] += b.size

    # core.rs:531-552
    def update_memory_peaks(self):
        v = sum(b.size for b in self.blocks if b.tier == VRAM)
        r = sum(b.size for b in self.blocks if b.tier == RAM)
        self.m["vram_peak"] = max(self.m["vram_peak"], v)
        self.m["ram_peak"] = max(self.m["ram_peak"], r)
