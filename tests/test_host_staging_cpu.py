"""Run planning of the staged host tier (``pager_hf/host_staging.plan_host_runs``)."""

import numpy as np
import torch

from pager_hf.host_staging import HOST_SLOT_BIT, STAGE_SLOT_BIT, plan_host_runs


def test_runs_cover_distinct_host_slots_in_order():
    H = HOST_SLOT_BIT
    table = torch.tensor([[0, 5 | H, 6 | H, -1, 9 | H],
                          [1, 7 | H, 5 | H, 2, 12 | H]], dtype=torch.int32)
    staged, slots, (src, dst, ln) = plan_host_runs(table)
    assert slots.tolist() == [5, 6, 7, 9, 12]
    # runs of consecutive host slots -> consecutive staging slots
    assert src.tolist() == [5, 9, 12] and dst.tolist() == [0, 3, 4] and ln.tolist() == [3, 1, 1]
    # device entries and absent entries unchanged; host entries renamed to their staging slot
    assert staged[0, 0] == 0 and staged[1, 3] == 2 and staged[0, 3] == -1
    expect = {5: 0, 6: 1, 7: 2, 9: 3, 12: 4}
    for (r, c) in [(0, 1), (0, 2), (0, 4), (1, 1), (1, 2), (1, 4)]:
        e = int(table[r, c])
        assert int(staged[r, c]) == (expect[e & (H - 1)] | STAGE_SLOT_BIT)
    assert int(np.sum(ln)) == len(slots)


def test_table_without_host_blocks_has_no_runs():
    table = torch.tensor([[0, 1, -1], [2, 3, 4]], dtype=torch.int32)
    staged, slots, runs = plan_host_runs(table)
    assert torch.equal(staged, table) and slots.numel() == 0 and all(len(r) == 0 for r in runs)


def test_only_blocks_the_kernel_reads_are_staged():
    """Blocks beyond num_blocks, outside [valid_lo, valid_hi) or in inactive rows keep their host tag."""
    H = HOST_SLOT_BIT
    tpb = 16
    table = torch.tensor([[0 | H, 1 | H, 2 | H, 3 | H],
                          [4 | H, 5 | H, 6 | H, 7 | H],
                          [8 | H, 9 | H, 10 | H, 11 | H]], dtype=torch.int32)
    nb = torch.tensor([4, 3, 4], dtype=torch.int32)
    lo = torch.tensor([20, 0, 0], dtype=torch.int32)   # row 0: block 0 (tokens 0..15) is before the window
    hi = torch.tensor([64, 33, 64], dtype=torch.int32)  # row 1: tokens 33.. excluded -> block 2 starts at 32: kept
    active = torch.tensor([1, 1, 0], dtype=torch.int32)
    staged, slots, _ = plan_host_runs(table, tpb, nb, lo, hi, active)
    assert slots.tolist() == [1, 2, 3, 4, 5, 6]
    assert int(staged[0, 0]) == 0 | H                  # outside the window: still a host entry
    assert int(staged[1, 3]) == 7 | H                  # beyond num_blocks
    assert all(int(staged[2, j]) == table[2, j] for j in range(4))  # inactive row
    assert int(staged[1, 2]) & STAGE_SLOT_BIT


def test_auto_choice_counts_one_submission_per_copy():
    """``auto`` stages a host tier that lies in a few long runs of slots and reads a scattered one
    zero-copy: each run is one copy submission (``COPY_SUBMIT_S`` of host time), overlapped with
    the copies themselves."""
    from pager_hf import host_staging as hs

    dev = torch.device("cuda", 7)  # a recorded (fake) link: nothing touches a GPU
    try:
        hs.record_link_bandwidth(dev, copy_gbs=55.6, zero_copy_gbs=51.5)
        assert hs.choose_host_read(dev) == "staged"  # without sizes: the faster link
        assert hs.choose_host_read(dev, 362 << 20, copies_per_layer=1) == "staged"  # one contiguous run
        assert hs.choose_host_read(dev, 225 << 20, copies_per_layer=566) == "zero_copy"  # scattered slots
        # a windowed layer: 8 runs of 2 MiB, submitted while the copies run
        assert hs.choose_host_read(dev, 16 << 20, copies_per_layer=8) == "staged"
        # break-even: submissions take as long as zero-copy reads of the same bytes
        nbytes = 64 << 20
        k = int(nbytes / 51.5e9 / hs.COPY_SUBMIT_S)
        assert hs.choose_host_read(dev, nbytes, copies_per_layer=k) == "staged"
        assert hs.choose_host_read(dev, nbytes, copies_per_layer=k + 2) == "zero_copy"
        hs.record_link_bandwidth(dev, copy_gbs=40.0, zero_copy_gbs=51.5)
        assert hs.choose_host_read(dev, 362 << 20, copies_per_layer=1) == "zero_copy"
    finally:
        hs._LINK.pop(7, None)


def test_plan_properties_on_random_tables():
    """Over seeded random tables (device, host and absent entries; per-row num_blocks, token windows
    and active flags): every entry the kernel reads from the host tier is renamed to a staging slot
    that the runs fill from the same host slot; every other entry is unchanged; the runs are maximal
    and fill the staging buffer densely in ascending host-slot order."""
    H = HOST_SLOT_BIT
    rng = np.random.default_rng(7)
    for _ in range(200):
        B, nb, tpb = int(rng.integers(1, 6)), int(rng.integers(1, 24)), int(rng.choice([1, 16, 64]))
        kind = rng.integers(0, 3, (B, nb))
        slot = rng.integers(0, 40, (B, nb))
        table = torch.tensor(np.where(kind == 0, -1, np.where(kind == 1, slot, slot | H)), dtype=torch.int32)
        num_blocks = torch.tensor(rng.integers(0, nb + 1, B), dtype=torch.int32)
        hi = torch.tensor(rng.integers(0, nb * tpb + 1, B), dtype=torch.int32)
        lo = torch.tensor([int(rng.integers(0, int(h) + 1)) for h in hi], dtype=torch.int32)
        active = torch.tensor(rng.integers(0, 2, B), dtype=torch.int32)
        staged, slots, (src, dst, ln) = plan_host_runs(table, tpb, num_blocks, lo, hi, active)

        stage_of = np.full(int(ln.sum()), -1)  # host slot each staging slot receives
        for s, d, n in zip(src, dst, ln):
            stage_of[d:d + n] = np.arange(s, s + n)
        assert stage_of.tolist() == slots.tolist() and np.all(np.diff(stage_of) > 0)
        assert np.all(src[1:] != src[:-1] + ln[:-1]) and np.all(dst == np.concatenate(([0], np.cumsum(ln)[:-1])))

        for b in range(B):
            for j in range(nb):
                e, g = int(table[b, j]), int(staged[b, j])
                read = (e >= 0 and e & H and j < num_blocks[b] and (j + 1) * tpb > lo[b] and j * tpb < hi[b]
                        and active[b])
                if read:
                    assert g & STAGE_SLOT_BIT and stage_of[g & (STAGE_SLOT_BIT - 1)] == e & (H - 1)
                else:
                    assert g == e
