"""Staged host-tier reads (copy engines + TMA) give the same bits as zero-copy reads.

The staged path copies each layer's host blocks into a device buffer on a copy
stream, double-buffered across layers; the kernel then reads the same bytes
through TMA instead of consumer-side loads from mapped memory, so outputs and
block mass must be bit-identical.  Covered: odd and even layer counts (the
next-step prefetch then lands in the half the last layer reads), prefetch on
and off, three decode steps with one plan, rows mixing device, host and absent
blocks plus tails.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

HOST = 0x40000000


def _setup(seed, L, B=3, Hq=16, Hkv=4, D=128, tpb=32, nb=9, dtype=torch.bfloat16):
    from pager_hf.host_pool import HostPool

    g = torch.Generator().manual_seed(seed)
    dev = torch.randn(B * nb, L, 2, Hkv, tpb, D, generator=g).to(dtype).cuda()
    host = HostPool((B * nb + 3, L, 2, Hkv, tpb, D), dtype)
    host.tensor.copy_(torch.randn(host.shape, generator=g).to(dtype))
    table = torch.full((B, nb), -1, dtype=torch.int32)
    d = h = 0
    for b in range(B):
        for j in range(nb):
            if (b, j) == (1, 4):
                continue  # absent block
            if j % 3 == 0:
                table[b, j] = d
                d += 1
            else:
                table[b, j] = (h + (2 if b == 2 else 0)) | HOST  # row 2's host slots start after a gap
                h += 1
    tails = torch.tensor([5, 32, 1], dtype=torch.int32)
    return dict(dev=dev, host=host, table=table.cuda(), nb=torch.full((B,), nb, dtype=torch.int32).cuda(), lo=None,
                tk=torch.randn(B, Hkv, tpb, D, generator=g).to(dtype).cuda(),
                tv=torch.randn(B, Hkv, tpb, D, generator=g).to(dtype).cuda(), tails=tails.cuda(),
                q=[torch.randn(B, Hq, D, generator=g).to(dtype).cuda() for _ in range(3 * L)],
                B=B, Hq=Hq, L=L, tpb=tpb, max_row=nb * tpb + tpb, dtype=dtype)


def _run(s, host_read, prefetch):
    from pager_hf.streaming_attention import PagedDecodePlan

    mass = torch.zeros(s["B"], s["table"].shape[1], device="cuda")
    plan = PagedDecodePlan(batch=s["B"], num_query_heads=s["Hq"], dev_pool=s["dev"], host_pool=s["host"].tensor,
                           num_layers=s["L"], tokens_per_block=s["tpb"], block_table=s["table"],
                           num_blocks=s["nb"], max_row_tokens=s["max_row"], tail_k=s["tk"], tail_v=s["tv"],
                           tail_len=s["tails"], valid_lo=s["lo"], mass_accum=mass, mass_mode="row_mean",
                           host_read=host_read,
                           prefetch_next_step=prefetch)
    assert plan.host_read == host_read
    outs = []
    for step in range(3):
        for layer in range(s["L"]):
            out = torch.empty(s["B"], s["Hq"], 128, dtype=s["dtype"], device="cuda")
            plan.run(s["q"][step * s["L"] + layer], layer, out)
            outs.append(out)
    torch.cuda.synchronize()
    return torch.stack(outs).cpu(), mass.cpu()


@pytest.mark.parametrize("L", [1, 3, 4])
@pytest.mark.parametrize("prefetch", [False, True])
def test_staged_reads_match_zero_copy_bit_for_bit(L, prefetch):
    from pager_hf import _lib

    s = _setup(40 + L, L)
    try:
        ref_out, ref_mass = _run(s, "zero_copy", False)
        out, mass = _run(s, "staged", prefetch)
        assert torch.equal(out, ref_out)
        assert torch.equal(mass, ref_mass)
        assert float(mass.sum()) > 0
        assert _lib.device_status(0) == 0
    finally:
        s["host"].close()


def test_auto_mode_picks_from_measured_link():
    from pager_hf.host_staging import choose_host_read, link_bandwidth

    bw = link_bandwidth("cuda")
    assert bw["copy_gbs"] > 1 and bw["zero_copy_gbs"] > 1
    assert choose_host_read("cuda") == ("staged" if bw["copy_gbs"] > bw["zero_copy_gbs"] else "zero_copy")


def test_window_rows_mix_staged_and_zero_copy_entries():
    """With a window only some host blocks are staged; the rest stay zero-copy in the same launch."""
    from pager_hf import _lib

    s = _setup(77, 2)
    s["lo"] = torch.tensor([100, 0, 250], dtype=torch.int32).cuda()
    try:
        ref_out, ref_mass = _run(s, "zero_copy", False)
        out, mass = _run(s, "staged", True)
        assert torch.equal(out, ref_out) and torch.equal(mass, ref_mass)
        assert float(mass[0, :3].abs().sum()) == 0  # blocks before the window carry no mass
        assert _lib.device_status(0) == 0
    finally:
        s["host"].close()
