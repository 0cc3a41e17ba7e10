"""GPU parity of the fused block-table op ``paged_decode_attention``.

The oracle is the reference's own two-pass sequence (stats over all blocks and
the tail, then accumulate + fold_fixed; pager_hf/paged_model.py:993-1039)
restated in numpy (oracle/streaming_attention_oracle.py, pinned to the
reference's kernels by tests/test_oracle_golden.py), run on the KV each row's
block table gathers (paged_model.py:878-924).  Blocks live in a device pool,
in a pinned host pool (read zero-copy) or are absent; rows are ragged, with
left padding and sliding-window ranges.

Tolerances: output max-abs 2e-3 (fp16), 5e-3 (bf16; P rounds to bf16 before
P.V in both the reference and here), per-block mass 1e-4 relative.
"""

import numpy as np
import pytest
import torch

from oracle import streaming_attention_oracle as orc

pytestmark = pytest.mark.gpu

HOST = 0x40000000


@pytest.fixture(scope="module")
def mods():
    from pager_hf import _lib, streaming_attention
    from pager_hf.host_pool import HostPool

    return streaming_attention, HostPool, _lib


def _np(t):
    return t.detach().float().cpu().numpy()


def build(seed, B, Hq, Hkv, D, tpb, L, nbs, tails, dtype, host_every=2, absent=(), lo=None, hi=None):
    g = torch.Generator().manual_seed(seed)
    slots = sum(nbs) + 2
    dev = torch.randn(slots, L, 2, Hkv, tpb, D, generator=g).to(dtype)
    host = torch.randn(slots, L, 2, Hkv, tpb, D, generator=g).to(dtype)
    max_blocks = max(max(nbs), 1)
    table = torch.full((B, max_blocks), -1, dtype=torch.int32)
    nxt = 0
    for b, nb in enumerate(nbs):
        for j in range(nb):
            if (b, j) in absent:
                continue
            table[b, j] = (nxt | HOST) if (j % host_every == 1) else nxt
            nxt += 1
    tail_cap = max(tails)
    tk = torch.randn(B, Hkv, tail_cap, D, generator=g).to(dtype)
    tv = torch.randn(B, Hkv, tail_cap, D, generator=g).to(dtype)
    q = torch.randn(B, Hq, D, generator=g).to(dtype)
    return dict(q=q, dev=dev, host=host, table=table, nbs=nbs, tails=tails, tk=tk, tv=tv, tpb=tpb, L=L, lo=lo, hi=hi)


def oracle_row(s, b, layer, dt, scale=None, softcap=None):
    """Reference two-pass decode for row b on the KV its block table names."""
    tpb, nb, tl = s["tpb"], s["nbs"][b], s["tails"][b]
    Hkv, D = s["dev"].shape[3], s["dev"].shape[5]
    k = np.zeros((1, Hkv, nb * tpb, D), np.float32)
    v = np.zeros_like(k)
    valid = np.zeros((1, nb * tpb + tl), np.int32)
    for j in range(nb):
        e = int(s["table"][b, j])
        if e < 0:
            continue
        pool = s["host"] if e & HOST else s["dev"]
        slot = e & (HOST - 1)
        k[0, :, j * tpb:(j + 1) * tpb] = _np(pool[slot, layer, 0])
        v[0, :, j * tpb:(j + 1) * tpb] = _np(pool[slot, layer, 1])
        valid[0, j * tpb:(j + 1) * tpb] = 1
    valid[0, nb * tpb:] = 1
    lo = 0 if s["lo"] is None else s["lo"][b]
    hi = nb * tpb + tl if s["hi"] is None else min(s["hi"][b], nb * tpb + tl)
    valid[0, :lo] = 0
    valid[0, hi:] = 0
    tk = _np(s["tk"][b:b + 1, :, :tl])
    tv = _np(s["tv"][b:b + 1, :, :tl])
    q = _np(s["q"][b:b + 1])
    out, mass, m, l = orc.two_pass_decode(q, k, v, tk, tv, nb, tpb, max(nb, 1), valid=valid[:, :nb * tpb],
                                          tail_valid=valid[:, nb * tpb:], scale=scale, softcap=softcap,
                                          v_dtype=dt, out_dtype=dt)
    return out[0], mass[0]


def run_gpu(sa, HostPool, s, layer, mass_mode="row_mean", **kw):
    B = s["q"].shape[0]
    hp = HostPool(s["host"].shape, s["host"].dtype)
    hp.tensor.copy_(s["host"])
    dev = s["dev"].cuda()
    max_blocks = s["table"].shape[1]
    block_mass = torch.zeros(B, s["q"].shape[1], max_blocks, device="cuda")
    accum = torch.zeros((B, max_blocks) if mass_mode == "row_mean" else (max_blocks,), device="cuda")
    max_row = max(nb * s["tpb"] + t for nb, t in zip(s["nbs"], s["tails"]))
    cu = lambda x: None if x is None else torch.tensor(x, dtype=torch.int32, device="cuda")
    out = sa.paged_decode_attention(
        s["q"].cuda(), s["table"].cuda(), cu(s["nbs"]), dev_pool=dev, host_pool=hp.tensor, num_layers=s["L"],
        layer=layer, tokens_per_block=s["tpb"], max_row_tokens=max_row, tail_k=s["tk"].cuda(), tail_v=s["tv"].cuda(),
        tail_len=cu(s["tails"]), valid_lo=cu(s["lo"]), valid_hi=cu(s["hi"]), block_mass=block_mass,
        mass_accum=accum, mass_mode=mass_mode, **kw)
    torch.cuda.synchronize()
    res = (out.float().cpu(), block_mass.cpu(), accum.cpu())
    hp.close()
    return res


CFGS = [
    # (seed, B, Hq, Hkv, D, tpb, L, nbs, tails, dtype, absent, lo, hi)
    (1, 3, 14, 2, 64, 16, 2, [9, 4, 0], [7, 3, 5], torch.float16, {(0, 3)}, None, None),
    (2, 2, 32, 8, 128, 64, 3, [5, 3], [9, 1], torch.bfloat16, set(), [70, 0], None),
    (3, 2, 32, 4, 64, 32, 1, [7, 6], [3, 30], torch.float16, set(), [0, 40], [200, 150]),
    (4, 1, 14, 2, 64, 64, 1, [64], [1], torch.float32, set(), None, None),
    (5, 2, 32, 8, 128, 16, 2, [12, 1], [16, 2], torch.float16, {(0, 0), (0, 11)}, None, None),
    # Gemma geometry: head_dim 256 (tensor cores under "auto"), n_rep 2, a left-padded row
    (6, 2, 8, 4, 256, 32, 2, [7, 3], [5, 20], torch.bfloat16, set(), [10, 0], None),
]


@pytest.mark.parametrize("cfg", CFGS, ids=[f"cfg{c[0]}" for c in CFGS])
@pytest.mark.parametrize("backend", ["auto", "fma"])
def test_paged_matches_reference_two_pass(mods, cfg, backend):
    sa, HostPool, lib = mods
    seed, B, Hq, Hkv, D, tpb, L, nbs, tails, dtype, absent, lo, hi = cfg
    s = build(seed, B, Hq, Hkv, D, tpb, L, nbs, tails, dtype, absent=absent, lo=lo, hi=hi)
    dt = {torch.float16: "f16", torch.bfloat16: "bf16", torch.float32: "f32"}[dtype]
    layer = L - 1
    sa.set_backend(backend)
    try:
        out, bm, accum = run_gpu(sa, HostPool, s, layer)
    finally:
        sa.set_backend("auto")
    atol = 5e-3 if dtype == torch.bfloat16 else 2e-3
    for b in range(B):
        ref_out, ref_mass = oracle_row(s, b, layer, dt)
        np.testing.assert_allclose(out[b].numpy(), ref_out, rtol=0, atol=atol)
        nb = nbs[b]
        np.testing.assert_allclose(bm[b, :, :nb].numpy(), ref_mass[:, :nb], rtol=1e-4, atol=1e-6)
        np.testing.assert_allclose(accum[b, :nb].numpy(), ref_mass[:, :nb].mean(0), rtol=1e-4, atol=1e-6)
    assert lib.device_status(0) == 0


@pytest.mark.parametrize("hq,hkv", [(14, 2), (48, 16)])
def test_batch_mean_mass_mode(mods, hq, hkv):
    sa, HostPool, lib = mods
    s = build(7, 2, hq, hkv, 64, 16, 1, [6, 6], [2, 2], torch.float16)
    _, bm, accum = run_gpu(sa, HostPool, s, 0, mass_mode="batch_mean")
    np.testing.assert_allclose(accum.numpy(), bm.mean(dim=(0, 1)).numpy(), rtol=1e-5, atol=1e-7)
    ref = np.stack([oracle_row(s, b, 0, "f16")[1] for b in range(2)]).mean(axis=(0, 1))
    np.testing.assert_allclose(accum.numpy(), ref, rtol=1e-4, atol=1e-6)


def test_out_of_range_slot_is_flagged_not_read(mods):
    """A block-table entry beyond the pool is skipped (treated as absent) and flagged on the device."""
    sa, HostPool, lib = mods
    s = build(8, 1, 8, 2, 64, 16, 1, [4], [2], torch.float16)
    s["table"][0, 2] = 10_000  # no such device slot
    lib.device_status(0)
    out, bm, _ = run_gpu(sa, HostPool, s, 0)
    assert lib.device_status(0) == 6
    s["table"][0, 2] = -1
    ref_out, ref_mass = oracle_row(s, 0, 0, "f16")
    np.testing.assert_allclose(out[0].numpy(), ref_out, rtol=0, atol=2e-3)
    np.testing.assert_allclose(bm[0].numpy(), ref_mass, rtol=1e-4, atol=1e-6)


def test_row_with_nothing_to_read_next_to_full_rows(mods):
    """A row with no block and no tail token (no tile at all) gets the reference's 0/0 output and zero
    mass; the other rows of the same launch are unaffected."""
    sa, HostPool, lib = mods
    s = build(9, 3, 8, 2, 64, 16, 1, [5, 0, 3], [4, 0, 2], torch.float16)
    out, bm, accum = run_gpu(sa, HostPool, s, 0)
    assert torch.isnan(out[1]).all()
    assert float(bm[1].abs().sum()) == 0 and float(accum[1].abs().sum()) == 0
    for b in (0, 2):
        ref_out, ref_mass = oracle_row(s, b, 0, "f16")
        np.testing.assert_allclose(out[b].numpy(), ref_out, rtol=0, atol=2e-3)
        nb = s["nbs"][b]
        np.testing.assert_allclose(accum[b, :nb].numpy(), ref_mass[:, :nb].mean(0), rtol=1e-4, atol=1e-6)
    assert lib.device_status(0) == 0


EXTRA = [
    # (name, seed, B, Hq, Hkv, D, tpb, L, nbs, tails, dtype, kw) -- kw: scale / softcap / backend
    ("softcap_mma_d128", 11, 2, 16, 8, 128, 64, 2, [6, 3], [9, 2], torch.bfloat16, dict(scale=0.0625, softcap=50.0)),
    ("softcap_d256", 12, 2, 8, 4, 256, 32, 1, [5, 2], [4, 31], torch.bfloat16, dict(scale=1 / 16, softcap=30.0)),
    ("fp16_d256_n_rep_8", 22, 2, 16, 2, 256, 64, 1, [6, 4], [9, 63], torch.float16, {}),
    ("blocks_of_256", 13, 2, 8, 2, 64, 256, 1, [3, 2], [200, 17], torch.float16, {}),
    ("blocks_of_8", 14, 2, 8, 2, 64, 8, 1, [40, 7], [5, 8], torch.float16, {}),
    ("n_rep_16", 15, 2, 32, 2, 128, 64, 1, [4, 5], [3, 60], torch.float16, {}),
    ("n_rep_1_mha", 16, 2, 4, 4, 64, 32, 2, [6, 2], [1, 30], torch.float16, {}),
    ("fp32_d8", 17, 3, 4, 2, 8, 16, 1, [5, 1, 3], [2, 16, 1], torch.float32, {}),
    ("fp16_d32", 18, 2, 6, 3, 32, 16, 1, [9, 4], [15, 1], torch.float16, {}),
    ("bf16_d16", 23, 2, 8, 2, 16, 16, 1, [7, 3], [12, 0], torch.bfloat16, {}),
    ("fp32_d256_softcap", 24, 1, 4, 2, 256, 16, 1, [5], [3], torch.float32, dict(softcap=20.0)),
    # the mass pass finalizes heads in chunks of 32: 48 heads end on a partial chunk, 80 on two more
    ("heads_48_chunked_mass", 19, 2, 48, 16, 64, 16, 1, [9, 3], [4, 11], torch.float16, {}),
    ("heads_80_bf16_d128", 20, 1, 80, 8, 128, 64, 1, [5], [7], torch.bfloat16, {}),
    # one row, two kv heads, 300 blocks: planned at 37 splits, more than a warp's lanes hold at once
    ("many_splits_one_row", 21, 1, 8, 2, 64, 64, 1, [300], [13], torch.float16, {}),
]


@pytest.mark.parametrize("case", EXTRA, ids=[c[0] for c in EXTRA])
def test_paged_op_options_match_the_reference(mods, case):
    """Softcap and custom scale (MMA and FMA), blocks larger than a tile and the smallest blocks,
    GQA fan-out 16 and plain MHA, fp32 and small head dims, more query heads than the mass pass
    finalizes at once, and a row split more ways than a warp has lanes."""
    sa, HostPool, lib = mods
    name, seed, B, Hq, Hkv, D, tpb, L, nbs, tails, dtype, kw = case
    s = build(seed, B, Hq, Hkv, D, tpb, L, nbs, tails, dtype)
    dt = {torch.float16: "f16", torch.bfloat16: "bf16", torch.float32: "f32"}[dtype]
    layer = L - 1
    out, bm, _ = run_gpu(sa, HostPool, s, layer, **kw)
    atol = 5e-3 if dtype == torch.bfloat16 else 2e-3
    for b in range(B):
        ref_out, ref_mass = oracle_row(s, b, layer, dt, scale=kw.get("scale"), softcap=kw.get("softcap"))
        np.testing.assert_allclose(out[b].numpy(), ref_out, rtol=0, atol=atol, err_msg=f"{name} row {b}")
        nb = nbs[b]
        np.testing.assert_allclose(bm[b, :, :nb].numpy(), ref_mass[:, :nb], rtol=1e-4, atol=1e-6)
    assert lib.device_status(0) == 0


def test_host_pool_only_and_batch_mean_with_inactive_rows(mods):
    """No device pool at all (every block in the pinned host pool), one inactive row: the inactive row's
    output is untouched and the batch mean divides by all rows and heads, as the separate mass kernel does."""
    sa, HostPool, lib = mods
    s = build(19, 3, 8, 2, 64, 16, 1, [6, 4, 5], [3, 9, 2], torch.float16, host_every=1)
    s["table"] = torch.where(s["table"] >= 0, s["table"] | HOST, s["table"])  # every entry in the host pool
    hp = HostPool(s["host"].shape, s["host"].dtype)
    hp.tensor.copy_(s["host"])
    B, Hq, D = 3, 8, 64
    cu = lambda x: torch.tensor(x, dtype=torch.int32, device="cuda")
    out = torch.full((B, Hq, D), 7.0, dtype=torch.float16, device="cuda")
    accum = torch.zeros(s["table"].shape[1], device="cuda")
    bm = torch.zeros(B, Hq, s["table"].shape[1], device="cuda")
    sa.paged_decode_attention(
        s["q"].cuda(), s["table"].cuda(), cu(s["nbs"]), dev_pool=None, host_pool=hp.tensor, num_layers=1, layer=0,
        tokens_per_block=16, max_row_tokens=max(nb * 16 + t for nb, t in zip(s["nbs"], s["tails"])),
        tail_k=s["tk"].cuda(), tail_v=s["tv"].cuda(), tail_len=cu(s["tails"]), active=cu([1, 0, 1]),
        out=out, block_mass=bm, mass_accum=accum, mass_mode="batch_mean")
    torch.cuda.synchronize()
    hp.close()
    assert torch.all(out[1] == 7.0)  # inactive row untouched
    refs = {b: oracle_row(s, b, 0, "f16") for b in (0, 2)}
    for b, (ref_out, _) in refs.items():
        np.testing.assert_allclose(out[b].float().cpu().numpy(), ref_out, rtol=0, atol=2e-3)
    want = np.zeros(s["table"].shape[1], np.float32)
    for b, (_, ref_mass) in refs.items():
        want[:s["nbs"][b]] += ref_mass[:, :s["nbs"][b]].sum(0)
    np.testing.assert_allclose(accum.cpu().numpy(), want / (B * Hq), rtol=1e-4, atol=1e-7)
    assert lib.device_status(0) == 0
