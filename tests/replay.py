"""Replay the reference's call sequences through the drop-in ``pager_hf.streaming_attention``.

Mirrors tests/golden/make_golden.py (which ran them through the reference's
own kernels) so GPU results can be compared with the golden fixtures.
"""

import torch

from cases import CASES, batched_combined_layout, build_batched, build_contiguous, group_row_active


def run_case(sa, name, device="cuda"):
    """Returns dict with out (float32 CPU), and m, l, acc, block_mass / session_mass where defined."""
    c = CASES[name]
    if c["kind"] == "batched":
        return _run_batched(sa, c, device)
    q, k, v, valid, active = (t.to(device) for t in build_contiguous(c))
    B, Hq, D = c["B"], c["Hq"], c["D"]
    if c["kind"] == "steps":
        m, l, acc = sa.streaming_attention_state_init(B, Hq, D, device)
        T, g = c["T"], c["group"]
        for s in range(0, T, g):
            e = min(s + g, T)
            sa.streaming_attention_step(q, k[:, :, s:e], v[:, :, s:e], m, l, acc, valid=valid[:, s:e], active=active,
                                        scale=c.get("scale"), softcap=c.get("softcap"))
        out = sa.streaming_attention_finalize(acc, l, q.dtype)
        return dict(out=out.float().cpu(), m=m.cpu(), l=l.cpu(), acc=acc.cpu())
    tpb, nb, tail = c["tpb"], c["nb"], c["tail"]
    full, gt = nb * tpb, c["group_blocks"] * tpb
    act = active if c.get("active") else None
    m, l, _ = sa.streaming_attention_state_init(B, Hq, D, device)
    for s in range(0, full, gt):
        e = min(s + gt, full)
        sa.streaming_attention_stats_step(q, k[:, :, s:e], m, l, valid=valid[:, s:e], active=act)
    if tail:
        sa.streaming_attention_stats_step(q, k[:, :, full:], m, l, valid=valid[:, full:])
    acc = torch.zeros(B, Hq, D, dtype=torch.float32, device=device)
    bm = torch.zeros(B, Hq, max(nb, 1), dtype=torch.float32, device=device)
    for s in range(0, full, gt):
        e = min(s + gt, full)
        sa.streaming_attention_accumulate_step(q, k[:, :, s:e], v[:, :, s:e], m, l, acc, bm, s // tpb, tpb,
                                               valid=valid[:, s:e], active=act)
    if tail:
        sa.streaming_attention_fold_fixed_step(q, k[:, :, full:], v[:, :, full:], m, l, acc, valid=valid[:, full:])
    out = sa.streaming_attention_finalize(acc, l, q.dtype)
    return dict(out=out.float().cpu(), m=m.cpu(), l=l.cpu(), acc=acc.cpu(), block_mass=bm[:, :, :nb].cpu())


def _run_batched(sa, c, device):
    q, bk, bv, tk, tv = build_batched(c)
    k, v, valid, pad_blocks, tail_k, tail_v = batched_combined_layout(c, bk, bv, tk, tv)
    q, k, v, valid, tail_k, tail_v = (t.to(device) for t in (q, k, v, valid, tail_k, tail_v))
    S, Hq, D, tpb, group = q.shape[0], c["Hq"], c["D"], c["tpb"], c["group_blocks"]
    max_blocks = max(c["nbs"])
    m, l, acc = sa.streaming_attention_state_init(S, Hq, D, device)
    for i in range(0, max_blocks, group):
        n = min(group, max_blocks - i)
        sl = slice(i * tpb, (i + n) * tpb)
        sa.streaming_attention_stats_step(q, k[:, :, sl], m, l, valid=valid[:, sl],
                                          active=group_row_active(pad_blocks, i, n).to(device))
    sa.streaming_attention_stats_step(q, tail_k, m, l)
    bm = torch.zeros(S, Hq, max(max_blocks, 1), dtype=torch.float32, device=device)
    for i in range(0, max_blocks, group):
        n = min(group, max_blocks - i)
        sl = slice(i * tpb, (i + n) * tpb)
        sa.streaming_attention_accumulate_step(q, k[:, :, sl], v[:, :, sl], m, l, acc, bm, i, tpb, valid=valid[:, sl],
                                               active=group_row_active(pad_blocks, i, n).to(device))
    sa.streaming_attention_fold_fixed_step(q, tail_k, tail_v, m, l, acc)
    out = sa.streaming_attention_finalize(acc, l, q.dtype)
    per_row = bm.mean(dim=1).cpu()
    session_mass = torch.zeros(S, max(max_blocks, 1))
    for row, nb in enumerate(c["nbs"]):
        session_mass[row, :nb] = per_row[row, pad_blocks[row]:pad_blocks[row] + nb]
    return dict(out=out.float().cpu(), m=m.cpu(), l=l.cpu(), acc=acc.cpu(), session_mass=session_mass)
