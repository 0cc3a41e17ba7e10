"""Model-level parity helpers: the reference's attention for one fused-op call, from the pools.

``reference_attention(plan, q, layer, rule)`` gathers each row's KV the way the reference's
``PagedModel._gather_layer_kv_group`` does (paged_model.py:878-924: per block, the layer's K and V
from whichever tier holds it), masks the row's attended range, and runs the vectorised torch
restatement of the reference's per-layer sequence (``oracle/streaming_attention_torch.py``) with
the plan's tile structure.  ``install`` swaps it in for ``PagedDecodePlan.run`` (a greedy run whose
every layer attends with the reference's algorithm) or runs it beside the kernel and records both.
Test infrastructure only.
"""

from __future__ import annotations

import torch

from oracle import streaming_attention_torch as ort

HOST = 0x40000000


def reference_attention(plan, q: torch.Tensor, layer: int, rule: str):
    """Returns (out [B, Hq, D] in q's dtype, block mass [B, Hq, max_blocks] = per-block sum of p / l)."""
    B, Hq, tpb = plan.B, plan.Hq, plan.tpb
    dev = q.device
    nbs = plan.num_blocks.tolist()
    table = plan.block_table.cpu()
    lo = plan.valid_lo.tolist() if plan.valid_lo is not None else [0] * B
    hi = plan.valid_hi.tolist() if plan.valid_hi is not None else [n * tpb for n in nbs]
    tails = plan.ref_tail_start.tolist() if plan.ref_tail_start is not None else [n * tpb for n in nbs]
    shifts = plan.ref_shift.tolist() if plan.ref_shift is not None else [0] * B
    pool = plan.dev_pool if plan.dev_pool is not None else plan.host_pool
    Hkv, D = pool.shape[3], pool.shape[5]
    outs = torch.empty(B, Hq, D, dtype=q.dtype, device=dev)
    mass = torch.zeros(B, Hq, plan.max_blocks, device=dev)
    for b in range(B):
        n = nbs[b]
        ids = table[b, :n]
        K = torch.zeros(n, 2, Hkv, tpb, D, dtype=pool.dtype, device=dev)
        present = torch.zeros(n, dtype=torch.bool)
        on_dev = (ids >= 0) & ((ids & HOST) == 0)
        on_host = (ids >= 0) & ((ids & HOST) != 0)
        if bool(on_dev.any()):
            K[on_dev.to(dev)] = plan.dev_pool[ids[on_dev].long().to(dev), layer]
        if bool(on_host.any()):
            K[on_host.to(dev)] = plan.host_pool[(ids[on_host] & (HOST - 1)).long(), layer].to(dev)
        present |= on_dev | on_host
        k = K[:, 0].permute(1, 0, 2, 3).reshape(1, Hkv, n * tpb, D)
        v = K[:, 1].permute(1, 0, 2, 3).reshape(1, Hkv, n * tpb, D)
        valid = present.repeat_interleave(tpb).to(dev)
        cols = torch.arange(n * tpb, device=dev)
        valid &= (cols >= lo[b]) & (cols < hi[b])
        keys = ort.reference_tile_keys(n * tpb, tails[b], shifts[b], plan.ref_group_tokens, device=dev)
        out, _, _, pl = ort.reference_decode(q[b:b + 1], k, v, valid[None], keys[None], rule, scale=plan.scale,
                                             softcap=plan.softcap or None)
        outs[b] = out[0]
        mass[b, :, :n] = pl[0].reshape(Hq, n, tpb).sum(-1)
    return outs, mass


def accumulate_mass(plan, mass: torch.Tensor) -> None:
    """What the fused op adds to its plan's ``mass_accum`` for the given per-head block mass."""
    if plan.mass_accum is None or plan.mass_mode == 0:
        return
    if plan.mass_mode == 1:  # row mean
        plan.mass_accum += mass.mean(dim=1)[:, : plan.mass_accum.shape[1]]
    else:  # batch mean
        plan.mass_accum += mass.mean(dim=(0, 1))[: plan.mass_accum.shape[0]]


def install(monkeypatch, rule: str, mode: str, record: list | None = None) -> None:
    """``mode="reference"``: every ``PagedDecodePlan.run`` computes the reference's attention instead
    of launching the kernels.  ``mode="compare"``: the kernels run, then the reference on the same
    pools; ``record`` gets (layer, max-abs output difference, fraction of differing rounded outputs,
    max relative mass difference, the worst difference in units of the larger of 2e-3 and one ulp of
    the output dtype at the reference value) per call.  Eager steps only (the hooks run Python per
    layer)."""
    from pager_hf.streaming_attention import PagedDecodePlan

    orig = PagedDecodePlan.run

    def run(self, q, layer, out, stream=None):
        if mode == "reference":
            o, mass = reference_attention(self, q, layer, rule)
            out.copy_(o)
            accumulate_mass(self, mass)
            return out
        before = None if self.mass_accum is None else self.mass_accum.clone()
        orig(self, q, layer, out, stream)
        torch.cuda.synchronize()
        o, mass = reference_attention(self, q, layer, rule)
        got, want = out.float(), o.float()
        mass_err = 0.0
        if before is not None:
            ref_acc = before.clone()
            tmp = self.mass_accum
            self.mass_accum = ref_acc
            accumulate_mass(self, mass)
            self.mass_accum = tmp
            scale = ref_acc.abs().max().clamp(min=1e-30)
            mass_err = float(((tmp - ref_acc).abs() / scale).max())
        ulp = torch.finfo(out.dtype).eps * want.abs()
        units = float(((got - want).abs() / torch.clamp(ulp, min=2e-3)).max())
        record.append((layer, float((got - want).abs().max()), float((got != want).float().mean()), mass_err, units))
        return out

    monkeypatch.setattr(PagedDecodePlan, "run", run)


def record_logits(pm) -> list:
    """Wraps a PagedModel's step so that each step's last-position logits (float, per row) are kept."""
    steps = []
    orig = pm._forward_step

    def step(input_ids, attention_mask):
        logits, info = orig(input_ids, attention_mask)
        steps.append(logits[:, -1].float().clone())
        return logits, info

    pm._forward_step = step
    return steps


def first_divergences(got: list, want: list, ref_logits: list, dtype) -> list:
    """Per row: None when the token lists are equal, else (step, got token, reference token, the
    reference run's own gap between those two logits in ulps of the model's dtype at that size)."""
    res = []
    eps = torch.finfo(dtype).eps
    for row, (a, b) in enumerate(zip(got, want)):
        div = None
        for i, (x, y) in enumerate(zip(a, b)):
            if x != y:
                lg = ref_logits[i][row]
                gap = abs(float(lg[x]) - float(lg[y]))
                ulp = eps * max(abs(float(lg[y])), 1e-3)
                div = (i, x, y, gap / ulp)
                break
        if div is None and len(a) != len(b):
            div = (min(len(a), len(b)), None, None, float("inf"))
        res.append(div)
    return res
