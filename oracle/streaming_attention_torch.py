"""Vectorised torch restatement of the reference's decode attention, for model-level parity.

TEST INFRASTRUCTURE ONLY, like ``streaming_attention_oracle``: only ``tests/`` use it, as the
checker.  It computes what the reference's per-layer sequence computes -- the one-pass path of
pager_hf/paged_model.py:1055-1072 or the two-pass path of :993-1039 -- in one vectorised pass per
call, so that a whole greedy generation can run with it as the attention of every layer:

* scores are the fp32 product of the (fp16/bf16/fp32) query and keys, times ``scale``, then the
  optional softcap and the mask (streaming_attention.py:158-161);
* p = exp(s - m) is rounded to the value dtype before P.V and summed unrounded into l
  (:177-179; :346-349 in the two-pass path), m being the reference's running max after the
  64-token tile holding the token (``rule="running"``; a tile's max rises only when the tile is
  folded in, :163-164) or the row's final max (``rule="final"``);
* the reference's acc * alpha rescaling per tile is the same sum as weighting each tile's
  contribution by exp(m_tile - m_final): only the fp32 association differs.

It is pinned to the numpy oracle (``single_pass_decode`` / ``two_pass_decode``) by
``tests/test_oracle_torch_cpu.py``.
"""

from __future__ import annotations

import torch

BLOCK_KV = 64  # streaming_attention.py:11


def reference_tile_keys(n_tokens: int, tail_start: int, shift: int = 0, group_tokens: int = 0,
                        device=None) -> torch.Tensor:
    """The reference's tile of each row-local token as an increasing key: 64-token tiles from the
    start of each chunk -- groups of ``group_tokens`` tokens of a numbering in which token j sits at
    ``shift + j`` (batched_decode.py:185-234 pads shorter sessions in front), then the tail chunk
    from ``tail_start`` (paged_model.py:1055-1070)."""
    j = torch.arange(n_tokens, device=device, dtype=torch.int64)
    c = j + shift
    if group_tokens > 0:
        grp = c // group_tokens
        key = grp * ((group_tokens + BLOCK_KV - 1) // BLOCK_KV) + (c - grp * group_tokens) // BLOCK_KV
    else:
        key = c // BLOCK_KV
    tail = (1 << 40) + (j - tail_start) // BLOCK_KV
    return torch.where(j >= tail_start, tail, key)


def reference_decode(q, k, v, valid, keys, rule: str, scale=None, softcap=None, out_dtype=None):
    """q [B, Hq, D]; k, v [B, Hkv, N, D]; valid [B, N] (bool or 0/1); keys [B, N] increasing tile
    keys (``reference_tile_keys``).  Returns (out [B, Hq, D] in ``out_dtype`` (default q's dtype),
    m_final [B, Hq], l [B, Hq], p_over_l [B, Hq, N]: each token's unrounded p / l, from which the
    per-block mass of the two-pass path (:349-350) is a sum)."""
    B, Hq, D = q.shape
    Hkv, N = k.shape[1], k.shape[2]
    n_rep = Hq // Hkv
    if scale is None:
        scale = 1.0 / D ** 0.5
    out_dtype = q.dtype if out_dtype is None else out_dtype
    vd = v.dtype
    qg = q.float().reshape(B, Hkv, n_rep, D)
    kf = k.float().masked_fill(~valid.bool()[:, None, :, None], 0.0)
    s = torch.matmul(qg, kf.transpose(-1, -2)) * scale  # [B, Hkv, n_rep, N]
    if softcap:
        s = softcap * torch.tanh(s / softcap)
    mask = valid.bool()[:, None, None, :]
    s = s.masked_fill(~mask, float("-inf"))
    if rule == "final":
        mtok = s.amax(dim=-1, keepdim=True).expand_as(s)
    elif rule == "running":
        # each tile's max, then the running max over tiles in order, broadcast back to the tokens
        dense = torch.stack([torch.unique_consecutive(keys[b], return_inverse=True)[1] for b in range(B)])
        T = int(dense.max()) + 1
        d4 = dense[:, None, None, :].expand_as(s)
        tmax = torch.full(s.shape[:-1] + (T,), float("-inf"), device=s.device)
        tmax = tmax.scatter_reduce(-1, d4, s, reduce="amax", include_self=True)
        run = torch.cummax(tmax, dim=-1).values
        mtok = torch.gather(run, -1, d4)
    else:
        raise ValueError(f"rule must be 'running' or 'final', got {rule!r}")
    mfin = s.amax(dim=-1, keepdim=True)
    empty_tok = mtok == float("-inf")
    p = torch.where(empty_tok, torch.zeros_like(s), torch.exp(s - torch.where(empty_tok, torch.zeros_like(mtok), mtok)))
    pr = p.to(vd).float()
    w = torch.where(empty_tok, torch.zeros_like(s), torch.exp(mtok - torch.where(mfin == float("-inf"),
                                                                               torch.zeros_like(mfin), mfin)))
    vf = v.float().masked_fill(~valid.bool()[:, None, :, None], 0.0)
    acc = torch.matmul(pr * w, vf)  # [B, Hkv, n_rep, D]
    l = (p * w).sum(dim=-1)
    out = (acc / l[..., None]).to(out_dtype).reshape(B, Hq, D)
    p_over_l = (p * w / l[..., None]).reshape(B, Hq, N)
    return out, mfin[..., 0].reshape(B, Hq), l.reshape(B, Hq), p_over_l


def dense_reference(q, k, v, n_rep: int, tokens_per_block: int, valid=None, scale=None, softcap=None):
    """Dense GQA decode attention with per-block mass, as the reference's own test oracle computes it
    (tests/test_streaming_attention.py:20-40): K and V repeated per query head, fp32 scores times
    ``scale``, optional softcap, masked softmax, P.V, and the attention weights summed per block of
    ``tokens_per_block`` tokens (a ragged last block included).  This torch path on the host cores is
    the CPU baseline the benchmark times.  q [B, Hq, D]; k, v [B, Hkv, T, D]; valid [B, T] or None.
    Returns (out [B, Hq, D] fp32, block_mass [B, Hq, ceil(T / tokens_per_block)])."""
    key = k.repeat_interleave(n_rep, dim=1).float()
    value = v.repeat_interleave(n_rep, dim=1).float()
    if scale is None:
        scale = 1.0 / q.shape[-1] ** 0.5
    s = torch.einsum("bhd,bhtd->bht", q.float(), key) * scale
    if softcap is not None:
        s = softcap * torch.tanh(s / softcap)
    if valid is not None:
        s = s.masked_fill(valid[:, None, :] == 0, float("-inf"))
    w = torch.softmax(s, dim=-1)
    out = torch.einsum("bht,bhtd->bhd", w, value)
    T = k.shape[2]
    nb = (T + tokens_per_block - 1) // tokens_per_block
    mass = torch.stack([w[:, :, b * tokens_per_block:(b + 1) * tokens_per_block].sum(dim=-1) for b in range(nb)],
                       dim=2)
    return out, mass
