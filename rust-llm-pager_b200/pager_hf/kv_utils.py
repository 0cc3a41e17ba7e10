"""KV-cache helpers with the reference's names and behaviour (``pager_hf/kv_utils.py``).

Host-side tensor bookkeeping around the block store: normalising a model's
cache to ``[(key, value)] * layers`` with ``[batch, kv_heads, seq, head_dim]``
tensors, cutting it into full blocks and a tail, the block layout
``[layers, batch, block_len, kv_heads, head_dim]`` the store's ``put_gpu``
takes, the inverse reconstruction, and per-block attention from per-token
attention.  The decode path of this package never reconstructs the cache:
blocks stay in the pools and the fused op reads them in place; these helpers
serve callers of the reference API and tests.
"""

from __future__ import annotations

import torch


def get_legacy_past_key_values(outputs):
    """``outputs.past_key_values`` as a list of per-layer ``(key, value)`` (``kv_utils.py:8-20``).

    Accepts the tuple form, cache objects with ``key_cache`` / ``value_cache``
    lists, and the installed transformers' cache objects whose ``layers`` hold
    ``keys`` / ``values``."""
    past = outputs.past_key_values
    if past is None:
        raise RuntimeError("Model did not return past_key_values.")
    if isinstance(past, (tuple, list)):
        return list(past)
    if hasattr(past, "key_cache") and hasattr(past, "value_cache"):
        return list(zip(past.key_cache, past.value_cache))
    layers = getattr(past, "layers", None)
    if layers is not None and all(hasattr(x, "keys") and hasattr(x, "values") for x in layers):
        return [(x.keys, x.values) for x in layers]
    raise TypeError(f"Unsupported past_key_values type: {type(past)!r}")


def split_full_blocks_and_tail(past_key_values, *, tokens_per_block: int):
    """``(full_past, tail_past, full_tokens)``: the first ``floor(seq / tpb) * tpb`` tokens of every layer
    and the remainder (``kv_utils.py:23-34``)."""
    seq = past_key_values[0][0].shape[2]
    full = seq - seq % tokens_per_block
    head, tail = [], []
    for key, value in past_key_values:
        head.append((key[:, :, :full, :].contiguous(), value[:, :, :full, :].contiguous()))
        tail.append((key[:, :, full:, :].contiguous(), value[:, :, full:, :].contiguous()))
    return head, tail, full


def extract_single_block_from_past(past_key_values, *, block_id: int, tokens_per_block: int):
    """Block ``block_id`` of every layer as ``[layers, batch, block_len, kv_heads, head_dim]`` key and value
    (``kv_utils.py:37-53``)."""
    lo = block_id * tokens_per_block
    hi = lo + tokens_per_block
    keys = torch.stack([k[:, :, lo:hi, :].permute(0, 2, 1, 3) for k, _ in past_key_values], dim=0)
    values = torch.stack([v[:, :, lo:hi, :].permute(0, 2, 1, 3) for _, v in past_key_values], dim=0)
    return keys.contiguous(), values.contiguous()


def real_past_to_blocks(past_key_values, *, tokens_per_block: int):
    """Every full block of the cache, in order (``kv_utils.py:56-61``)."""
    n = past_key_values[0][0].shape[2] // tokens_per_block
    return [extract_single_block_from_past(past_key_values, block_id=j, tokens_per_block=tokens_per_block)
            for j in range(n)]


def token_attention_to_blocks(attn_to_keys: torch.Tensor, *, tokens_per_block: int, num_blocks: int):
    """Per-token attention summed per block and normalised to sum 1; uniform when the total is not positive
    (``kv_utils.py:64-77``).  Each block is summed token by token in double precision (a running sum),
    as the reference's loop does."""
    import numpy as np

    n = num_blocks * tokens_per_block
    if attn_to_keys.numel() < n:
        raise IndexError(f"attention covers {attn_to_keys.numel()} tokens, the blocks {n}")
    if num_blocks == 0:
        return []
    per_token = attn_to_keys[:n].detach().cpu().double().numpy().reshape(num_blocks, tokens_per_block)
    sums = np.cumsum(per_token, axis=1)[:, -1].tolist()
    total = sum(sums)
    if total <= 0:
        return [1.0 / num_blocks] * num_blocks
    return [x / total for x in sums]


def extract_last_query_block_attention(outputs, *, tokens_per_block: int, num_blocks: int):
    """The last query token's block attention, averaged over layers, heads and batch rows, normalised
    (``kv_utils.py:80-108``)."""
    attentions = outputs.attentions
    if attentions is None:
        raise RuntimeError("Model did not return attentions.")
    per_layer = [token_attention_to_blocks(a.detach().float().cpu()[:, :, -1, :].mean(dim=(0, 1)),
                                           tokens_per_block=tokens_per_block, num_blocks=num_blocks)
                 for a in attentions]
    mean = [sum(col) / len(per_layer) for col in zip(*per_layer)]
    total = sum(mean)
    if total <= 0:
        return [1.0 / num_blocks] * num_blocks
    return [x / total for x in mean]


def reconstruct_past_from_store(*, store, num_layers: int, num_blocks: int, tail_past=None):
    """The cache rebuilt from ``store.get_gpu(0..num_blocks-1)`` plus an optional tail, written into one
    pre-sized tensor per layer (``kv_utils.py:111-178``).  With no blocks the shape comes from the tail;
    with neither, ``ValueError``."""
    if num_blocks > 0:
        k0, _ = store.get_gpu(0)
        _, batch, tpb, kv_heads, head_dim = k0.shape
        like = [(k0[i].dtype, k0[i].device) for i in range(num_layers)]
    elif tail_past:
        batch, kv_heads, _, head_dim = tail_past[0][0].shape
        tpb = 0
        like = [(tail_past[i][0].dtype, tail_past[i][0].device) for i in range(num_layers)]
    else:
        raise ValueError("reconstruct_past_from_store: no blocks and no tail to reconstruct from.")
    tail_len = tail_past[0][0].shape[2] if tail_past else 0
    start_tail = num_blocks * tpb
    total = start_tail + tail_len
    out = [(torch.empty(batch, kv_heads, total, head_dim, dtype=dt, device=dev),
            torch.empty(batch, kv_heads, total, head_dim, dtype=dt, device=dev)) for dt, dev in like]
    for j in range(num_blocks):
        key, value = store.get_gpu(j)
        lo = j * tpb
        for layer in range(num_layers):
            out[layer][0][:, :, lo:lo + tpb, :] = key[layer].permute(0, 2, 1, 3)
            out[layer][1][:, :, lo:lo + tpb, :] = value[layer].permute(0, 2, 1, 3)
    if tail_past:
        for layer in range(num_layers):
            out[layer][0][:, :, start_tail:, :] = tail_past[layer][0]
            out[layer][1][:, :, start_tail:, :] = tail_past[layer][1]
    return out
