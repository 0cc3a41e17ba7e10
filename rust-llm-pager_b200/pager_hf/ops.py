"""The decode-attention entry points as torch operators (``torch.ops.pager_b200.*``).

The functions of ``streaming_attention`` call the C ABI directly (one ctypes call each, cheap
enough for a CUDA graph).  Registered here as ``torch.library`` custom operators, the same calls
become visible to ``torch.ops``, to fake-tensor tracing (each has a fake implementation that only
propagates shapes and dtypes) and to ``torch.compile``, which treats them as opaque ops: the
in-place state arguments are declared as mutated, exactly as the reference's functions mutate them
(``pager_hf/streaming_attention.py:452-670``).

    import pager_hf.ops  # registers the operators
    torch.ops.pager_b200.streaming_attention_step(q, k, v, m, l, acc, None, None, None, None)
"""

from __future__ import annotations

import torch

from . import streaming_attention as sa

_NS = "pager_b200"


@torch.library.custom_op(f"{_NS}::streaming_attention_step", mutates_args=("m", "l", "acc"))
def streaming_attention_step(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, m: torch.Tensor, l: torch.Tensor,
                             acc: torch.Tensor, valid: torch.Tensor | None, active: torch.Tensor | None,
                             scale: float | None, softcap: float | None) -> None:
    sa.streaming_attention_step(q, k, v, m, l, acc, valid=valid, active=active, scale=scale, softcap=softcap)


@streaming_attention_step.register_fake
def _(q, k, v, m, l, acc, valid, active, scale, softcap):
    return None


@torch.library.custom_op(f"{_NS}::streaming_attention_stats_step", mutates_args=("m", "l"))
def streaming_attention_stats_step(q: torch.Tensor, k: torch.Tensor, m: torch.Tensor, l: torch.Tensor,
                                   valid: torch.Tensor | None, active: torch.Tensor | None, scale: float | None,
                                   softcap: float | None) -> None:
    sa.streaming_attention_stats_step(q, k, m, l, valid=valid, active=active, scale=scale, softcap=softcap)


@streaming_attention_stats_step.register_fake
def _(q, k, m, l, valid, active, scale, softcap):
    return None


@torch.library.custom_op(f"{_NS}::streaming_attention_accumulate_step", mutates_args=("acc", "block_mass"))
def streaming_attention_accumulate_step(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, m: torch.Tensor,
                                        l: torch.Tensor, acc: torch.Tensor, block_mass: torch.Tensor,
                                        block_id_offset: int, tokens_per_block: int, valid: torch.Tensor | None,
                                        active: torch.Tensor | None, scale: float | None,
                                        softcap: float | None) -> None:
    sa.streaming_attention_accumulate_step(q, k, v, m, l, acc, block_mass, block_id_offset, tokens_per_block,
                                           valid=valid, active=active, scale=scale, softcap=softcap)


@streaming_attention_accumulate_step.register_fake
def _(q, k, v, m, l, acc, block_mass, block_id_offset, tokens_per_block, valid, active, scale, softcap):
    return None


@torch.library.custom_op(f"{_NS}::streaming_attention_fold_fixed_step", mutates_args=("acc",))
def streaming_attention_fold_fixed_step(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, m: torch.Tensor,
                                        l: torch.Tensor, acc: torch.Tensor, valid: torch.Tensor | None,
                                        scale: float | None, softcap: float | None) -> None:
    sa.streaming_attention_fold_fixed_step(q, k, v, m, l, acc, valid=valid, scale=scale, softcap=softcap)


@streaming_attention_fold_fixed_step.register_fake
def _(q, k, v, m, l, acc, valid, scale, softcap):
    return None


@torch.library.custom_op(f"{_NS}::streaming_attention_finalize", mutates_args=())
def streaming_attention_finalize(acc: torch.Tensor, l: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    return sa.streaming_attention_finalize(acc, l, dtype)


@streaming_attention_finalize.register_fake
def _(acc, l, dtype):
    return torch.empty(acc.shape, dtype=dtype, device=acc.device)


@torch.library.custom_op(f"{_NS}::paged_decode_attention", mutates_args=("mass_accum",))
def paged_decode_attention(q: torch.Tensor, block_table: torch.Tensor, num_blocks: torch.Tensor,
                           dev_pool: torch.Tensor | None, host_pool: torch.Tensor | None, num_layers: int, layer: int,
                           tokens_per_block: int, max_row_tokens: int, tail_k: torch.Tensor | None,
                           tail_v: torch.Tensor | None, tail_len: torch.Tensor | None, valid_lo: torch.Tensor | None,
                           valid_hi: torch.Tensor | None, active: torch.Tensor | None, scale: float | None,
                           softcap: float | None, mass_accum: torch.Tensor | None, mass_mode: str,
                           rounding: str) -> torch.Tensor:
    return sa.paged_decode_attention(
        q, block_table, num_blocks, dev_pool=dev_pool, host_pool=host_pool, num_layers=num_layers, layer=layer,
        tokens_per_block=tokens_per_block, max_row_tokens=max_row_tokens, tail_k=tail_k, tail_v=tail_v,
        tail_len=tail_len, valid_lo=valid_lo, valid_hi=valid_hi, active=active, scale=scale, softcap=softcap,
        mass_accum=mass_accum, mass_mode=mass_mode, rounding=rounding)


@paged_decode_attention.register_fake
def _(q, block_table, num_blocks, dev_pool, host_pool, num_layers, layer, tokens_per_block, max_row_tokens, tail_k,
      tail_v, tail_len, valid_lo, valid_hi, active, scale, softcap, mass_accum, mass_mode, rounding):
    return torch.empty(q.shape, dtype=q.dtype, device=q.device)
