"""Streaming decode attention on B200: drop-in for rust-llm-pager's
``pager_hf/streaming_attention.py``.

The six public functions keep the reference's names, signatures, defaults,
in-place semantics and error behaviour (streaming_attention.py:444-670); the
work is done by ``libpager_b200.so`` (split-KV kernels for sm_100a reached
through its C ABI, include/pager_b200.h).  ``paged_decode_attention`` is the
new fused entry that walks a block table in one pass (device pool, pinned
host pool, tail) and emits the per-block attention mass alongside the output.

There is no Triton and no CPU fallback: every function requires CUDA tensors
and raises if the native library is missing.
"""

from __future__ import annotations

import torch

from . import _lib as L

# Kept for callers that read or monkeypatch them (the reference's bench
# scripts patch _BLOCK_KV, bench/streaming_attention_kernel_scaling_probe.py:56-66);
# the CUDA kernels choose their own tile sizes.
_BLOCK_KV = 64
_M_TILE = 16
_MIN_DOT_DIM = 16

_BACKEND = L.BACKEND_AUTO


def set_backend(name: str) -> None:
    """Select the split kernel's compute backend: "auto", "mma" (tensor cores) or "fma" (CUDA cores)."""
    global _BACKEND
    _BACKEND = {"auto": L.BACKEND_AUTO, "mma": L.BACKEND_MMA, "fma": L.BACKEND_FMA}[name]


def _validate_n_rep(n_rep: int) -> None:
    """streaming_attention.py:69-74."""
    if n_rep > _M_TILE:
        raise NotImplementedError(
            f"streaming attention's GQA query-head packing supports n_rep up to {_M_TILE}, got {n_rep}. "
            "This architecture's query/KV head ratio is wider than any currently supported model."
        )


def _default_valid(k: torch.Tensor) -> torch.Tensor:
    """All-valid mask, [batch, chunk_tokens] (streaming_attention.py:433-436)."""
    batch_size, _, total_tokens, _ = k.shape
    return torch.ones((batch_size, total_tokens), dtype=torch.int32, device=k.device)


def _default_active(batch_size: int, device: torch.device) -> torch.Tensor:
    """All-active [batch] switch (streaming_attention.py:439-441)."""
    return torch.ones((batch_size,), dtype=torch.int32, device=device)


def _dtype_code(t: torch.Tensor, what: str) -> int:
    try:
        return L.DTYPE_CODE[t.dtype]
    except KeyError:
        raise ValueError(f"{what} must be float32, float16 or bfloat16, got {t.dtype}") from None


def _require_cuda(**tensors) -> None:
    for name, t in tensors.items():
        if t is not None and not t.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor (the B200 path has no CPU fallback)")


def _state(t: torch.Tensor, name: str, shape: tuple) -> torch.Tensor:
    if t.dtype != torch.float32 or not t.is_contiguous() or tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} must be a contiguous float32 tensor of shape {tuple(shape)}, got "
                         f"{t.dtype} {tuple(t.shape)} contiguous={t.is_contiguous()}")
    return t


def _aligned(t: torch.Tensor) -> torch.Tensor:
    t = t.contiguous()
    return t if t.data_ptr() % 16 == 0 else t.clone()


def _mask(t: torch.Tensor | None) -> torch.Tensor | None:
    if t is None:
        return None
    return t.to(torch.int32).contiguous()


def _scratch(nbytes: int, device: torch.device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


def _common(q, k):
    if q.dim() != 3 or k.dim() != 4:
        raise ValueError(f"expected q [batch, heads, dim] and k [batch, kv_heads, tokens, dim], got {tuple(q.shape)} "
                         f"and {tuple(k.shape)}")
    batch_size, num_query_heads, head_dim = q.shape
    _, num_kv_heads, total_tokens, _ = k.shape
    n_rep = num_query_heads // num_kv_heads
    _validate_n_rep(n_rep)
    return batch_size, num_query_heads, num_kv_heads, total_tokens, head_dim


def streaming_attention_state_init(batch_size: int, num_query_heads: int, head_dim: int, device: torch.device):
    """Fresh online-softmax state (m=-inf, l=0, acc=0) before any KV chunk (streaming_attention.py:444-449)."""
    device = torch.device(device)
    m = torch.empty((batch_size, num_query_heads), dtype=torch.float32, device=device)
    l = torch.empty((batch_size, num_query_heads), dtype=torch.float32, device=device)
    acc = torch.empty((batch_size, num_query_heads, head_dim), dtype=torch.float32, device=device)
    _require_cuda(m=m)
    with torch.cuda.device(device):
        L.check(L.lib().pager_attn_state_init(m.data_ptr(), l.data_ptr(), acc.data_ptr(), batch_size * num_query_heads,
                                              head_dim, L.stream_of(m)))
    return m, l, acc


def streaming_attention_step(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    m: torch.Tensor,
    l: torch.Tensor,
    acc: torch.Tensor,
    valid: torch.Tensor | None = None,
    active: torch.Tensor | None = None,
    scale: float | None = None,
    softcap: float | None = None,
) -> None:
    """Fold one KV chunk into the running (m, l, acc) state, in place (streaming_attention.py:452-513).

    q: [batch, num_query_heads, head_dim]; k, v: [batch, num_kv_heads, chunk_tokens, head_dim].
    valid: optional [batch, chunk_tokens] 0/1 mask; active: optional [batch] 0/1 row switch
    (active=0 leaves that row's state bit-for-bit untouched); scale defaults to 1/sqrt(head_dim);
    softcap None/0 disables logit softcapping.
    """
    B, Hq, Hkv, T, D = _common(q, k)
    _require_cuda(q=q, k=k, v=v, m=m, l=l, acc=acc, valid=valid, active=active)
    _state(m, "m", (B, Hq))
    _state(l, "l", (B, Hq))
    _state(acc, "acc", (B, Hq, D))
    if scale is None:
        scale = 1.0 / (D**0.5)
    q, k, v = q.contiguous(), _aligned(k), _aligned(v)
    if v.dtype != k.dtype:
        raise ValueError(f"k and v must share a dtype, got {k.dtype} and {v.dtype}")
    valid, active = _mask(valid), _mask(active)
    kvd = _dtype_code(k, "k")
    lib = L.lib()
    with torch.cuda.device(q.device):
        nbytes = lib.pager_attn_chunk_scratch_bytes(0, B, Hq, Hkv, T, D, kvd, 16)
        scratch = _scratch(nbytes, q.device)
        L.check(lib.pager_attn_step(q.data_ptr(), _dtype_code(q, "q"), k.data_ptr(), v.data_ptr(), kvd, L.ptr(valid),
                                    L.ptr(active), m.data_ptr(), l.data_ptr(), acc.data_ptr(), B, Hq, Hkv, T, D,
                                    float(scale), float(softcap or 0.0), _BACKEND, scratch.data_ptr(), scratch.numel(),
                                    L.stream_of(q)))


def streaming_attention_stats_step(
    q: torch.Tensor,
    k: torch.Tensor,
    m: torch.Tensor,
    l: torch.Tensor,
    valid: torch.Tensor | None = None,
    active: torch.Tensor | None = None,
    scale: float | None = None,
    softcap: float | None = None,
) -> None:
    """Pass 1: fold one chunk's K into running (m, l) only (streaming_attention.py:516-560)."""
    B, Hq, Hkv, T, D = _common(q, k)
    _require_cuda(q=q, k=k, m=m, l=l, valid=valid, active=active)
    _state(m, "m", (B, Hq))
    _state(l, "l", (B, Hq))
    if scale is None:
        scale = 1.0 / (D**0.5)
    q, k = q.contiguous(), _aligned(k)
    valid, active = _mask(valid), _mask(active)
    kvd = _dtype_code(k, "k")
    lib = L.lib()
    with torch.cuda.device(q.device):
        nbytes = lib.pager_attn_chunk_scratch_bytes(1, B, Hq, Hkv, T, D, kvd, 16)
        scratch = _scratch(nbytes, q.device)
        L.check(lib.pager_attn_stats_step(q.data_ptr(), _dtype_code(q, "q"), k.data_ptr(), kvd, L.ptr(valid),
                                          L.ptr(active), m.data_ptr(), l.data_ptr(), B, Hq, Hkv, T, D, float(scale),
                                          float(softcap or 0.0), _BACKEND, scratch.data_ptr(), scratch.numel(),
                                          L.stream_of(q)))


def streaming_attention_accumulate_step(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    m: torch.Tensor,
    l: torch.Tensor,
    acc: torch.Tensor,
    block_mass: torch.Tensor,
    block_id_offset: int,
    tokens_per_block: int,
    valid: torch.Tensor | None = None,
    active: torch.Tensor | None = None,
    scale: float | None = None,
    softcap: float | None = None,
) -> None:
    """Pass 2: fold a block-aligned chunk into acc with final (m, l) and write its per-block
    attention mass (streaming_attention.py:563-621).  block_mass [batch, heads, max_blocks] is
    written at columns block_id_offset + j; rows with active=0 are left untouched."""
    B, Hq, Hkv, T, D = _common(q, k)
    _require_cuda(q=q, k=k, v=v, m=m, l=l, acc=acc, block_mass=block_mass, valid=valid, active=active)
    _state(m, "m", (B, Hq))
    _state(l, "l", (B, Hq))
    _state(acc, "acc", (B, Hq, D))
    if block_mass.dtype != torch.float32 or not block_mass.is_contiguous() or block_mass.dim() != 3 or \
            tuple(block_mass.shape[:2]) != (B, Hq):
        raise ValueError(f"block_mass must be a contiguous float32 [batch, heads, max_blocks] tensor, got "
                         f"{block_mass.dtype} {tuple(block_mass.shape)}")
    max_blocks = block_mass.shape[2]
    if scale is None:
        scale = 1.0 / (D**0.5)
    q, k, v = q.contiguous(), _aligned(k), _aligned(v)
    valid, active = _mask(valid), _mask(active)
    kvd = _dtype_code(k, "k")
    lib = L.lib()
    with torch.cuda.device(q.device):
        nbytes = lib.pager_attn_chunk_scratch_bytes(2, B, Hq, Hkv, T, D, kvd, int(tokens_per_block))
        scratch = _scratch(nbytes, q.device)
        L.check(lib.pager_attn_accumulate_step(
            q.data_ptr(), _dtype_code(q, "q"), k.data_ptr(), v.data_ptr(), kvd, L.ptr(valid), L.ptr(active),
            m.data_ptr(), l.data_ptr(), acc.data_ptr(), block_mass.data_ptr(), max_blocks, int(block_id_offset),
            int(tokens_per_block), B, Hq, Hkv, T, D, float(scale), float(softcap or 0.0), _BACKEND,
            scratch.data_ptr(), scratch.numel(), L.stream_of(q)))


def streaming_attention_fold_fixed_step(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    m: torch.Tensor,
    l: torch.Tensor,
    acc: torch.Tensor,
    valid: torch.Tensor | None = None,
    scale: float | None = None,
    softcap: float | None = None,
) -> None:
    """Pass-2 fold of a non-block chunk (the tail): acc only, no mass (streaming_attention.py:624-665)."""
    B, Hq, Hkv, T, D = _common(q, k)
    _require_cuda(q=q, k=k, v=v, m=m, l=l, acc=acc, valid=valid)
    _state(m, "m", (B, Hq))
    _state(l, "l", (B, Hq))
    _state(acc, "acc", (B, Hq, D))
    if scale is None:
        scale = 1.0 / (D**0.5)
    q, k, v = q.contiguous(), _aligned(k), _aligned(v)
    valid = _mask(valid)
    kvd = _dtype_code(k, "k")
    lib = L.lib()
    with torch.cuda.device(q.device):
        nbytes = lib.pager_attn_chunk_scratch_bytes(3, B, Hq, Hkv, T, D, kvd, 16)
        scratch = _scratch(nbytes, q.device)
        L.check(lib.pager_attn_fold_fixed_step(
            q.data_ptr(), _dtype_code(q, "q"), k.data_ptr(), v.data_ptr(), kvd, L.ptr(valid), m.data_ptr(),
            l.data_ptr(), acc.data_ptr(), B, Hq, Hkv, T, D, float(scale), float(softcap or 0.0), _BACKEND,
            scratch.data_ptr(), scratch.numel(), L.stream_of(q)))


def streaming_attention_finalize(acc: torch.Tensor, l: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """(acc / l).to(dtype), once every chunk has been folded in (streaming_attention.py:668-670)."""
    _require_cuda(acc=acc, l=l)
    if dtype not in L.DTYPE_CODE:
        raise ValueError(f"finalize dtype must be float32, float16 or bfloat16, got {dtype}")
    acc = acc.float().contiguous()
    l = l.float().contiguous()
    out = torch.empty(acc.shape, dtype=dtype, device=acc.device)
    rows = acc.numel() // acc.shape[-1] if acc.numel() else 0
    with torch.cuda.device(acc.device):
        L.check(L.lib().pager_attn_finalize(acc.data_ptr(), l.data_ptr(), out.data_ptr(), L.DTYPE_CODE[dtype], rows,
                                            acc.shape[-1], L.stream_of(acc)))
    return out


_MASS_MODES = {"none": L.MASS_NONE, "row_mean": L.MASS_ROW_MEAN, "batch_mean": L.MASS_BATCH_MEAN}


def paged_decode_attention(
    q: torch.Tensor,
    block_table: torch.Tensor,
    num_blocks: torch.Tensor,
    *,
    dev_pool: torch.Tensor | None,
    host_pool: torch.Tensor | None,
    num_layers: int,
    layer: int,
    tokens_per_block: int,
    max_row_tokens: int,
    tail_k: torch.Tensor | None = None,
    tail_v: torch.Tensor | None = None,
    tail_len: torch.Tensor | None = None,
    valid_lo: torch.Tensor | None = None,
    valid_hi: torch.Tensor | None = None,
    active: torch.Tensor | None = None,
    scale: float | None = None,
    softcap: float | None = None,
    out: torch.Tensor | None = None,
    block_mass: torch.Tensor | None = None,
    mass_accum: torch.Tensor | None = None,
    mass_mode: str = "none",
    scratch: torch.Tensor | None = None,
    rounding: str = "one_pass",
    ref_group_tokens: int = 0,
    ref_shift: torch.Tensor | None = None,
    ref_tail_start: torch.Tensor | None = None,
) -> torch.Tensor:
    """Fused decode attention over a block table, in one pass.

    Replaces, per layer, the group loop of PagedModel._build_streaming_layer_forward
    (paged_model.py:993-1072) and batched_decode_step's layer forward
    (batched_decode.py:238-287), including the per-block gather
    (paged_model.py:878-924).

    q [B, Hq, D]; dev_pool [dev_slots, L, 2, Hkv, tpb, D] (CUDA) and host_pool
    [host_slots, L, 2, Hkv, tpb, D] (pinned, device-mapped host memory; see
    ``host_pool.HostPool``); block_table [B, max_blocks] int32 with
    entries slot (device), slot | HOST_SLOT_BIT (host) or -1 (absent);
    num_blocks [B]; tail_k/tail_v [B, Hkv, tail_cap, D] with tail_len [B];
    valid_lo/valid_hi [B] bound the attended tokens (left padding, sliding
    window).  Returns out [B, Hq, D] in q's dtype.  Mass: ``block_mass``
    [B, Hq, max_blocks] receives sum(p over block)/l per head (the two-pass
    reference's block_mass); ``mass_accum`` += the head mean ("row_mean",
    [B, max_blocks]) or the batch-and-head mean ("batch_mean", [max_blocks]).

    ``rounding``: how p is rounded to the KV dtype before P.V.  "one_pass" is the
    fused one-pass kernel (p against split-local running maxima).  "running" and
    "final" round exactly as the reference does -- against its running max after
    each 64-token tile of the chunks it is handed (its one-pass path for
    recent_only / sinks_recent), or against the row's final max (its two-pass path
    for the heavy-hitter policies) -- by a K pass to scores, a scan and a V pass
    (include/pager_b200.h, PAGER_ROUND_*).  The reference's chunks for "running":
    groups of ``ref_group_tokens`` tokens (streaming_group_size_blocks *
    tokens_per_block; 0: one chunk) of a numbering in which row b's token j sits at
    ``ref_shift[b] + j``, then the tail chunk from row token ``ref_tail_start[b]``
    (default num_blocks[b] * tokens_per_block).
    """
    if q.dim() != 3:
        raise ValueError(f"q must be [batch, heads, dim], got {tuple(q.shape)}")
    B, Hq, D = q.shape
    pool = dev_pool if dev_pool is not None else host_pool
    if pool is None:
        raise ValueError("at least one of dev_pool / host_pool is required")
    if pool.dim() != 6 or pool.shape[1] != num_layers or pool.shape[2] != 2 or pool.shape[4] != tokens_per_block or \
            pool.shape[5] != D:
        raise ValueError(f"pool must be [slots, {num_layers}, 2, kv_heads, {tokens_per_block}, {D}], got "
                         f"{tuple(pool.shape)}")
    Hkv = pool.shape[3]
    if Hq % Hkv:
        raise ValueError(f"num_query_heads ({Hq}) is not a multiple of num_kv_heads ({Hkv})")
    _validate_n_rep(Hq // Hkv)
    for other in (dev_pool, host_pool):
        if other is not None and (tuple(other.shape[1:]) != tuple(pool.shape[1:]) or other.dtype != pool.dtype):
            raise ValueError("dev_pool and host_pool must share layout and dtype")
    _require_cuda(q=q, block_table=block_table, num_blocks=num_blocks, dev_pool=dev_pool, tail_k=tail_k,
                  tail_v=tail_v, tail_len=tail_len, valid_lo=valid_lo, valid_hi=valid_hi, active=active,
                  out=out, block_mass=block_mass, mass_accum=mass_accum)
    if host_pool is not None and host_pool.is_cuda:
        raise ValueError("host_pool must be pinned host memory")
    if block_table.dtype != torch.int32 or block_table.dim() != 2 or block_table.shape[0] != B:
        raise ValueError("block_table must be int32 [batch, max_blocks]")
    block_table = block_table.contiguous()
    max_blocks = block_table.shape[1]
    num_blocks = _mask(num_blocks)
    tail_cap = 0
    if tail_len is not None:
        if tail_k is None or tail_v is None or tail_k.shape != tail_v.shape or tail_k.dim() != 4:
            raise ValueError("tail_k / tail_v must be [batch, kv_heads, tail_cap, head_dim]")
        if tail_k.dtype != pool.dtype:
            raise ValueError("tail tensors must share the pool dtype")
        tail_k, tail_v = _aligned(tail_k), _aligned(tail_v)
        tail_cap = tail_k.shape[2]
        tail_len = _mask(tail_len)
    valid_lo, valid_hi, active = _mask(valid_lo), _mask(valid_hi), _mask(active)
    if scale is None:
        scale = 1.0 / (D**0.5)
    if out is None:
        out = torch.empty((B, Hq, D), dtype=q.dtype, device=q.device)
    elif tuple(out.shape) != (B, Hq, D) or not out.is_contiguous():
        raise ValueError("out must be a contiguous [batch, heads, dim] tensor")
    if block_mass is not None:
        _state(block_mass, "block_mass", (B, Hq, max_blocks))
    mode = _MASS_MODES[mass_mode]
    if mode == L.MASS_ROW_MEAN:
        _state(mass_accum, "mass_accum", (B, max_blocks))
    elif mode == L.MASS_BATCH_MEAN:
        _state(mass_accum, "mass_accum", (max_blocks,))
    q = q.contiguous()
    kvd = _dtype_code(pool, "pool")
    rcode = _rounding_code(rounding)
    ref_shift, ref_tail_start = _mask(ref_shift), _mask(ref_tail_start)
    _require_cuda(ref_shift=ref_shift, ref_tail_start=ref_tail_start)
    lib = L.lib()
    with torch.cuda.device(q.device):
        nbytes = lib.pager_paged_decode_scratch_bytes_rounded(B, Hq, Hkv, D, kvd, tokens_per_block,
                                                              int(max_row_tokens), rcode)
        if scratch is None or scratch.numel() < nbytes:
            scratch = _scratch(nbytes, q.device)
        L.check(lib.pager_paged_decode_attention_rounded(
            q.data_ptr(), _dtype_code(q, "q"), L.ptr(dev_pool), 0 if dev_pool is None else dev_pool.shape[0],
            L.ptr(host_pool), 0 if host_pool is None else host_pool.shape[0], None, 0, kvd, num_layers, layer, Hkv,
            tokens_per_block, D, block_table.data_ptr(), max_blocks, num_blocks.data_ptr(), L.ptr(tail_k),
            L.ptr(tail_v), L.ptr(tail_len), tail_cap, L.ptr(valid_lo), L.ptr(valid_hi), L.ptr(active), B, Hq,
            float(scale), float(softcap or 0.0), int(max_row_tokens), out.data_ptr(), _dtype_code(out, "out"),
            L.ptr(block_mass), L.ptr(mass_accum), mode, _BACKEND, rcode, int(ref_group_tokens), L.ptr(ref_shift),
            L.ptr(ref_tail_start), scratch.data_ptr(), scratch.numel(), L.stream_of(q)))
    return out


def _rounding_code(rounding: str) -> int:
    try:
        return L.ROUNDING_CODE[rounding]
    except KeyError:
        raise ValueError(f"rounding must be 'one_pass', 'running' or 'final', got {rounding!r}") from None


class PagedDecodePlan:
    """A validated, reusable call of ``paged_decode_attention`` for one decode step.

    Everything that is fixed across the layers of a step (pools, block table,
    row lengths, tails, ranges, scratch) is checked and bound once; each
    ``run(q, layer, out)`` then goes straight to the C ABI.  This keeps the
    per-layer host cost at one ctypes call, so a step can also be captured in a
    CUDA graph.
    """

    def __init__(self, *, batch, num_query_heads, dev_pool, host_pool, num_layers, tokens_per_block, block_table,
                 num_blocks, max_row_tokens, tail_k=None, tail_v=None, tail_len=None, valid_lo=None, valid_hi=None,
                 active=None, scale=None, softcap=None, q_dtype=None, block_mass=None, mass_accum=None,
                 mass_mode="none", host_read="auto", prefetch_next_step=False, rounding="one_pass",
                 ref_group_tokens=0, ref_shift=None, ref_tail_start=None):
        pool = dev_pool if dev_pool is not None else host_pool
        if pool is None or pool.dim() != 6:
            raise ValueError("a [slots, layers, 2, kv_heads, tokens_per_block, head_dim] pool is required")
        self.B, self.Hq = int(batch), int(num_query_heads)
        self.Hkv, self.D = pool.shape[3], pool.shape[5]
        if self.Hq % self.Hkv:
            raise ValueError(f"num_query_heads ({self.Hq}) is not a multiple of num_kv_heads ({self.Hkv})")
        _validate_n_rep(self.Hq // self.Hkv)
        device = block_table.device
        _require_cuda(block_table=block_table, num_blocks=num_blocks, dev_pool=dev_pool, tail_k=tail_k, tail_v=tail_v,
                      tail_len=tail_len, valid_lo=valid_lo, valid_hi=valid_hi, active=active,
                      block_mass=block_mass, mass_accum=mass_accum)
        if block_table.dtype != torch.int32 or tuple(block_table.shape[:1]) != (self.B,):
            raise ValueError("block_table must be int32 [batch, max_blocks]")
        _require_cuda(ref_shift=ref_shift, ref_tail_start=ref_tail_start)
        self._keep = [block_table.contiguous(), _mask(num_blocks), _mask(tail_len), _mask(valid_lo), _mask(valid_hi),
                      _mask(active), _mask(ref_shift), _mask(ref_tail_start), dev_pool, host_pool]
        (self.block_table, self.num_blocks, self.tail_len, self.valid_lo, self.valid_hi, self.active, self.ref_shift,
         self.ref_tail_start) = self._keep[:8]
        self.rounding = _rounding_code(rounding)
        self.ref_group_tokens = int(ref_group_tokens)
        self.tail_k = None if tail_k is None else _aligned(tail_k)
        self.tail_v = None if tail_v is None else _aligned(tail_v)
        self._keep += [self.tail_k, self.tail_v]
        self.dev_pool, self.host_pool = dev_pool, host_pool
        self.num_layers, self.tpb = int(num_layers), int(tokens_per_block)
        self.max_blocks = self.block_table.shape[1]
        self.max_row_tokens = int(max_row_tokens)
        self.scale = float(scale if scale is not None else 1.0 / (self.D**0.5))
        self.softcap = float(softcap or 0.0)
        self.kv_dtype = _dtype_code(pool, "pool")
        self.q_dtype = self.kv_dtype if q_dtype is None else L.DTYPE_CODE[q_dtype]
        self.block_mass, self.mass_accum = block_mass, mass_accum
        self.mass_mode = _MASS_MODES[mass_mode]
        lib = L.lib()
        with torch.cuda.device(device):
            nbytes = lib.pager_paged_decode_scratch_bytes_rounded(self.B, self.Hq, self.Hkv, self.D, self.kv_dtype,
                                                                  self.tpb, self.max_row_tokens, self.rounding)
        self.scratch = _scratch(nbytes, device)
        self.device = device
        self._fn = lib.pager_paged_decode_attention_rounded
        self._static = (
            L.ptr(dev_pool), 0 if dev_pool is None else dev_pool.shape[0], L.ptr(host_pool),
            0 if host_pool is None else host_pool.shape[0], self.kv_dtype, self.num_layers)
        # host tier: zero-copy reads, or staged per layer by the copy engines (host_staging.py)
        self.staging = None
        if host_read not in ("auto", "zero_copy", "staged"):
            raise ValueError(f"host_read must be 'auto', 'zero_copy' or 'staged', got {host_read!r}")
        if host_pool is not None and host_read != "zero_copy":
            tbl = self.block_table
            has_host = bool(((tbl >= 0) & ((tbl & L.HOST_SLOT_BIT) != 0)).any())
            if has_host:
                from .host_staging import HostStaging, choose_host_read, plan_host_runs

                plan = plan_host_runs(tbl, self.tpb, self.num_blocks, self.valid_lo, self.valid_hi, self.active)
                n_slots, n_runs = int(plan[1].numel()), len(plan[2][0])
                mode = "staged"
                if host_read == "auto":
                    chunk = 2 * host_pool.shape[3] * host_pool.shape[4] * host_pool.shape[5] * host_pool.element_size()
                    mode = choose_host_read(device, n_slots * chunk, n_runs)
                if mode == "staged" and n_slots > 0:  # with no host block read there is nothing to stage
                    self.staging = HostStaging(tbl, host_pool, self.num_layers, device, prefetch_next_step,
                                               self.tpb, self.num_blocks, self.valid_lo, self.valid_hi, self.active,
                                               plan=plan)
        self.host_read = "staged" if self.staging is not None else "zero_copy"

    def run(self, q: torch.Tensor, layer: int, out: torch.Tensor, stream: int | None = None) -> torch.Tensor:
        dp, ds, hp, hs, kvd, nl = self._static
        stg = self.staging
        if stg is None:
            sp, ss, table = None, 0, self.block_table
            sh = torch.cuda.current_stream(self.device).cuda_stream if stream is None else stream
        else:
            st = (torch.cuda.current_stream(self.device) if stream is None
                  else torch.cuda.ExternalStream(stream, device=self.device))
            sp, ss, table, sh = stg.before_kernel(layer, st).data_ptr(), stg.num_slots, stg.table, st.cuda_stream
        rc = self._fn(
            q.data_ptr(), self.q_dtype, dp, ds, hp, hs, sp, ss, kvd, nl, layer, self.Hkv, self.tpb, self.D,
            table.data_ptr(), self.max_blocks, self.num_blocks.data_ptr(), L.ptr(self.tail_k),
            L.ptr(self.tail_v), L.ptr(self.tail_len), 0 if self.tail_k is None else self.tail_k.shape[2],
            L.ptr(self.valid_lo), L.ptr(self.valid_hi), L.ptr(self.active), self.B, self.Hq, self.scale, self.softcap,
            self.max_row_tokens, out.data_ptr(), L.DTYPE_CODE[out.dtype], L.ptr(self.block_mass),
            L.ptr(self.mass_accum), self.mass_mode, _BACKEND, self.rounding, self.ref_group_tokens,
            L.ptr(self.ref_shift), L.ptr(self.ref_tail_start), self.scratch.data_ptr(), self.scratch.numel(), sh)
        if stg is not None:
            stg.after_kernel(layer, st)
        if rc:
            L.check(rc)
        return out
