"""CPU oracle for the streaming decode-attention hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the shipped package imports this module:
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may use it, and only as the checker (or the timed CPU reference arm),
never as the thing measured on the GPU.

This is a numpy restatement of the algorithm in rust-llm-pager's
``pager_hf/streaming_attention.py`` (the four Triton kernels and their
wrappers) and of the call sequence ``pager_hf/paged_model.py`` runs around
them.  Each function cites the reference lines it follows.  Parity of this
restatement is pinned against vectors produced by the reference's own
Triton kernels run on the CPU (``TRITON_INTERPRET=1``), committed under
``tests/golden/`` together with the script that made them.

Arithmetic follows the reference exactly where it matters for the result:

* scores are an fp32 dot product of the (fp16/bf16/fp32) inputs, times
  ``scale``, then optional softcap ``c*tanh(s/c)``, then the token mask
  (``-inf``) -- streaming_attention.py:158-161;
* the online update guards the "nothing valid yet" case with alpha=0/p=0
  (streaming_attention.py:171-177);
* ``p`` is rounded to the value dtype before the P.V product
  (``p.to(v_chunk.dtype)``, streaming_attention.py:178, :347, :428);
  ``l`` and the block mass sum the unrounded fp32 ``p``;
* the one-pass kernel walks the chunk in ``_BLOCK_KV = 64``-token tiles
  (streaming_attention.py:11, :143), the accumulate kernel in
  ``tokens_per_block`` tiles (:325-327).

bf16 has no numpy dtype: bf16 data is carried as float32 arrays holding
bf16-representable values, and ``round_to(x, "bf16")`` rounds to nearest even.
"""

from __future__ import annotations

import numpy as np

BLOCK_KV = 64  # streaming_attention.py:11
M_TILE = 16  # streaming_attention.py:55 (n_rep guard)

_F32 = np.float32


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to ``dtype`` ("f32", "f16", "bf16") and return float32."""
    x = np.asarray(x, dtype=_F32)
    if dtype == "f32":
        return x
    if dtype == "f16":
        return x.astype(np.float16).astype(_F32)
    if dtype == "bf16":
        bits = x.view(np.uint32).astype(np.uint64)
        nan = np.isnan(x)
        # round to nearest, ties to even, on the upper 16 bits
        rounded = (bits + 0x7FFF + ((bits >> 16) & 1)) & 0xFFFF0000
        out = rounded.astype(np.uint32).view(_F32).copy()
        out[nan] = np.nan
        return out
    raise ValueError(f"unknown dtype {dtype!r}")


def validate_n_rep(n_rep: int) -> None:
    """streaming_attention.py:69-74 -- GQA fan-out above M_TILE is rejected."""
    if n_rep > M_TILE:
        raise NotImplementedError(f"n_rep up to {M_TILE} supported, got {n_rep}")


def state_init(batch: int, num_query_heads: int, head_dim: int):
    """streaming_attention.py:444-449."""
    m = np.full((batch, num_query_heads), -np.inf, dtype=_F32)
    l = np.zeros((batch, num_query_heads), dtype=_F32)
    acc = np.zeros((batch, num_query_heads, head_dim), dtype=_F32)
    return m, l, acc


def finalize(acc: np.ndarray, l: np.ndarray, dtype: str) -> np.ndarray:
    """streaming_attention.py:668-670: ``(acc / l).to(dtype)``."""
    with np.errstate(divide="ignore", invalid="ignore"):
        return round_to(acc / l[..., None], dtype)


def _grouped(q, k, v, num_kv_heads):
    batch, hq, d = q.shape
    n_rep = hq // num_kv_heads
    validate_n_rep(n_rep)
    qg = np.asarray(q, _F32).reshape(batch, num_kv_heads, n_rep, d)
    kk = np.asarray(k, _F32)
    vv = None if v is None else np.asarray(v, _F32)
    return qg, kk, vv, n_rep


def _scores(qg, k_chunk, mask, scale, softcap):
    """streaming_attention.py:158-161 for a [B,Hkv,n_rep,D] x [B,Hkv,t,D] tile."""
    k_chunk = np.where(mask[:, None, :, None], k_chunk, _F32(0))
    s = np.matmul(qg, np.swapaxes(k_chunk, -1, -2)).astype(_F32) * _F32(scale)
    if softcap:
        s = (_F32(softcap) * np.tanh(s / _F32(softcap))).astype(_F32)
    return np.where(mask[:, None, None, :], s, _F32(-np.inf)).astype(_F32)


def _defaults(k, valid, active, scale, head_dim):
    batch, _, tokens, _ = k.shape
    if valid is None:
        valid = np.ones((batch, tokens), dtype=np.int32)  # :433-436
    if active is None:
        active = np.ones((batch,), dtype=np.int32)  # :439-441
    if scale is None:
        scale = 1.0 / (head_dim**0.5)  # :491-492
    return np.asarray(valid), np.asarray(active), scale


def step(q, k, v, m, l, acc, valid=None, active=None, scale=None, softcap=None, v_dtype="f32"):
    """One-pass fold of a chunk into (m, l, acc), in place.

    Follows ``_decode_attention_step_kernel`` (streaming_attention.py:77-185)
    and its wrapper ``streaming_attention_step`` (:452-513).
    """
    batch, hq, d = q.shape
    hkv, tokens = k.shape[1], k.shape[2]
    qg, kk, vv, n_rep = _grouped(q, k, v, hkv)
    valid, active, scale = _defaults(k, valid, active, scale, d)
    mg = m.reshape(batch, hkv, n_rep).copy()
    lg = l.reshape(batch, hkv, n_rep).copy()
    ag = acc.reshape(batch, hkv, n_rep, d).copy()
    act = active != 0
    with np.errstate(invalid="ignore", over="ignore"):
        for start in range(0, tokens, BLOCK_KV):  # :143
            end = min(start + BLOCK_KV, tokens)
            mask = (valid[:, start:end] != 0) & act[:, None]  # :144-147
            s = _scores(qg, kk[:, :, start:end], mask, scale, softcap)
            chunk_max = s.max(axis=-1)  # :163
            m_new = np.maximum(mg, chunk_max)  # :164
            empty = m_new == -np.inf  # :171
            alpha = np.where(empty, _F32(0), np.exp(mg - m_new)).astype(_F32)  # :172
            p = np.where(empty[..., None], _F32(0), np.exp(s - m_new[..., None])).astype(_F32)  # :177
            vc = np.where(mask[:, None, :, None], vv[:, :, start:end], _F32(0))
            pv = np.matmul(round_to(p, v_dtype), vc).astype(_F32)  # :178
            upd = act[:, None, None]
            ag = np.where(upd[..., None], ag * alpha[..., None] + pv, ag).astype(_F32)  # :174, :178
            lg = np.where(upd, lg * alpha + p.sum(axis=-1, dtype=_F32), lg).astype(_F32)  # :175, :179
            mg = np.where(upd, m_new, mg).astype(_F32)  # :181
    m[...] = mg.reshape(batch, hq)
    l[...] = lg.reshape(batch, hq)
    acc[...] = ag.reshape(batch, hq, d)


def stats_step(q, k, m, l, valid=None, active=None, scale=None, softcap=None):
    """Pass 1: fold a chunk's K into (m, l) only.

    ``_decode_attention_stats_kernel`` (streaming_attention.py:188-261),
    wrapper ``streaming_attention_stats_step`` (:516-560).
    """
    batch, hq, d = q.shape
    hkv, tokens = k.shape[1], k.shape[2]
    qg, kk, _, n_rep = _grouped(q, k, None, hkv)
    valid, active, scale = _defaults(k, valid, active, scale, d)
    mg = m.reshape(batch, hkv, n_rep).copy()
    lg = l.reshape(batch, hkv, n_rep).copy()
    act = active != 0
    with np.errstate(invalid="ignore", over="ignore"):
        for start in range(0, tokens, BLOCK_KV):  # :234
            end = min(start + BLOCK_KV, tokens)
            mask = (valid[:, start:end] != 0) & act[:, None]
            s = _scores(qg, kk[:, :, start:end], mask, scale, softcap)
            m_new = np.maximum(mg, s.max(axis=-1))  # :251-252
            empty = m_new == -np.inf  # :255
            l_new = lg * np.where(empty, _F32(0), np.exp(mg - m_new))  # :256
            l_new = l_new + np.where(empty[..., None], _F32(0), np.exp(s - m_new[..., None])).sum(
                axis=-1, dtype=_F32
            )  # :257
            upd = act[:, None, None]
            lg = np.where(upd, l_new, lg).astype(_F32)
            mg = np.where(upd, m_new, mg).astype(_F32)
    m[...] = mg.reshape(batch, hq)
    l[...] = lg.reshape(batch, hq)


def accumulate_step(
    q, k, v, m, l, acc, block_mass, block_id_offset, tokens_per_block,
    valid=None, active=None, scale=None, softcap=None, v_dtype="f32",
):
    """Pass 2: acc += P.V with final (m, l); write per-block attention mass.

    ``_decode_attention_accumulate_kernel`` (streaming_attention.py:264-352),
    wrapper ``streaming_attention_accumulate_step`` (:563-621).  The mass of
    local block j is ``sum(p over the block's tokens) / l_final`` (:349-350);
    rows with active=0 leave acc and block_mass untouched (:322-325).
    """
    batch, hq, d = q.shape
    hkv, tokens = k.shape[1], k.shape[2]
    qg, kk, vv, n_rep = _grouped(q, k, v, hkv)
    valid, active, scale = _defaults(k, valid, active, scale, d)
    max_blocks = block_mass.shape[2]
    mg = m.reshape(batch, hkv, n_rep)
    lg = l.reshape(batch, hkv, n_rep)
    ag = acc.reshape(batch, hkv, n_rep, d).copy()
    bm = block_mass.reshape(batch, hkv, n_rep, max_blocks)
    act = active != 0
    num_local = (tokens + tokens_per_block - 1) // tokens_per_block  # :323
    with np.errstate(invalid="ignore", over="ignore", divide="ignore"):
        for j in range(num_local):  # :325
            start = j * tokens_per_block
            end = min(start + tokens_per_block, tokens)
            mask = valid[:, start:end] != 0
            s = _scores(qg, kk[:, :, start:end], mask, scale, softcap)
            p = np.exp(s - mg[..., None]).astype(_F32)  # :346
            vc = np.where(mask[:, None, :, None], vv[:, :, start:end], _F32(0))
            pv = np.matmul(round_to(p, v_dtype), vc).astype(_F32)  # :347
            upd = act[:, None, None]
            ag = np.where(upd[..., None], ag + pv, ag).astype(_F32)
            mass = (p.sum(axis=-1, dtype=_F32) / lg).astype(_F32)  # :349
            col = block_id_offset + j
            bm[:, :, :, col] = np.where(upd, mass, bm[:, :, :, col])  # :350
    acc[...] = ag.reshape(batch, hq, d)


def fold_fixed_step(q, k, v, m, l, acc, valid=None, scale=None, softcap=None, v_dtype="f32"):
    """Pass-2 fold of the non-block tail: acc only, no mass, no active switch.

    ``_decode_attention_fold_fixed_kernel`` (streaming_attention.py:355-430),
    wrapper ``streaming_attention_fold_fixed_step`` (:624-665).
    """
    batch, hq, d = q.shape
    hkv, tokens = k.shape[1], k.shape[2]
    qg, kk, vv, n_rep = _grouped(q, k, v, hkv)
    valid, _, scale = _defaults(k, valid, None, scale, d)
    mg = m.reshape(batch, hkv, n_rep)
    ag = acc.reshape(batch, hkv, n_rep, d).copy()
    with np.errstate(invalid="ignore", over="ignore"):
        for start in range(0, tokens, BLOCK_KV):  # :407
            end = min(start + BLOCK_KV, tokens)
            mask = valid[:, start:end] != 0
            s = _scores(qg, kk[:, :, start:end], mask, scale, softcap)
            p = np.exp(s - mg[..., None]).astype(_F32)  # :427
            vc = np.where(mask[:, None, :, None], vv[:, :, start:end], _F32(0))
            ag = (ag + np.matmul(round_to(p, v_dtype), vc)).astype(_F32)  # :428
    acc[...] = ag.reshape(batch, hq, d)


def dense_reference(q, k, v, n_rep, tokens_per_block, valid=None, scale=None, softcap=None):
    """Dense GQA decode attention with per-block mass.

    Restates ``_dense_reference`` of the reference's
    tests/test_streaming_attention.py:20-40 (repeat_interleave GQA, fp32,
    softcap, mask, softmax, per-``tokens_per_block`` mass incl. a ragged last
    block).  Used for softcap cases and as the CPU timing baseline shape.
    """
    q = np.asarray(q, _F32)
    key = np.repeat(np.asarray(k, _F32), n_rep, axis=1)
    value = np.repeat(np.asarray(v, _F32), n_rep, axis=1)
    if scale is None:
        scale = 1.0 / (q.shape[-1] ** 0.5)
    s = np.einsum("bhd,bhtd->bht", q, key).astype(_F32) * _F32(scale)
    if softcap is not None:
        s = _F32(softcap) * np.tanh(s / _F32(softcap))
    if valid is not None:
        s = np.where(np.asarray(valid)[:, None, :] == 0, -np.inf, s)
    s = s - s.max(axis=-1, keepdims=True)
    w = np.exp(s)
    w = (w / w.sum(axis=-1, keepdims=True)).astype(_F32)
    out = np.einsum("bht,bhtd->bhd", w, value).astype(_F32)
    tokens = k.shape[2]
    nb = (tokens + tokens_per_block - 1) // tokens_per_block
    mass = np.stack(
        [w[:, :, b * tokens_per_block : (b + 1) * tokens_per_block].sum(axis=-1) for b in range(nb)], axis=2
    )
    return out, mass


def two_pass_decode(
    q, k, v, tail_k, tail_v, num_blocks, tokens_per_block, group_size_blocks,
    valid=None, tail_valid=None, scale=None, softcap=None, v_dtype="f32", out_dtype="f32",
):
    """The reference's per-layer mass-tracking decode sequence on gathered KV.

    Follows ``_build_streaming_layer_forward`` in pager_hf/paged_model.py:993-1048:
    pass 1 folds every ``group_size_blocks`` group then the tail into (m, l)
    (:993-1006); pass 2 accumulates each group with its block mass (:1008-1035)
    then folds the tail (:1037-1039); finalize (:1072).  ``k``/``v`` hold the
    ``num_blocks * tokens_per_block`` block tokens, ``tail_k``/``tail_v`` the
    tail including the new token.  Returns (out, block_mass[B,Hq,nb]).
    """
    batch, hq, d = q.shape
    full = num_blocks * tokens_per_block
    if valid is None:
        valid = np.ones((batch, full), dtype=np.int32)
    if tail_valid is None:
        tail_valid = np.ones((batch, tail_k.shape[2]), dtype=np.int32)
    m, l, acc = state_init(batch, hq, d)
    gt = group_size_blocks * tokens_per_block
    for g0 in range(0, full, gt):
        g1 = min(g0 + gt, full)
        stats_step(q, k[:, :, g0:g1], m, l, valid=valid[:, g0:g1], scale=scale, softcap=softcap)
    stats_step(q, tail_k, m, l, valid=tail_valid, scale=scale, softcap=softcap)
    block_mass = np.zeros((batch, hq, max(num_blocks, 1)), dtype=_F32)
    for g0 in range(0, full, gt):
        g1 = min(g0 + gt, full)
        accumulate_step(
            q, k[:, :, g0:g1], v[:, :, g0:g1], m, l, acc, block_mass, g0 // tokens_per_block,
            tokens_per_block, valid=valid[:, g0:g1], scale=scale, softcap=softcap, v_dtype=v_dtype,
        )
    fold_fixed_step(q, tail_k, tail_v, m, l, acc, valid=tail_valid, scale=scale, softcap=softcap, v_dtype=v_dtype)
    return finalize(acc, l, out_dtype), block_mass[:, :, :num_blocks], m, l


def single_pass_decode(
    q, k, v, tail_k, tail_v, num_blocks, tokens_per_block, group_size_blocks,
    valid=None, tail_valid=None, scale=None, softcap=None, v_dtype="f32", out_dtype="f32",
):
    """The reference's per-layer decode sequence for the policies without an attention signal.

    Follows ``_build_streaming_layer_forward`` in pager_hf/paged_model.py:1055-1072 (recent_only,
    sinks_recent): one ``streaming_attention_step`` per group of ``group_size_blocks`` blocks
    (:1055-1067), then one over the tail including the new token (:1068-1070), then finalize
    (:1072).  Each step walks its chunk in 64-token tiles from the chunk's start, so p is rounded
    against the running max after each such tile.  ``k``/``v`` hold the ``num_blocks *
    tokens_per_block`` block tokens; a row padded in front with empty blocks (the combined
    numbering of batched_decode.py:185-234) passes them with valid = 0.  Returns (out, m, l).
    """
    batch, hq, d = q.shape
    full = num_blocks * tokens_per_block
    if valid is None:
        valid = np.ones((batch, full), dtype=np.int32)
    if tail_valid is None:
        tail_valid = np.ones((batch, tail_k.shape[2]), dtype=np.int32)
    m, l, acc = state_init(batch, hq, d)
    gt = group_size_blocks * tokens_per_block
    for g0 in range(0, full, gt):
        g1 = min(g0 + gt, full)
        step(q, k[:, :, g0:g1], v[:, :, g0:g1], m, l, acc, valid=valid[:, g0:g1], scale=scale, softcap=softcap,
             v_dtype=v_dtype)
    step(q, tail_k, tail_v, m, l, acc, valid=tail_valid, scale=scale, softcap=softcap, v_dtype=v_dtype)
    return finalize(acc, l, out_dtype), m, l


def gather_paged_kv(pool_k, pool_v, block_table_row, layer):
    """Gather one row's blocks into contiguous [Hkv, nb*tpb, D] K and V.

    The oracle-side equivalent of ``PagedModel._gather_layer_kv_group``
    (paged_model.py:878-924): per block, the layer slice, permuted to
    [kv_heads, tokens, head_dim], concatenated along tokens.  Pools here are
    indexed [slot, layer, kv_head, token, head_dim].
    """
    ks = [pool_k[s, layer] for s in block_table_row]
    vs = [pool_v[s, layer] for s in block_table_row]
    if not ks:
        shape = (pool_k.shape[2], 0, pool_k.shape[4])
        return np.zeros(shape, _F32), np.zeros(shape, _F32)
    return np.concatenate(ks, axis=1), np.concatenate(vs, axis=1)


def dense_decode_gqa(q, k, v, tail_k, tail_v, tokens_per_block, valid=None, scale=None):
    """Dense decode attention + per-block mass without materialising the GQA repeat.

    The same mathematics as ``dense_reference`` (the reference's dense test
    oracle, tests/test_streaming_attention.py:20-40: softmax over all valid
    tokens, per-``tokens_per_block`` mass) on blocks followed by a tail, with
    the n_rep query heads of a KV head handled as one matrix product per KV
    head.  This is the CPU path the benchmark times as the reference arm.
    q [1, Hq, D]; k/v [1, Hkv, T, D]; tail_k/tail_v [1, Hkv, t, D]; valid [1, T]
    over the block tokens.  Returns (out [1, Hq, D], block_mass [1, Hq, T/tpb]).
    """
    _, hq, d = q.shape
    hkv = k.shape[1]
    n_rep = hq // hkv
    if scale is None:
        scale = 1.0 / (d**0.5)
    qg = np.asarray(q, _F32).reshape(hkv, n_rep, d)
    kk = np.concatenate([k[0], tail_k[0]], axis=1)  # [Hkv, T+t, D]
    vv = np.concatenate([v[0], tail_v[0]], axis=1)
    s = np.matmul(qg, np.swapaxes(kk, 1, 2)) * _F32(scale)  # [Hkv, n_rep, T+t]
    nblk = k.shape[2]
    if valid is not None:
        s[:, :, :nblk][:, :, np.asarray(valid)[0] == 0] = -np.inf
    s -= s.max(axis=-1, keepdims=True)
    np.exp(s, out=s)
    s /= s.sum(axis=-1, keepdims=True)
    out = np.matmul(s, vv).reshape(1, hq, d)
    nb = nblk // tokens_per_block
    mass = s[:, :, : nb * tokens_per_block].reshape(hkv, n_rep, nb, tokens_per_block).sum(-1).reshape(1, hq, nb)
    return out, mass
