"""Cross-session batched decode (``pager_hf/batched_decode.py``) against the oracle.

Sessions with ragged histories (a tail-only prompt, a prompt of exactly one
block, longer ones), unequal tails, one with a sliding window and mixed pager
policies decode 20 steps together: tails roll into blocks, pagers move blocks
to the host pool, and every layer's output and every session's block
attention must match the reference's per-session decode (the two-pass
sequence of ``paged_model.py:993-1072`` restated in the oracle) on that
session's full token history; each session's pager must reach the same
placement as the oracle pager fed the same attention
(``batched_decode.py:320-338``).
"""

import numpy as np
import pytest
import torch

from oracle import pager_core_oracle as porc
from oracle import streaming_attention_oracle as orc

pytestmark = pytest.mark.gpu

BLOCK = 16 * 1024 * 1024


def _np(t):
    return t.detach().float().cpu().numpy()


def _expected_attention(mass_sum, num_layers, num_blocks_after):
    """``_finalize_streaming_block_attention`` (paged_model.py:865-876) on the oracle's masses."""
    if mass_sum is None or num_blocks_after == 0:
        return [1.0 / num_blocks_after] * num_blocks_after if num_blocks_after else []
    averaged = (mass_sum / num_layers).tolist()
    total = sum(averaged)
    if total <= 0:
        return [1.0 / num_blocks_after] * num_blocks_after
    return [x / total for x in averaged]


def test_batched_decode_matches_per_session_reference():
    from pager_hf import _lib
    from pager_hf.batched_decode import BatchedDecodeAttention, DecodeSession
    from pager_hf.kv_block_store import KVPools

    g = torch.Generator().manual_seed(11)
    L, Hq, Hkv, D, tpb, dt = 2, 8, 2, 64, 16, torch.float16
    pools = KVPools(num_layers=L, kv_heads=Hkv, head_dim=D, tokens_per_block=tpb, dtype=dt, device="cuda",
                    gpu_groups=4, cpu_groups=2)
    prompts = [37, 16, 5, 70]
    windows = [None, None, None, 24]
    policies = ["sinks_heavy_hitter", "recent_only", "heavy_hitter", "heavy_hitter"]
    sessions, hist_k, hist_v, ref_pagers = [], [], [], []
    for T, w, pol in zip(prompts, windows, policies):
        ks = [torch.randn(1, Hkv, T, D, generator=g).to(dt) for _ in range(L)]
        vs = [torch.randn(1, Hkv, T, D, generator=g).to(dt) for _ in range(L)]
        kw = dict(vram=3 * BLOCK, ram=100 * BLOCK, recent=1, rebalance_interval=2, promote_margin=0.05,
                  ram_promote_margin=0.2, policy=pol)
        s = DecodeSession(pools, pager_kwargs=kw, sliding_window=w)
        s.prefill([k.cuda() for k in ks], [v.cuda() for v in vs])
        sessions.append(s)
        hist_k.append([k[0] for k in ks])  # per layer [Hkv, T, D] on the CPU
        hist_v.append([v[0] for v in vs])
        ref_pagers.append(porc.Pager(3 * BLOCK, 100 * BLOCK, 1, 2, 0.05, 0.2, pol))
    S = len(sessions)
    saw_host = False
    for step in range(20):
        plan = BatchedDecodeAttention(sessions, Hq)
        saw_host |= bool(((plan.table >= 0) & ((plan.table & 0x40000000) != 0)).any())
        nb_before = [s.num_blocks for s in sessions]
        mass_sum = [np.zeros(max(nb, 1), np.float64) for nb in nb_before]
        new_k, new_v = [], []
        for layer in range(L):
            q = torch.randn(S, Hq, D, generator=g).to(dt)
            kn = torch.randn(S, Hkv, D, generator=g).to(dt)
            vn = torch.randn(S, Hkv, D, generator=g).to(dt)
            new_k.append(kn)
            new_v.append(vn)
            out = plan.layer(layer, q.cuda(), kn.cuda(), vn.cuda())
            torch.cuda.synchronize()
            for r in range(S):
                k_all = torch.cat([hist_k[r][layer], kn[r][:, None]], dim=1)  # [Hkv, T+1, D]
                v_all = torch.cat([hist_v[r][layer], vn[r][:, None]], dim=1)
                nb = nb_before[r]
                full, total = nb * tpb, k_all.shape[1]
                valid = np.ones((1, total), np.int32)
                if windows[r] is not None:
                    valid[0, :max(0, total - windows[r])] = 0
                ref_out, ref_mass, _, _ = orc.two_pass_decode(
                    _np(q[r:r + 1]), _np(k_all[None, :, :full]), _np(v_all[None, :, :full]),
                    _np(k_all[None, :, full:]), _np(v_all[None, :, full:]), nb, tpb, max(nb, 1),
                    valid=valid[:, :full], tail_valid=valid[:, full:], v_dtype="f16", out_dtype="f16")
                np.testing.assert_allclose(_np(out[r]), ref_out[0], rtol=0, atol=2e-3,
                                           err_msg=f"step {step} layer {layer} row {r}")
                if nb:
                    mass_sum[r] += ref_mass[0][:, :nb].mean(0)
        attention = plan.finish()
        for r, s in enumerate(sessions):
            for layer in range(L):
                hist_k[r][layer] = torch.cat([hist_k[r][layer], new_k[layer][r][:, None]], dim=1)
                hist_v[r][layer] = torch.cat([hist_v[r][layer], new_v[layer][r][:, None]], dim=1)
            assert s.num_tokens == hist_k[r][0].shape[1]
            added = s.num_blocks > nb_before[r]
            if s.num_blocks == 0:
                assert attention[r] == []
                continue
            if s.needs_attention:
                want = _expected_attention(mass_sum[r][:nb_before[r]] if nb_before[r] else None, L, s.num_blocks)
            else:
                want = [1.0 / s.num_blocks] * s.num_blocks
            assert len(attention[r]) == len(want), (step, r)
            np.testing.assert_allclose(attention[r], want, rtol=2e-4, atol=1e-6, err_msg=f"step {step} row {r}")
            # replay the reference's post-step pager calls on the oracle pager with the same attention
            ref = ref_pagers[r]
            ref.on_step(s.num_blocks - 1, 0, attention[r])
            if added:
                ref.force_rebalance(s.num_blocks - 1)
            assert s.pager.tiers() == ref.tiers(), (step, r)
            assert s.store.gpu_block_ids() == [i for i, t in enumerate(ref.tiers()) if t == 0 and i < s.num_blocks]
    assert saw_host, "the pagers never moved a block to the host pool"
    assert _lib.device_status(0) == 0
    for s in sessions:
        s.close()
    pools.close()


def test_sessions_must_share_pools_and_be_single_row():
    from pager_hf.batched_decode import BatchedDecodeAttention, DecodeSession
    from pager_hf.kv_block_store import KVPools

    a = KVPools(num_layers=1, kv_heads=2, head_dim=64, tokens_per_block=16, dtype=torch.float16, device="cuda")
    b = KVPools(num_layers=1, kv_heads=2, head_dim=64, tokens_per_block=16, dtype=torch.float16, device="cuda")
    wide = KVPools(num_layers=1, kv_heads=2, head_dim=64, tokens_per_block=16, dtype=torch.float16, device="cuda",
                   rows_per_group=2)
    with pytest.raises(ValueError):
        DecodeSession(wide)
    s1, s2 = DecodeSession(a), DecodeSession(b)
    with pytest.raises(ValueError):
        BatchedDecodeAttention([s1, s2], 8)
    with pytest.raises(ValueError):
        BatchedDecodeAttention([], 8)
    for p in (a, b, wide):
        p.close()
