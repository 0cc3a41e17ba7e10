"""Full-size GPU checks (32k-token rows, deep pipelines, long splits).

Long splits keep many tiles in flight in the split kernel's stage ring, the
regime where pipeline ordering bugs show up; small parity cases never get
there.  The checker is the CPU oracle's dense decode (oracle/, the
reference's dense test oracle restated) on the same data, plus
size-independent identities: the one-pass step, the two-pass sequence and the
fused paged op agree with each other; masses are non-negative and the block
masses plus the tail's share sum to one.
"""

import numpy as np
import pytest
import torch

from oracle import streaming_attention_oracle as orc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def sa():
    from pager_hf import streaming_attention

    return streaming_attention


@pytest.mark.parametrize("backend", ["auto", "fma"])
def test_32k_contiguous_one_pass_two_pass_and_paged_agree(sa, backend):
    torch.manual_seed(21)
    B, Hq, Hkv, D, tpb, nb = 4, 32, 8, 128, 64, 512
    T = nb * tpb
    dt = torch.bfloat16
    q = torch.randn(B, Hq, D, device="cuda").to(dt)
    k = torch.randn(B, Hkv, T, D, device="cuda").to(dt)
    v = torch.randn(B, Hkv, T, D, device="cuda").to(dt)
    sa.set_backend(backend)
    try:
        m, l, acc = sa.streaming_attention_state_init(B, Hq, D, "cuda")
        sa.streaming_attention_step(q, k, v, m, l, acc)
        one = sa.streaming_attention_finalize(acc, l, torch.float32)
        m2, l2, _ = sa.streaming_attention_state_init(B, Hq, D, "cuda")
        sa.streaming_attention_stats_step(q, k, m2, l2)
        acc2 = torch.zeros(B, Hq, D, device="cuda")
        bm = torch.zeros(B, Hq, nb, device="cuda")
        sa.streaming_attention_accumulate_step(q, k, v, m2, l2, acc2, bm, 0, tpb)
        two = sa.streaming_attention_finalize(acc2, l2, torch.float32)
        # the same KV as a block pool: slot b*nb + j holds row b's block j
        pool = torch.stack([k.view(B, Hkv, nb, tpb, D), v.view(B, Hkv, nb, tpb, D)], dim=2)  # [B,Hkv,2,nb,tpb,D]
        pool = pool.permute(0, 3, 2, 1, 4, 5).reshape(B * nb, 1, 2, Hkv, tpb, D).contiguous()
        table = torch.arange(B * nb, dtype=torch.int32, device="cuda").view(B, nb)
        mass = torch.zeros(B, Hq, nb, device="cuda")
        paged = sa.paged_decode_attention(q, table, torch.full((B,), nb, dtype=torch.int32, device="cuda"),
                                          dev_pool=pool, host_pool=None, num_layers=1, layer=0,
                                          tokens_per_block=tpb, max_row_tokens=T, block_mass=mass,
                                          out=torch.empty(B, Hq, D, device="cuda"))
        torch.cuda.synchronize()
    finally:
        sa.set_backend("auto")
    from pager_hf import _lib

    assert _lib.device_status(0) == 0
    np.testing.assert_allclose(one.cpu().numpy(), two.cpu().numpy(), rtol=0, atol=5e-3)
    np.testing.assert_allclose(one.cpu().numpy(), paged.cpu().numpy(), rtol=0, atol=5e-3)
    np.testing.assert_allclose(bm.cpu().numpy(), mass.cpu().numpy(), rtol=1e-4, atol=1e-8)
    tot = mass.sum(-1).cpu().numpy()
    np.testing.assert_allclose(tot, np.ones_like(tot), rtol=1e-4)
    assert (mass >= 0).all()
    # oracle on two rows (dense decode restated on the CPU)
    for b in (0, B - 1):
        qn = q[b:b + 1].float().cpu().numpy()
        kn = k[b:b + 1].float().cpu().numpy()
        vn = v[b:b + 1].float().cpu().numpy()
        empty = np.zeros((1, Hkv, 0, D), np.float32)
        ref_out, ref_mass = orc.dense_decode_gqa(qn, kn, vn, empty, empty, tpb)
        np.testing.assert_allclose(paged[b].cpu().numpy(), ref_out[0], rtol=0, atol=5e-3)
        np.testing.assert_allclose(mass[b].cpu().numpy(), ref_mass[0], rtol=1e-4, atol=1e-8)
