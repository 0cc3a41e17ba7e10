"""``torch.ops.pager_b200.*`` run the same kernels as the direct calls: identical results, and the
operators pass torch's own consistency checks (schema, fake tensors, dispatch)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_operators_match_the_direct_calls_and_pass_opcheck():
    import pager_hf.ops  # noqa: F401
    from pager_hf import streaming_attention as sa

    g = torch.Generator().manual_seed(3)
    B, Hq, Hkv, D, T = 2, 32, 8, 128, 700
    q = torch.randn(B, Hq, D, generator=g).to(torch.bfloat16).cuda()
    k = torch.randn(B, Hkv, T, D, generator=g).to(torch.bfloat16).cuda()
    v = torch.randn(B, Hkv, T, D, generator=g).to(torch.bfloat16).cuda()
    m, l, acc = sa.streaming_attention_state_init(B, Hq, D, "cuda")
    m2, l2, acc2 = m.clone(), l.clone(), acc.clone()
    sa.streaming_attention_step(q, k, v, m, l, acc)
    torch.ops.pager_b200.streaming_attention_step(q, k, v, m2, l2, acc2, None, None, None, None)
    assert torch.equal(m, m2) and torch.equal(l, l2) and torch.equal(acc, acc2)
    out = sa.streaming_attention_finalize(acc, l, torch.bfloat16)
    assert torch.equal(out, torch.ops.pager_b200.streaming_attention_finalize(acc2, l2, torch.bfloat16))
    torch.library.opcheck(torch.ops.pager_b200.streaming_attention_finalize.default, (acc, l, torch.bfloat16))
    m3, l3, acc3 = sa.streaming_attention_state_init(B, Hq, D, "cuda")
    torch.library.opcheck(torch.ops.pager_b200.streaming_attention_step.default,
                          (q, k, v, m3, l3, acc3, None, None, None, None),
                          test_utils=("test_schema", "test_faketensor"))
