"""The entry points registered as torch operators: present under ``torch.ops.pager_b200`` and
traceable with fake tensors (shapes and dtypes only; no GPU and no kernel launch needed)."""

import torch


def test_operators_are_registered_and_trace_with_fake_tensors():
    from torch._subclasses.fake_tensor import FakeTensorMode

    import pager_hf.ops  # noqa: F401  (registers the operators)

    ops = torch.ops.pager_b200
    for name in ("streaming_attention_step", "streaming_attention_stats_step", "streaming_attention_accumulate_step",
                 "streaming_attention_fold_fixed_step", "streaming_attention_finalize", "paged_decode_attention"):
        assert hasattr(ops, name), name
    with FakeTensorMode():
        acc = torch.empty(2, 14, 64)
        l = torch.empty(2, 14)
        out = ops.streaming_attention_finalize(acc, l, torch.bfloat16)
        assert out.shape == (2, 14, 64) and out.dtype == torch.bfloat16
        q = torch.empty(2, 14, 64, dtype=torch.float16)
        pool = torch.empty(8, 2, 2, 2, 16, 64, dtype=torch.float16)
        table = torch.empty(2, 4, dtype=torch.int32)
        nb = torch.empty(2, dtype=torch.int32)
        o = ops.paged_decode_attention(q, table, nb, pool, None, 2, 1, 16, 64, None, None, None, None, None, None,
                                       None, None, None, "none", "running")
        assert o.shape == q.shape and o.dtype == q.dtype
        m = torch.empty(2, 14)
        ops.streaming_attention_step(q, torch.empty(2, 2, 32, 64, dtype=torch.float16),
                                     torch.empty(2, 2, 32, 64, dtype=torch.float16), m, l, acc, None, None, None, None)
