"""Host-side helpers of the model-level decode bench (``pager_hf.generate_bench``)."""

import pytest
import torch

gb = pytest.importorskip("pager_hf.generate_bench")


def test_prompt_rows_are_left_padded_to_the_longest(monkeypatch):
    monkeypatch.setattr(torch.Tensor, "cuda", lambda self: self)  # keep the prompt on the host
    c = dict(gb.CONFIGS["cfg3"], batch=4, lengths=(5, 12))
    ids, mask, lens = gb.build_prompt(c)
    assert ids.shape == mask.shape == (4, max(lens)) and all(5 <= n <= 12 for n in lens)
    for b, n in enumerate(lens):
        assert int(mask[b].sum()) == n and bool(mask[b, -n:].all())
        assert int(ids[b, : ids.shape[1] - n].abs().sum()) == 0
    again = gb.build_prompt(c)
    assert torch.equal(again[0], ids)  # seeded


def test_attended_bytes_count_valid_tokens_and_the_window():
    c = gb.CONFIGS["cfg2"]
    per_tok = 2 * c["num_key_value_heads"] * c["head_dim"] * 2 * c["num_hidden_layers"]
    assert gb.kv_bytes_per_step(c, [8192], 1) == 8193 * per_tok == 12288 * 8193
    w = gb.CONFIGS["cfg4"]
    per_tok4 = 2 * w["num_key_value_heads"] * w["head_dim"] * 2 * w["num_hidden_layers"]
    assert gb.kv_bytes_per_step(w, [32768] * 8, 65) == 8 * 4096 * per_tok4  # only the window is read


def test_first_divergences_are_measured_in_the_model_dtype_ulps():
    vocab = 8
    logits = [torch.zeros(2, vocab, dtype=torch.float16) for _ in range(3)]
    logits[1][0, 3], logits[1][0, 5] = 4.0, 4.0 + 4.0 * 2 ** -10  # one fp16 ulp apart at 4.0
    logits[2][1, 1], logits[2][1, 2] = 1.0, 1.25  # 256 fp16 ulps apart at 1.0
    paged = [[7, 3, 0], [7, 0, 1]]
    unpaged = [[7, 5, 1], [7, 0, 2]]
    div = gb.first_divergences(paged, unpaged, logits, torch.float16)
    assert [(d["row"], d["step"]) for d in div] == [(0, 1), (1, 2)]
    assert div[0]["gap_ulps"] <= 1.0 + 1e-6 and div[1]["gap_ulps"] > 200
    # the same gaps in bfloat16 ulps (8x coarser)
    div_bf = gb.first_divergences(paged, unpaged, logits, torch.bfloat16)
    assert abs(div_bf[1]["gap_ulps"] * 8 - div[1]["gap_ulps"]) < 1e-3
    assert gb.first_divergences(paged, paged, logits) == []
