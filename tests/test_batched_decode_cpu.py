"""``batched_decode_step``'s session checks, on CPU, with PagedModel instances whose session state is set
directly (the reference's ``tests/test_batched_decode.py`` pattern: every check runs before device work).

Checks kept from the reference: empty input, one underlying model, streaming sessions only, an active
``generate()`` session, one ``tokens_per_block``, single-row sessions.  Restrictions the fused paged op
lifts (different tail lengths, different ``streaming_group_size_blocks``, mixed attention-scoring and
uniform policies) pass validation here; their GPU behaviour is covered by the greedy-parity tests.
"""

import pytest
import torch

from pager_hf.batched_decode import _validate_sessions, batched_decode_step
from pager_hf.paged_model import PagedModel


def make_fake_session(**overrides) -> PagedModel:
    pm = PagedModel(model=object(), vram_budget=1_000, ram_budget=1_000)
    pm._store = object()  # only needs to be non-None for these checks
    pm._num_layers = 2
    pm._num_blocks = 1
    pm._tail_len = 3
    pm._pad = torch.zeros(1, dtype=torch.int32)
    pm._tail_past = [(torch.zeros(1, 2, 3, 4), torch.zeros(1, 2, 3, 4))]  # one row, tail of 3 tokens
    for key, value in overrides.items():
        setattr(pm, key, value)
    return pm


def test_empty_sessions_returns_empty_list():
    assert batched_decode_step([], [], torch.device("cpu")) == []


def test_rejects_sessions_with_different_underlying_models():
    a = make_fake_session()
    b = make_fake_session()
    with pytest.raises(ValueError, match="same underlying model"):
        batched_decode_step([a, b], [1, 2], torch.device("cpu"))


def test_rejects_non_streaming_sessions():
    a = make_fake_session(use_streaming_attention=False)
    with pytest.raises(ValueError, match="use_streaming_attention=True"):
        batched_decode_step([a], [1], torch.device("cpu"))


def test_non_streaming_construction_is_refused():
    with pytest.raises(NotImplementedError):
        PagedModel(model=object(), vram_budget=1_000, ram_budget=1_000, use_streaming_attention=False)


def test_rejects_sessions_without_an_active_generate_session():
    a = make_fake_session(_store=None)
    with pytest.raises(ValueError, match="active generate\\(\\) session"):
        batched_decode_step([a], [1], torch.device("cpu"))


def test_rejects_mismatched_tokens_per_block():
    a = make_fake_session()
    b = make_fake_session(model=a.model, tokens_per_block=32)
    with pytest.raises(ValueError, match="tokens_per_block"):
        batched_decode_step([a, b], [1, 2], torch.device("cpu"))


def test_rejects_batch_size_greater_than_one():
    a = make_fake_session(_pad=torch.zeros(2, dtype=torch.int32),
                          _tail_past=[(torch.zeros(2, 2, 3, 4), torch.zeros(2, 2, 3, 4))])
    with pytest.raises(ValueError, match="single-row"):
        batched_decode_step([a], [1], torch.device("cpu"))


def test_rejects_one_session_twice_and_a_wrong_token_count():
    a = make_fake_session()
    with pytest.raises(ValueError, match="same session twice"):
        batched_decode_step([a, a], [1, 2], torch.device("cpu"))
    b = make_fake_session(model=a.model)
    with pytest.raises(ValueError, match="one next input id per session"):
        batched_decode_step([a, b], [1], torch.device("cpu"))


def test_lifted_restrictions_pass_validation():
    """Different tails, group sizes and policy kinds: the reference rejects each of these; one paged
    launch per layer serves them all."""
    a = make_fake_session()
    b = make_fake_session(model=a.model, _tail_len=7, streaming_group_size_blocks=8)
    b._needs_attention = not a._needs_attention
    _validate_sessions([a, b], [1, 2])


def test_tail_past_is_none_without_a_session():
    assert PagedModel(model=object(), vram_budget=1_000, ram_budget=1_000)._tail_past is None
