"""``PagedModel``'s host-side rules, as the reference's CPU tests pin them (tests/test_concurrency.py,
tests/test_paged_model_padding.py, tests/test_sampling.py): the single-flight lock, position ids and
the left-padding check, and sampling.  No model or GPU is needed: a bare object stands in for it."""

import logging

import pytest
import torch

from pager_hf.paged_model import PagedModel


def _pm():
    return PagedModel(model=object(), vram_budget=1_000, ram_budget=1_000)


def _one_token_call(pm, mask=None):
    ids = torch.zeros(1, 1 if mask is None else mask.shape[1], dtype=torch.long)
    return pm.generate(input_ids=ids, attention_mask=torch.ones_like(ids) if mask is None else mask,
                       max_new_tokens=1)


# -- single flight (tests/test_concurrency.py)
def test_a_call_while_another_holds_the_lock_is_rejected_and_logged(caplog):
    pm = _pm()
    pm._lock.acquire()
    try:
        with caplog.at_level(logging.WARNING, logger="pager_hf.paged_model"):
            with pytest.raises(RuntimeError, match="already running"):
                _one_token_call(pm)
            with pytest.raises(RuntimeError, match="already running"):
                pm.reset()
    finally:
        pm._lock.release()
    assert sum(r.levelno == logging.WARNING and "already in flight" in r.message for r in caplog.records) == 2


def test_the_lock_is_free_after_a_rejected_mask_and_after_reset():
    pm = _pm()
    with pytest.raises(NotImplementedError):  # right padding is refused before the model is touched
        _one_token_call(pm, torch.tensor([[1, 0]]))
    assert not pm._lock.locked()
    pm.reset()
    assert not pm._lock.locked()


# -- position ids and padding (tests/test_paged_model_padding.py)
@pytest.mark.parametrize("mask,expected", [
    ([[1, 1, 1, 1, 1]], [[0, 1, 2, 3, 4]]),
    ([[0, 0, 1, 1, 1]], [[0, 0, 0, 1, 2]]),
    ([[1, 1, 1, 1], [0, 1, 1, 1], [0, 0, 0, 1]], [[0, 1, 2, 3], [0, 0, 1, 2], [0, 0, 0, 0]]),
])
def test_position_ids_count_real_tokens_from_zero(mask, expected):
    assert torch.equal(PagedModel._position_ids_from_mask(torch.tensor(mask)), torch.tensor(expected))


@pytest.mark.parametrize("mask", [[[1, 1, 1, 1], [1, 1, 1, 1]], [[0, 0, 1, 1], [1, 1, 1, 1]]])
def test_left_padded_masks_are_accepted(mask):
    PagedModel._validate_left_padded(torch.tensor(mask))


@pytest.mark.parametrize("mask", [[[1, 1, 1, 0]], [[0, 1, 0, 1]], [[0, 0, 0, 0]]])
def test_right_padded_interleaved_and_empty_rows_are_refused(mask):
    with pytest.raises(NotImplementedError):
        PagedModel._validate_left_padded(torch.tensor(mask))


# -- sampling (tests/test_sampling.py)
def _draw(logits, gen, temperature=1.0, top_k=None, top_p=None):
    return PagedModel._sample_next_token(logits, temperature=temperature, top_k=top_k, top_p=top_p,
                                         generator=gen).item()


def test_top_k_of_one_is_greedy():
    logits = torch.randn(5, 100, generator=torch.Generator().manual_seed(3))
    gen = torch.Generator().manual_seed(0)
    for row in range(5):
        assert _draw(logits[row:row + 1], gen, top_k=1) == int(logits[row].argmax())


def test_a_seeded_generator_reproduces_the_draw():
    logits = torch.tensor([[5.0, 1.0, 0.5, 0.1, -2.0]])
    assert _draw(logits, torch.Generator().manual_seed(42)) == _draw(logits, torch.Generator().manual_seed(42))


def test_top_k_and_top_p_cut_the_tail():
    gen = torch.Generator().manual_seed(0)
    assert {_draw(torch.tensor([[5.0, 4.0, 3.0, -10.0, -10.0]]), gen, top_k=2) for _ in range(20)} <= {0, 1}
    assert {_draw(torch.tensor([[10.0, -10.0, -10.0, -10.0, -10.0]]), gen, top_p=0.01) for _ in range(10)} == {0}


def test_a_low_temperature_favours_the_argmax():
    gen = torch.Generator().manual_seed(0)
    picks = [_draw(torch.tensor([[3.0, 2.9, 2.8]]), gen, temperature=0.05) for _ in range(20)]
    assert picks.count(0) >= 15


# -- beam search arguments (paged_model.py:480-495 of the reference): refused before the model is touched
@pytest.mark.parametrize("kw,exc", [
    (dict(num_beams=0, max_new_tokens=2), ValueError),
    (dict(num_beams=2, max_new_tokens=2, num_return_sequences=3), ValueError),
    (dict(num_beams=2, max_new_tokens=2, do_sample=True, temperature=0.0), ValueError),
    (dict(num_beams=2, max_new_tokens=2, do_sample=True, top_k=0), ValueError),
    (dict(num_beams=2, max_new_tokens=2, do_sample=True, top_p=1.5), ValueError),
])
def test_beam_search_argument_checks(kw, exc):
    pm = _pm()
    with pytest.raises(exc):
        pm.generate_beam_search(torch.zeros(1, 2, dtype=torch.long), torch.ones(1, 2, dtype=torch.long), **kw)
    assert not pm._lock.locked()
    with pytest.raises(NotImplementedError):  # right padding
        pm.generate_beam_search(torch.zeros(1, 2, dtype=torch.long), torch.tensor([[1, 0]]), num_beams=2,
                                max_new_tokens=2)
    assert not pm._lock.locked()
