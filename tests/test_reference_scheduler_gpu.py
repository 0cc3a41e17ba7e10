"""The reference's own serving scheduler, unmodified, running on this package.

``ContinuousBatchingScheduler`` (the reference's ``pager_hf/serving/scheduler.py``) creates
``PagedModel`` sessions, steps fresh or unpartnered ones with ``generate(..., max_new_tokens=1)`` and
groups started ones by ``_tail_past`` length for ``batched_decode_step`` (``scheduler.py:465-564``).
Its file is loaded from the offline install of the reference (``baseline/_ref``) as
``pager_hf.serving.scheduler``, so its relative imports bind to this package's ``PagedModel`` and
``batched_decode_step``; the test is skipped where that install is absent.  Rounds are driven by hand,
as the reference's scheduler tests do.  Every request's tokens must equal unpaged HF greedy decoding
of its prompt, and batched rounds must have run.
"""

import importlib.util
import os
import sys
import types

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_SERVING = os.path.join(ROOT, "baseline", "_ref", "pager_hf", "serving")
BLOCK = 16 * 1024 * 1024


def _load_reference_scheduler():
    path = os.path.join(REF_SERVING, "scheduler.py")
    if not os.path.isfile(path):
        pytest.skip("the reference is not installed under baseline/_ref")
    import pager_hf

    pkg = types.ModuleType("pager_hf.serving")
    pkg.__path__ = [REF_SERVING]
    sys.modules["pager_hf.serving"] = pkg
    pager_hf.serving = pkg
    spec = importlib.util.spec_from_file_location("pager_hf.serving.scheduler", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules["pager_hf.serving.scheduler"] = mod
    spec.loader.exec_module(mod)
    return mod


def test_reference_scheduler_drives_this_package_unchanged():
    from test_paged_model_gpu import _assert_greedy_match, _hf_greedy, _model

    import pager_hf.paged_model as ours

    sched_mod = _load_reference_scheduler()
    assert sched_mod.PagedModel is ours.PagedModel  # its relative import bound to this package
    model = _model("qwen2")
    sched = sched_mod.ContinuousBatchingScheduler(
        model, types.SimpleNamespace(eos_token_id=None), max_concurrent_sessions=4,
        total_vram_budget=8 * BLOCK, total_ram_budget=4000 * BLOCK, policy="sinks_heavy_hitter",
        tokens_per_block=16, device="cuda")
    g = torch.Generator().manual_seed(31)
    lengths = (50, 66, 82, 98)  # equal tails: (length - 1) % 16 == 1, so started sessions batch
    prompts = [torch.randint(0, 2000, (1, n), generator=g) for n in lengths]
    steps = 20
    reqs = [sched.submit(p, torch.ones_like(p), steps) for p in prompts]
    for _ in range(4 * steps):
        if all(r.done.is_set() for r in reqs):
            break
        sched._admit_new_requests()
        sched._run_once()
    assert all(r.done.is_set() and r.error is None for r in reqs)
    batched = sched._step_calls_total.labels(mode="batched", device="default")._value.get()
    assert batched > 0
    for p, r in zip(prompts, reqs):
        ids = p.cuda()
        want, logits = _hf_greedy(model, ids, torch.ones_like(ids), steps)
        _assert_greedy_match(r.generated_tokens, want[0], logits)


def test_reference_router_threads_and_sessions_run_on_this_package():
    """The reference's ``MultiGpuScheduler`` (``serving/multi_gpu.py``), unmodified, over two of its
    schedulers (labelled as two devices, both on this GPU), started as real serving threads: one-shot
    requests go to the least-loaded scheduler, a two-turn session stays on its owner and its second
    turn continues the first's KV cache.  Every result equals unpaged HF greedy decoding."""
    import importlib

    from test_paged_model_gpu import _assert_greedy_match, _hf_greedy, _model

    sched_mod = _load_reference_scheduler()
    multi_gpu = importlib.import_module("pager_hf.serving.multi_gpu")
    model = _model("qwen2")

    def scheduler(label):
        return sched_mod.ContinuousBatchingScheduler(
            model, types.SimpleNamespace(eos_token_id=None), max_concurrent_sessions=4,
            total_vram_budget=8 * BLOCK, total_ram_budget=4000 * BLOCK, policy="heavy_hitter", tokens_per_block=16,
            device="cuda", device_label=label)

    router = multi_gpu.MultiGpuScheduler([scheduler("gpu-a"), scheduler("gpu-b")])
    g = torch.Generator().manual_seed(37)
    prompts = [torch.randint(0, 2000, (1, n), generator=g) for n in (70, 45, 100)]
    turn1 = torch.randint(0, 2000, (1, 40), generator=g)
    turn2 = torch.randint(0, 2000, (1, 10), generator=g)
    router.start()
    try:
        reqs = [router.submit(p, torch.ones_like(p), 12) for p in prompts]
        sid = router.create_session()
        first = router.submit_turn(sid, turn1, torch.ones_like(turn1), 8)
        assert all(r.done.wait(timeout=180) for r in reqs + [first])
        second = router.submit_turn(sid, turn2, torch.ones_like(turn2), 8)
        assert second.done.wait(timeout=180)
        assert router.health()["thread_alive"]
    finally:
        router.stop(timeout=60)
    assert all(r.error is None for r in reqs + [first, second])
    for p, r in zip(prompts, reqs):
        ids = p.cuda()
        want, logits = _hf_greedy(model, ids, torch.ones_like(ids), 12)
        _assert_greedy_match(r.generated_tokens, want[0], logits)
    want1, logits1 = _hf_greedy(model, turn1.cuda(), torch.ones_like(turn1).cuda(), 8)
    _assert_greedy_match(first.generated_tokens, want1[0], logits1)
    full = torch.cat([turn1, torch.tensor([first.generated_tokens]), turn2], dim=1).cuda()
    want2, logits2 = _hf_greedy(model, full, torch.ones_like(full), 8)
    _assert_greedy_match(second.generated_tokens, want2[0], logits2)
