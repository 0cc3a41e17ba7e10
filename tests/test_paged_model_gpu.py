"""Greedy generation through ``pager_hf.paged_model.PagedModel`` matches unpaged HF greedy decoding.

The end-to-end criterion: greedy token IDs from
``PagedModel.generate`` on random-init weights match exactly.  The unpaged
reference is the model's own forward with a ``DynamicCache`` (transformers'
stock attention), one token at a time with argmax -- the reference project's
own correctness bar (greedy parity with plain HF generation).  Token IDs
must match exactly; the only tolerated difference is a tie at the model's
output precision in the unpaged run's own logits (two tokens within one ulp
of the model's dtype: either choice is within rounding of the exact result,
and the two runs then follow different continuations); in fp32 not even that.
Parity with the reference's own attention algorithm, rather than transformers'
attention, is tested in ``test_model_parity_gpu.py``.  The paged run
keeps most blocks in the pinned host tier (small VRAM budget), scores blocks
with the heavy-hitter mass the kernel emits, and rolls tails into blocks many
times.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

BLOCK = 16 * 1024 * 1024


@torch.inference_mode()
def _hf_greedy(model, input_ids, attention_mask, n):
    """Unpaged greedy decoding; returns (token lists per row, logits per step [rows, vocab])."""
    from transformers import DynamicCache

    cache = DynamicCache()
    mask = attention_mask
    pos = (mask.long().cumsum(-1) - 1).clamp(min=0)
    out = model(input_ids=input_ids, attention_mask=mask, position_ids=pos, past_key_values=cache, use_cache=True)
    toks, logits = [], []
    for _ in range(n):
        logits.append(out.logits[:, -1].float())
        nxt = out.logits[:, -1].argmax(-1, keepdim=True)
        toks.append(nxt)
        mask = torch.cat([mask, torch.ones_like(mask[:, :1])], dim=1)
        pos = (mask.long().cumsum(-1) - 1)[:, -1:]
        out = model(input_ids=nxt, attention_mask=mask, position_ids=pos, past_key_values=cache, use_cache=True)
    return torch.cat(toks, dim=1).tolist(), logits


def _assert_greedy_match(got, want, logits, row=0, dtype=torch.float16):
    """Token IDs must match exactly.  The one allowed exception: at the first differing step the
    unpaged run's own logits of the two tokens are a tie at the model's output precision (within one
    ulp of ``dtype``, the model's dtype: either choice is within rounding of the exact result); the
    continuations then differ and are not compared further.  Returns the step of that tie, or None."""
    for i, (a, b) in enumerate(zip(got, want)):
        if a == b:
            continue
        lg = logits[i][row]
        gap = abs(float(lg[a]) - float(lg[b]))
        ulp = float(torch.finfo(dtype).eps) * max(abs(float(lg[b])), 1e-3)
        assert gap <= ulp, f"step {i}: paged picked {a}, unpaged {b}; logit gap {gap:.5f} > 1 ulp {ulp:.5f}"
        print(f"tie at step {i}: logit gap {gap / ulp:.2f} ulp")
        return i
    assert len(got) == len(want)
    return None


def _model(kind, **over):
    from transformers import MistralConfig, MistralForCausalLM, Qwen2Config, Qwen2ForCausalLM

    torch.manual_seed(0)
    common = dict(hidden_size=256, intermediate_size=512, num_hidden_layers=4, num_attention_heads=4,
                  num_key_value_heads=2, head_dim=64, vocab_size=2000, max_position_embeddings=4096,
                  initializer_range=0.02)
    common.update(over)
    if kind == "qwen2":
        cfg = Qwen2Config(rope_theta=1e6, **common)
        m = Qwen2ForCausalLM(cfg)
    else:
        cfg = MistralConfig(sliding_window=64, **common)
        m = MistralForCausalLM(cfg)
    return m.to(device="cuda", dtype=torch.float16).eval()


@pytest.mark.parametrize("policy", ["sinks_heavy_hitter", "recent_only", "heavy_hitter"])
def test_greedy_tokens_match_unpaged_qwen2(policy):
    from pager_hf.paged_model import PagedModel

    model = _model("qwen2")
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, 2000, (1, 230), generator=g).cuda()
    mask = torch.ones_like(ids)
    want, logits = _hf_greedy(model, ids, mask, 40)
    pm = PagedModel(model, vram_budget=3 * BLOCK, ram_budget=1000 * BLOCK, recent_window=2, rebalance_interval=2,
                    policy=policy, tokens_per_block=16)
    got = pm.generate(ids, mask, 40)
    _assert_greedy_match(got, want[0], logits)
    assert pm._store.cpu_block_ids(), "no block reached the host tier"
    assert pm.last_run_stats.total_new_blocks >= 2


def test_greedy_tokens_match_with_sliding_window_mistral():
    from pager_hf.paged_model import PagedModel

    model = _model("mistral")
    g = torch.Generator().manual_seed(2)
    ids = torch.randint(0, 2000, (1, 150), generator=g).cuda()
    mask = torch.ones_like(ids)
    want, logits = _hf_greedy(model, ids, mask, 30)
    pm = PagedModel(model, vram_budget=2 * BLOCK, ram_budget=1000 * BLOCK, recent_window=1, policy="sinks_recent",
                    tokens_per_block=16)
    _assert_greedy_match(pm.generate(ids, mask, 30), want[0], logits)


def test_left_padded_batch_rows_match_single_row_runs():
    from pager_hf.paged_model import PagedModel

    model = _model("qwen2")
    g = torch.Generator().manual_seed(3)
    lens = [180, 131]
    rows = [torch.randint(0, 2000, (1, n), generator=g).cuda() for n in lens]
    T = max(lens)
    ids = torch.zeros(2, T, dtype=torch.long, device="cuda")
    mask = torch.zeros(2, T, dtype=torch.long, device="cuda")
    for b, r in enumerate(rows):
        ids[b, T - r.shape[1]:] = r[0]
        mask[b, T - r.shape[1]:] = 1
    refs = [_hf_greedy(model, r, torch.ones_like(r), 24) for r in rows]
    pm = PagedModel(model, vram_budget=3 * BLOCK, ram_budget=1000 * BLOCK, recent_window=2, policy="heavy_hitter",
                    tokens_per_block=16)
    got = pm.generate(ids, mask, 24)
    for b, (want, logits) in enumerate(refs):
        _assert_greedy_match(got[b], want[0], logits)


def test_session_continues_across_generate_calls():
    from pager_hf.paged_model import PagedModel

    model = _model("qwen2")
    g = torch.Generator().manual_seed(4)
    ids = torch.randint(0, 2000, (1, 100), generator=g).cuda()
    pm = PagedModel(model, vram_budget=2 * BLOCK, ram_budget=1000 * BLOCK, recent_window=1,
                    policy="sinks_heavy_hitter", tokens_per_block=16)
    first = pm.generate(ids, torch.ones_like(ids), 12)
    want1, logits1 = _hf_greedy(model, ids, torch.ones_like(ids), 12)
    _assert_greedy_match(first, want1[0], logits1)
    # the second call extends the session with the tokens it returned: compare with unpaged greedy
    # decoding from that same extended prompt
    ids2 = torch.cat([ids, torch.tensor([first], device="cuda")], dim=1)
    second = pm.generate(ids2, torch.ones_like(ids2), 18)
    want2, logits2 = _hf_greedy(model, ids2, torch.ones_like(ids2), 18)
    _assert_greedy_match(second, want2[0], logits2)
    with pytest.raises(ValueError):
        pm.generate(ids[:, :50], torch.ones_like(ids[:, :50]), 1)  # shorter than the primed session
    pm.reset()
    _assert_greedy_match(pm.generate(ids, torch.ones_like(ids), 5), want1[0][:5], logits1)


def test_baseline_config2_geometry_greedy_parity():
    """The greedy-generation benchmark config's architecture (random-init Qwen2.5-0.5B: 24 layers, hidden 896, 14/2 heads, D 64,
    fp16), 8192-token prompt, 10% of blocks resident, recent_only; 32 new tokens (128 in the benchmark config)."""
    from pager_hf.paged_model import PagedModel

    model = _model("qwen2", hidden_size=896, intermediate_size=4864, num_hidden_layers=24, num_attention_heads=14,
                   num_key_value_heads=2, head_dim=64, vocab_size=151936, max_position_embeddings=32768)
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, 151936, (1, 8192), generator=g).cuda()
    mask = torch.ones_like(ids)
    want, logits = _hf_greedy(model, ids, mask, 32)
    nblocks = 8192 // 64
    pm = PagedModel(model, vram_budget=-(-nblocks // 10) * BLOCK, ram_budget=10 * nblocks * BLOCK,
                    recent_window=-(-nblocks // 10) - 1, policy="recent_only", tokens_per_block=64)
    _assert_greedy_match(pm.generate(ids, mask, 32), want[0], logits)
    assert len(pm._store.gpu_block_ids()) <= -(-nblocks // 10) + 1


def test_fp32_greedy_tokens_equal_unpaged_decoding_exactly():
    """In fp32 the logits carry no ties at output precision: every token of a 48-token run with most
    blocks in the host tier, heavy-hitter scoring and tails rolled into blocks equals unpaged HF greedy
    decoding -- no tie exception."""
    from pager_hf.paged_model import PagedModel

    model = _model("qwen2").float()
    g = torch.Generator().manual_seed(9)
    ids = torch.randint(0, 2000, (1, 300), generator=g).cuda()
    mask = torch.ones_like(ids)
    want, _ = _hf_greedy(model, ids, mask, 48)
    pm = PagedModel(model, vram_budget=3 * BLOCK, ram_budget=1000 * BLOCK, recent_window=2,
                    policy="sinks_heavy_hitter", tokens_per_block=16)
    assert pm.generate(ids, mask, 48) == want[0]
    assert pm._store.cpu_block_ids() and pm.last_run_stats.total_new_blocks >= 2


def test_captured_decode_steps_match_eager_steps():
    """Decode steps replayed from CUDA graphs (the default) give the same tokens and pager decisions
    as eager steps: a left-padded two-row batch, heavy-hitter scoring from the kernel's mass, tails
    rolled into blocks several times (each a new capture)."""
    from pager_hf.paged_model import PagedModel

    model = _model("qwen2")
    g = torch.Generator().manual_seed(5)
    ids = torch.randint(0, 2000, (2, 200), generator=g).cuda()
    mask = torch.ones_like(ids)
    mask[1, :37] = 0
    runs = {}
    for graphs in (False, True):
        pm = PagedModel(model, vram_budget=3 * BLOCK, ram_budget=64 * BLOCK, recent_window=1, policy="heavy_hitter",
                        tokens_per_block=16, decode_graphs=graphs)
        toks = pm.generate(ids, mask, 40)
        runs[graphs] = (toks, sorted(pm._store.gpu_block_ids()), pm.last_run_stats.total_new_blocks,
                        pm.last_host_read)
        pm.reset()
    assert runs[True][0] == runs[False][0]
    assert runs[True][1:3] == runs[False][1:3]
    assert runs[True][3] == "zero_copy"


def test_sessions_in_two_threads_capture_and_replay_concurrently():
    """Two threads, each driving its own session (the serving scheduler's one thread per session or
    device), decode at the same time while their first steps capture graphs; each thread's tokens
    equal a sequential run's."""
    import threading

    from pager_hf.paged_model import PagedModel

    model = _model("qwen2")
    g = torch.Generator().manual_seed(8)
    prompts = [torch.randint(0, 2000, (1, n), generator=g).cuda() for n in (170, 90)]

    def run(ids, out, i):
        torch.cuda.set_device(0)
        pm = PagedModel(model, vram_budget=2 * BLOCK, ram_budget=1000 * BLOCK, recent_window=1,
                        policy="sinks_heavy_hitter", tokens_per_block=16)
        out[i] = pm.generate(ids, torch.ones_like(ids), 30)
        pm.reset()

    sequential = [None, None]
    for i, ids in enumerate(prompts):
        run(ids, sequential, i)
    concurrent, errors = [None, None], []

    def guarded(ids, i):
        try:
            run(ids, concurrent, i)
        except Exception as e:  # noqa: BLE001 - reported by the assertion below
            errors.append(e)

    threads = [threading.Thread(target=guarded, args=(ids, i)) for i, ids in enumerate(prompts)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=300)
    assert not errors, errors
    assert concurrent == sequential


def _family_model(kind):
    """Small random-init models of the other families the reference verified (``paged_model.py:81-85``)."""
    import transformers as T

    torch.manual_seed(0)
    common = dict(hidden_size=256, intermediate_size=512, num_hidden_layers=4, num_attention_heads=4,
                  num_key_value_heads=2, head_dim=64, vocab_size=2000, max_position_embeddings=4096,
                  initializer_range=0.02)
    extra = {
        # sliding layers alternate with global ones; the window is shorter than the prompts
        "gemma2": dict(sliding_window=64, query_pre_attn_scalar=64),
        "phi3": dict(pad_token_id=0, sliding_window=None),
        "starcoder2": dict(sliding_window=None),
        # every expert active: the routing weights stay continuous in the hidden state, so a 1-ulp
        # difference in attention cannot switch experts
        "qwen2_moe": dict(moe_intermediate_size=128, shared_expert_intermediate_size=256, num_experts=4,
                          num_experts_per_tok=4),
        "gemma": {},
    }[kind]
    cls = {"gemma": (T.GemmaConfig, T.GemmaForCausalLM), "gemma2": (T.Gemma2Config, T.Gemma2ForCausalLM),
           "phi3": (T.Phi3Config, T.Phi3ForCausalLM), "starcoder2": (T.Starcoder2Config, T.Starcoder2ForCausalLM),
           "qwen2_moe": (T.Qwen2MoeConfig, T.Qwen2MoeForCausalLM)}[kind]
    m = cls[1](cls[0](**common, **extra))
    return m.to(device="cuda", dtype=torch.float16).eval()


@pytest.mark.parametrize("kind", ["gemma", "gemma2", "phi3", "starcoder2", "qwen2_moe"])
def test_greedy_tokens_match_unpaged_for_the_other_families(kind):
    """Gemma (scaled embeddings), Gemma2 (alternating sliding/global layers, attention and final logit
    softcaps, extra feed-forward norms), Phi3 (fused qkv projection), Starcoder2 (biased projections,
    LayerNorm) and Qwen2-MoE (sparse MoE feed-forward, whose steps stay eager: its expert routing
    cannot be captured): greedy tokens of captured decode steps, and of eager ones, match unpaged HF
    greedy decoding with most blocks in the host tier."""
    from pager_hf.paged_model import PagedModel

    model = _family_model(kind)
    g = torch.Generator().manual_seed(11)
    ids = torch.randint(0, 2000, (1, 150), generator=g).cuda()
    mask = torch.ones_like(ids)
    want, logits = _hf_greedy(model, ids, mask, 24)
    for graphs in (True, False):
        pm = PagedModel(model, vram_budget=2 * BLOCK, ram_budget=1000 * BLOCK, recent_window=1,
                        policy="sinks_heavy_hitter", tokens_per_block=16, decode_graphs=graphs)
        assert pm.decode_graphs == (graphs and kind != "qwen2_moe")
        _assert_greedy_match(pm.generate(ids, mask, 24), want[0], logits)
        assert pm._store.cpu_block_ids(), "no block reached the host tier"
        pm.reset()


def test_beam_search_with_one_beam_is_greedy_decoding():
    from pager_hf.paged_model import PagedModel

    model = _model("qwen2")
    g = torch.Generator().manual_seed(41)
    ids = torch.randint(0, 2000, (1, 120), generator=g).cuda()
    mask = torch.ones_like(ids)
    kw = dict(vram_budget=2 * BLOCK, ram_budget=1000 * BLOCK, recent_window=1, policy="sinks_heavy_hitter",
              tokens_per_block=16)
    beam = PagedModel(model, **kw).generate_beam_search(ids, mask, num_beams=1, max_new_tokens=20,
                                                        length_penalty=0.0)
    assert beam == PagedModel(model, **kw).generate(ids, mask, 20)


def test_beam_search_matches_hf_beam_search_in_fp32():
    """num_beams hypotheses per prompt, rows reordered to their parents every step across both KV
    tiers and the tail; with fp32 weights (no near-ties at output precision) the result equals
    transformers' own beam search at length_penalty 0, the setting the reference verified."""
    from pager_hf.paged_model import PagedModel

    model = _model("qwen2").float()
    g = torch.Generator().manual_seed(43)
    lens = [90, 57]
    T = max(lens)
    ids = torch.zeros(2, T, dtype=torch.long)
    mask = torch.zeros(2, T, dtype=torch.long)
    for b, n in enumerate(lens):
        ids[b, T - n:] = torch.randint(0, 2000, (n,), generator=g)
        mask[b, T - n:] = 1
    ids, mask = ids.cuda(), mask.cuda()
    pm = PagedModel(model, vram_budget=2 * BLOCK, ram_budget=1000 * BLOCK, recent_window=1,
                    policy="sinks_heavy_hitter", tokens_per_block=16)
    got = pm.generate_beam_search(ids, mask, num_beams=3, max_new_tokens=12, length_penalty=0.0)
    with torch.inference_mode():
        ref = model.generate(input_ids=ids, attention_mask=mask, num_beams=3, max_new_tokens=12, do_sample=False,
                             length_penalty=0.0, early_stopping=False, num_return_sequences=1, pad_token_id=0)
    assert got == ref[:, T:].tolist()
    three = pm.generate_beam_search(ids[:1], mask[:1], num_beams=3, max_new_tokens=12, length_penalty=0.0,
                                    num_return_sequences=3)
    assert len(three) == 3 and three[0] == got[0]


def test_captured_step_logits_are_not_overwritten_by_the_next_step():
    """The logits a captured decode step returns are the caller's: the next replay writes the
    graph's own buffer, not the tensor handed out (as an eager step's logits are fresh tensors)."""
    from pager_hf.paged_model import PagedModel

    model = _model("qwen2")
    g = torch.Generator().manual_seed(6)
    ids = torch.randint(0, 2000, (2, 120), generator=g).cuda()
    mask = torch.ones_like(ids)
    pm = PagedModel(model, vram_budget=3 * BLOCK, ram_budget=64 * BLOCK, recent_window=1, policy="recent_only",
                    tokens_per_block=16, decode_graphs=True)
    kept, copies = [], []
    orig = pm._forward_step

    def step(input_ids, attention_mask):
        logits, info = orig(input_ids, attention_mask)
        kept.append(logits)  # no copy: must stay this step's values
        copies.append(logits.clone())
        return logits, info

    pm._forward_step = step
    pm.generate(ids, mask, 6)
    assert len(kept) >= 5
    for a, b in zip(kept, copies):
        assert torch.equal(a, b)
    assert not torch.equal(kept[-2], kept[-1])
