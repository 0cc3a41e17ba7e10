"""Host-side rules of ``PagedModel``'s captured decode steps (no GPU needed)."""

from pager_hf.paged_model import _DecodeGraph


def test_graph_table_width_covers_blocks_and_tail_in_fixed_steps():
    """A captured step's block table holds the blocks plus the tail column, rounded up to a multiple
    of ``WIDTH_STEP``: a session re-captures once per ``WIDTH_STEP`` new blocks, not per block."""
    step = _DecodeGraph.WIDTH_STEP
    widths = [_DecodeGraph.width_for(nb) for nb in range(0, 5 * step)]
    for nb, w in enumerate(widths):
        assert w >= nb + 1 and w % step == 0 and w - (nb + 1) < step
    assert len(set(widths)) == 5  # one width per WIDTH_STEP blocks


def _tiny(kind, **over):
    import transformers as T

    common = dict(hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
                  num_key_value_heads=2, head_dim=16, vocab_size=100, max_position_embeddings=256)
    common.update(over)
    cls = {"gemma": (T.GemmaConfig, T.GemmaForCausalLM), "gemma2": (T.Gemma2Config, T.Gemma2ForCausalLM),
           "phi3": (T.Phi3Config, T.Phi3ForCausalLM), "starcoder2": (T.Starcoder2Config, T.Starcoder2ForCausalLM),
           "qwen2_moe": (T.Qwen2MoeConfig, T.Qwen2MoeForCausalLM), "qwen2": (T.Qwen2Config, T.Qwen2ForCausalLM),
           "llama": (T.LlamaConfig, T.LlamaForCausalLM), "mistral": (T.MistralConfig, T.MistralForCausalLM)}[kind]
    return cls[1](cls[0](**common))


def test_architecture_of_every_family_the_reference_verified():
    """``PagedModel`` reads per family what its decode step needs (``paged_model.py:81-175`` of the
    reference): the distinct sliding windows and each layer's, the attention and final logit
    softcaps (Gemma2), a fused qkv projection (Phi3) and Gemma2's extra feed-forward norms."""
    from pager_hf.paged_model import PagedModel

    def arch(kind, **over):
        return PagedModel(_tiny(kind, **over), vram_budget=1, ram_budget=1)._arch()

    a = arch("gemma2", sliding_window=32, query_pre_attn_scalar=16)
    assert a["windows"] == [None, 32] and a["layer_window"] == [1, 0]
    assert a["softcap"] == 50.0 and a["final_softcap"] == 30.0 and a["sandwich_norms"] and not a["qkv_fused"]
    a = arch("phi3", pad_token_id=0, sliding_window=None)
    assert a["qkv_fused"] and a["windows"] == [None] and a["layer_window"] == [0, 0]
    a = arch("mistral", sliding_window=64)
    assert a["windows"] == [64] and a["layer_window"] == [0, 0] and a["softcap"] is None
    a = arch("qwen2_moe", moe_intermediate_size=32, shared_expert_intermediate_size=64, num_experts=4,
             num_experts_per_tok=2)
    assert a["windows"] == [None] and a["final_softcap"] is None
    for kind in ("gemma", "starcoder2", "qwen2", "llama"):
        a = arch(kind)
        assert a["windows"] == [None] and not a["qkv_fused"] and not a["sandwich_norms"], kind
