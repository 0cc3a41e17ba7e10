"""``PagedModel``: greedy / sampled generation with the KV cache paged by the pager.

Same surface as the reference's ``pager_hf/paged_model.py:192-420``
(``PagedModel(model, *, vram_budget, ram_budget, recent_window,
rebalance_interval, promote_margin, ram_promote_margin, policy,
tokens_per_block, ...)``, ``generate(input_ids, attention_mask,
max_new_tokens, *, do_sample, temperature, top_k, top_p, generator)``,
``reset()``, one session per instance that later ``generate`` calls extend,
``last_run_stats``), for the decoder families whose layers are
``input_layernorm -> self_attn(q/k/v/o_proj, RoPE) -> post_attention_layernorm
-> mlp`` (Qwen2, Llama, Mistral) in the installed transformers.

The reference patches each attention module's ``forward`` for the
transformers 4.44 API and gathers every block group per layer.  Here:

* prefill is the model's own forward (the prompt minus its last token, like
  ``_start_session``, ``:671-690``), whose cache is moved into a device slot
  pool as blocks of ``tokens_per_block`` tokens (all batch rows of a block in
  one slot group) plus a tail slot group;
* every decode step drives the decoder modules directly: norms, projections,
  RoPE and MLP from the model, and per layer one ``pager_append_tokens``
  (the new K/V into the tail slots) and one fused ``paged_decode_attention``
  launch over the block table (device, staged/zero-copy host blocks, tail),
  which also accumulates the batch-and-head mean block mass the heavy-hitter
  policies score (``paged_model.py:1048``);
* after each token, the pager gets exactly the reference's calls
  (``_forward_step_streaming`` / ``_append_new_full_blocks_from_grown_tail``):
  ``on_step(query_block, 0, block_attention)``, ``force_rebalance`` when the
  tail became a block (adopted in place, no copy), then ``apply_tiers``.
"""

from __future__ import annotations

import logging
import threading
from dataclasses import dataclass

import torch

from . import _lib as L
from .kv_block_store import KVBlockStore, KVPools
from .streaming_attention import PagedDecodePlan

logger = logging.getLogger(__name__)

_POLICIES_WITHOUT_ATTENTION_SIGNAL = frozenset({"recent_only", "sinks_recent"})
# The families the reference verified its patched forward on (``paged_model.py:81-85``).
_SUPPORTED_MODEL_TYPES = frozenset({"qwen2", "qwen2_moe", "starcoder2", "llama", "mistral", "gemma", "phi3", "gemma2"})
# Families whose attention takes its window from the config (every layer); the others keep a
# per-layer ``sliding_window`` on the attention module (Gemma2 and Qwen2 alternate by layer type).
_CONFIG_WINDOW_MODEL_TYPES = frozenset({"mistral", "phi3", "starcoder2"})
# Families whose decode step cannot be captured in a CUDA graph: Qwen2-MoE's sparse block routes
# tokens to experts with offsets copied from host memory each step.
_EAGER_ONLY_MODEL_TYPES = frozenset({"qwen2_moe"})


@dataclass
class GenerationStats:
    total_new_blocks: int = 0
    final_num_blocks: int = 0
    total_gpu_to_cpu_mb: float = 0.0
    total_cpu_to_gpu_mb: float = 0.0
    total_gpu_to_cpu_copies: int = 0
    total_cpu_to_gpu_copies: int = 0
    mean_attention_in_gpu: float = 0.0
    min_attention_in_gpu: float = 0.0
    max_attention_in_gpu: float = 0.0


def _rope_fn(model):
    import importlib

    mod = importlib.import_module(type(model).__module__)
    return mod.apply_rotary_pos_emb


@dataclass
class AttentionGroup:
    """Rows of a decode batch whose KV lives in one ``KVPools``: the fused op's plans over them (one
    per distinct sliding window of the model, ``arch["windows"]``; layers use the plan of their
    window), each row's tail slot and the token index in it that the row's new K/V goes to.
    ``rows``: the rows' indices in the batch (device int64), or None for every row in order."""

    pools: KVPools
    plans: list
    slots: torch.Tensor
    positions: torch.Tensor
    rows: torch.Tensor | None = None


def run_decoder_step(model, arch: dict, groups: list[AttentionGroup], input_ids, position_ids):
    """One token per row through the decoder: embeddings, then per layer the input norm, q/k/v
    projections (fused ``qkv_proj`` for Phi3) and RoPE from the model for all rows at once; per group
    of rows sharing pools, the new K/V written into each row's tail slot (``pager_append_tokens``)
    and one fused paged attention launch of the group's plan for this layer's window; o_proj, the
    residual and the MLP for all rows (Gemma2: normalized attention output and MLP between its
    pre/post feed-forward norms); final norm, lm_head and Gemma2's final logit softcap.
    Returns logits ``[rows, 1, vocab]``."""
    B = input_ids.shape[0]
    a = arch
    rope = _rope_fn(model)
    hidden = model.model.embed_tokens(input_ids)
    cos, sin = model.model.rotary_emb(hidden, position_ids)
    lib = L.lib()
    dev = input_ids.device
    stream = torch.cuda.current_stream(dev).cuda_stream
    out = torch.empty(B, a["hq"], a["d"], dtype=hidden.dtype, device=dev)
    parts = [out if g.rows is None else torch.empty(g.rows.numel(), a["hq"], a["d"], dtype=hidden.dtype, device=dev)
             for g in groups]
    for li, layer in enumerate(model.model.layers):
        residual = hidden
        h = layer.input_layernorm(hidden)
        attn = layer.self_attn
        if a["qkv_fused"]:
            qkv = attn.qkv_proj(h)
            nq, nkv = a["hq"] * a["d"], a["hkv"] * a["d"]
            q, k, v = qkv[..., :nq], qkv[..., nq:nq + nkv], qkv[..., nq + nkv:]
        else:
            q, k, v = attn.q_proj(h), attn.k_proj(h), attn.v_proj(h)
        q = q.view(B, 1, -1, a["d"]).transpose(1, 2)
        k = k.view(B, 1, -1, a["d"]).transpose(1, 2)
        v = v.view(B, 1, -1, a["d"]).transpose(1, 2)
        q, k = rope(q, k, cos, sin)
        q, k, v = q[:, :, 0], k[:, :, 0], v[:, :, 0]
        for g, part in zip(groups, parts):
            if g.rows is None:
                gq, gk, gv = q.contiguous(), k.contiguous(), v.contiguous()
            else:
                gq, gk, gv = q.index_select(0, g.rows), k.index_select(0, g.rows), v.index_select(0, g.rows)
            p = g.pools
            L.check(lib.pager_append_tokens(p.dev_pool.data_ptr(), L.DTYPE_CODE[p.dtype], p.dev_pool.shape[0],
                                            a["layers"], li, a["hkv"], p.tokens_per_block, a["d"],
                                            g.slots.data_ptr(), g.positions.data_ptr(), gk.data_ptr(), gv.data_ptr(),
                                            gk.shape[0], stream))
            g.plans[a["layer_window"][li]].run(gq, li, part)
            if g.rows is not None:
                out.index_copy_(0, g.rows, part)
        attn_out = attn.o_proj(out.reshape(B, 1, -1))
        if a["sandwich_norms"]:  # Gemma2DecoderLayer
            hidden = residual + layer.post_attention_layernorm(attn_out)
            hidden = hidden + layer.post_feedforward_layernorm(layer.mlp(layer.pre_feedforward_layernorm(hidden)))
        else:
            hidden = residual + attn_out
            hidden = hidden + layer.mlp(layer.post_attention_layernorm(hidden))
    logits = model.lm_head(model.model.norm(hidden))
    if a["final_softcap"]:
        logits = torch.tanh(logits / a["final_softcap"]) * a["final_softcap"]
    return logits


_TENSOR_CORE_HEAD_DIMS = frozenset({64, 128, 256})  # head_dims the tensor-core kernels serve


def step_rounding(mode: str, needs_attention: bool, dtype, head_dim: int, tokens_per_block: int) -> str:
    """The fused op's ``rounding`` for a decode step.  ``mode="reference"``: p is rounded as the
    reference rounds it -- against its running max per 64-token tile ("running") in the one-pass
    path it runs for policies without an attention signal (paged_model.py:1055-1072), against the
    row's final max ("final") in the two-pass path of the heavy-hitter policies (:993-1039).  fp32
    rounds nothing either way, so it keeps the one pass, as ``mode="one_pass"`` always does; so does
    the running rule on the tensor-core kernels with blocks shorter than 16 tokens."""
    if mode not in ("reference", "one_pass"):
        raise ValueError(f"attention_rounding must be 'reference' or 'one_pass', got {mode!r}")
    if mode == "one_pass" or dtype == torch.float32:
        return "one_pass"
    if needs_attention:
        return "final"
    if tokens_per_block < 16 and head_dim in _TENSOR_CORE_HEAD_DIMS:
        return "one_pass"
    return "running"


def window_lo(pad: int, total: int, window) -> int:
    """First attended column of a row: after its left padding and, with a sliding window, within the
    last ``window`` columns (``paged_model.py:975-980``)."""
    return max(pad, total - int(window)) if window is not None else pad


class _DecodeGraph:
    """One decode step of a ``PagedModel`` session captured as a CUDA graph.

    Eager decode steps are bound by the host: each layer runs a dozen small modules
    (norms, projections, RoPE, MLP) plus the paged op, ~800 launches per step for a 24-layer
    model.  The graph replays them with one launch.  Its inputs live in static device buffers
    refreshed before each replay: the token ids and position ids, and one packed int32 buffer
    holding the block table, the rows' block counts, range ends, tail slots, tail positions, first
    tail tokens (where the reference's tail chunk starts, for its rounding of p) and first attended
    columns (one per distinct sliding window) -- a single host copy per step.
    Shapes and pointers the launches bake in -- batch, table width (``width`` block columns, a
    multiple of ``WIDTH_STEP`` at least the blocks plus the tail; it also bounds the split plan),
    the pools (their ``version`` changes when they grow) -- form the key, so a new graph is
    captured once per ``WIDTH_STEP`` blocks; columns past a row's blocks are absent.  Host-tier
    blocks are read zero-copy inside the graph."""

    WIDTH_STEP = 64

    @classmethod
    def width_for(cls, nb: int) -> int:
        return -(-(nb + 1) // cls.WIDTH_STEP) * cls.WIDTH_STEP

    def __init__(self, pm, arch: dict, key: tuple, B: int, width: int, dev):
        p = pm._pools
        self.key, self.pm, self.arch, self.pools, self.B, self.width = key, pm, arch, p, B, width
        w, nw = width, len(arch["windows"])
        self.ints = torch.zeros(B * w + (5 + nw) * B, dtype=torch.int32, device=dev)
        self.table = self.ints[: B * w].view(B, w)
        cols = self.ints[B * w:].view(5 + nw, B).unbind(0)
        self.num_blocks, self.hi, self.slots, self.positions, self.tail_start = cols[:5]
        self.los = cols[5:]  # first attended column per row, one per distinct window
        self.input_ids = torch.zeros(B, 1, dtype=torch.long, device=dev)
        self.position_ids = torch.zeros(B, 1, dtype=torch.long, device=dev)
        self.mass = torch.zeros(w, dtype=torch.float32, device=dev) if pm._needs_attention else None
        self.plans = [PagedDecodePlan(
            batch=B, num_query_heads=arch["hq"], dev_pool=p.dev_pool, host_pool=p.host_pool.tensor,
            num_layers=arch["layers"], tokens_per_block=pm.tokens_per_block, block_table=self.table,
            num_blocks=self.num_blocks, max_row_tokens=w * pm.tokens_per_block, valid_lo=lo, valid_hi=self.hi,
            scale=arch["scale"], softcap=arch["softcap"], mass_accum=self.mass,
            mass_mode="batch_mean" if self.mass is not None else "none", host_read="zero_copy",
            rounding=pm._rounding(arch), ref_group_tokens=pm._ref_group_tokens(), ref_tail_start=self.tail_start)
            for lo in self.los]
        self.device = torch.device(dev)
        self.graph = None
        self.logits = None

    def load(self, ints_cpu: torch.Tensor, input_ids: torch.Tensor, position_ids: torch.Tensor) -> None:
        self.ints.copy_(ints_cpu, non_blocking=False)
        self.input_ids.copy_(input_ids)
        self.position_ids.copy_(position_ids)

    def _run(self):
        if self.mass is not None:
            self.mass.zero_()
        group = AttentionGroup(self.pools, self.plans, self.slots, self.positions)
        return run_decoder_step(self.pm.model, self.arch, [group], self.input_ids, self.position_ids)

    def step(self) -> torch.Tensor:
        """Run the loaded step: the first time eagerly on a side stream (the step's own values, so
        its tail write is the one the replay repeats), then captured; afterwards by replay.  The
        capture is thread-local: threads driving other GPUs in the same process are not affected."""
        with torch.cuda.device(self.device):
            if self.graph is None:
                cur = torch.cuda.current_stream()
                side = torch.cuda.Stream()
                side.wait_stream(cur)
                with torch.cuda.stream(side):
                    self._run()
                cur.wait_stream(side)
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, capture_error_mode="thread_local"):
                    self.logits = self._run()
                self.graph = graph
            self.graph.replay()
        return self.logits


class PagedModel:
    """A HuggingFace causal LM whose KV cache lives in paged device / host pools."""

    def __init__(self, model, *, vram_budget: int, ram_budget: int, recent_window: int = 64,
                 rebalance_interval: int = 4, promote_margin: float = 0.05, ram_promote_margin: float = 0.20,
                 policy: str = "sinks_heavy_hitter", tokens_per_block: int = 16, prefill_chunk_tokens: int = 512,
                 use_streaming_attention: bool = True, streaming_group_size_blocks: int = 64,
                 host_read: str = "auto", pools: KVPools | None = None, decode_graphs: bool = True,
                 attention_rounding: str = "reference"):
        if not use_streaming_attention:
            raise NotImplementedError("only the streaming (fused paged) attention path is implemented")
        self.model = model
        self.tokens_per_block = tokens_per_block
        self.prefill_chunk_tokens = prefill_chunk_tokens
        self.use_streaming_attention = True
        # one launch per layer covers every group; the reference's groups still set the tiles its
        # one-pass path rounds p over, which the "reference" rounding reproduces
        self.streaming_group_size_blocks = streaming_group_size_blocks
        step_rounding(attention_rounding, False, torch.float16, 64, tokens_per_block)  # validates the name
        self.attention_rounding = attention_rounding
        self.host_read = host_read
        self.last_host_read: str | None = None  # the host-tier read mode of the last decode step's plan
        # decode steps captured and replayed as CUDA graphs (host tier read zero-copy); staged host
        # reads and models whose step cannot be captured keep the eager step
        self.decode_graphs = (bool(decode_graphs) and host_read != "staged"
                              and getattr(getattr(model, "config", None), "model_type", None)
                              not in _EAGER_ONLY_MODEL_TYPES)
        # pools shared with other single-row sessions (``batched_decode_step`` decodes them in one
        # launch); None: the session allocates its own
        if pools is not None and (pools.rows_per_group != 1 or pools.tokens_per_block != tokens_per_block):
            raise ValueError("shared pools must hold single-row blocks of tokens_per_block tokens")
        self.shared_pools = pools
        self._needs_attention = policy not in _POLICIES_WITHOUT_ATTENTION_SIGNAL
        self._ram_budget = ram_budget
        self._pager_kwargs = dict(vram=vram_budget, ram=ram_budget, recent=recent_window,
                                  rebalance_interval=rebalance_interval, promote_margin=promote_margin,
                                  ram_promote_margin=ram_promote_margin, policy=policy)
        self.last_run_stats: GenerationStats | None = None
        self._lock = threading.Lock()
        self._clear_session()

    # ------------------------------------------------------------------ session state
    def _clear_session(self):
        self._graph = None
        self._tail_past_override = None
        self._pools = None
        self._store = None
        self._rust_pager = None
        self._num_layers = None
        self._num_blocks = None
        self._tail_group = None
        self._tail_len = 0
        self._pad = None  # per row: left-padding columns
        self._total = 0  # columns in the sequence so far (padding included)
        self._mass_accum = None
        self._primed_tokens = 0
        self._primed_prefix = None

    @property
    def _tail_past(self):
        """The tail (tokens after the last full block) per layer as ``(key, value)`` views
        ``[rows, kv_heads, tail_len, head_dim]`` of the session's tail slots: the layout of the
        reference's ``_tail_past`` (``paged_model.py:638-641``), which its serving scheduler groups
        sessions by (``serving/scheduler.py:486``).  None without an active session."""
        if getattr(self, "_tail_past_override", None) is not None:
            return self._tail_past_override
        if self._store is None or self._pools is None:
            return None
        p = self._pools
        tail = p.dev_pool[p.group_slots(self._tail_group)]
        n = self._tail_len
        return [(tail[:, layer, 0, :, :n], tail[:, layer, 1, :, :n]) for layer in range(p.num_layers)]

    @_tail_past.setter
    def _tail_past(self, value):
        """Assignable like the reference's attribute (its tests build fake sessions by setting it);
        an assigned value is returned instead of the view until it is set back to None."""
        self._tail_past_override = value

    def _note_fed_token(self, token_id: int) -> None:
        """A token decoded outside ``generate`` (``batched_decode_step``) is now part of the session:
        extend the primed prefix so a later ``generate`` call continues after it instead of feeding
        it again."""
        tok = torch.tensor([[token_id]], dtype=self._primed_prefix.dtype)
        self._primed_prefix = torch.cat([self._primed_prefix, tok], dim=1)
        self._primed_tokens += 1

    def _acquire_or_raise(self) -> None:
        """Single-flight guard (``paged_model.py:270-282``): a second concurrent call is logged and
        rejected instead of waiting."""
        if not self._lock.acquire(blocking=False):
            logger.warning("PagedModel call rejected: another generate() or reset() is already in flight on "
                           "this instance.")
            raise RuntimeError(
                "Another generate() or reset() call is already running on this PagedModel instance. It holds one "
                "mutable session, so concurrent calls from another thread would corrupt its state rather than run "
                "as independent requests. Use a separate PagedModel per concurrent session, or synchronize calls "
                "to this one yourself.")

    def reset(self) -> None:
        """Drop the current session; the next generate() call starts fresh."""
        self._acquire_or_raise()
        try:
            self._release_pools()
            self._clear_session()
        finally:
            self._lock.release()

    def _release_pools(self):
        if self._store is not None:
            self._store.close()
        if self._pools is not None and self._pools is self.shared_pools:
            if self._tail_group is not None:
                self._pools.dev_groups.give(self._tail_group)
        elif self._pools is not None:
            self._pools.close()

    # ------------------------------------------------------------------ helpers
    @staticmethod
    def _validate_left_padded(attention_mask: torch.Tensor) -> None:
        mask = attention_mask.bool()
        if not mask.any(dim=1).all():
            raise NotImplementedError("attention_mask has a row with no real (non-padding) tokens.")
        if not torch.all(mask[:, :-1] <= mask[:, 1:]):
            raise NotImplementedError(
                "PagedModel only supports left-padding (zero or more leading zeros, then all ones, per row); "
                "right-padding or interleaved masking is not supported.")

    @staticmethod
    def _position_ids_from_mask(attention_mask: torch.Tensor) -> torch.Tensor:
        position_ids = attention_mask.long().cumsum(-1) - 1
        return position_ids.masked_fill(attention_mask == 0, 0)

    @staticmethod
    def _sample_next_token(logits, *, temperature, top_k, top_p, generator):
        """``paged_model.py:643-670``: temperature, top-k, top-p (nucleus), then a multinomial draw."""
        logits = logits / temperature
        if top_k is not None:
            kth_value = torch.topk(logits, min(top_k, logits.shape[-1]), dim=-1).values[:, -1, None]
            logits = logits.masked_fill(logits < kth_value, float("-inf"))
        if top_p is not None:
            sorted_logits, sorted_indices = torch.sort(logits, descending=True, dim=-1)
            sorted_probs = torch.softmax(sorted_logits, dim=-1)
            cumulative_probs = torch.cumsum(sorted_probs, dim=-1)
            sorted_logits = sorted_logits.masked_fill(cumulative_probs - sorted_probs > top_p, float("-inf"))
            logits = torch.full_like(logits, float("-inf")).scatter(-1, sorted_indices, sorted_logits)
        probs = torch.softmax(logits, dim=-1)
        return torch.multinomial(probs, num_samples=1, generator=generator)

    def _rounding(self, arch: dict) -> str:
        """The fused op's rounding of p for this session's decode steps (``step_rounding``)."""
        return step_rounding(self.attention_rounding, self._needs_attention, self.model.dtype, arch["d"],
                             self.tokens_per_block)

    def _ref_group_tokens(self) -> int:
        return self.streaming_group_size_blocks * self.tokens_per_block

    def _arch(self):
        cfg = self.model.config
        model_type = getattr(cfg, "model_type", None)
        if model_type not in _SUPPORTED_MODEL_TYPES:
            raise NotImplementedError(f"PagedModel doesn't recognize model_type={model_type!r}.")
        layers = self.model.model.layers
        attn = layers[0].self_attn
        head_dim = getattr(attn, "head_dim", cfg.hidden_size // cfg.num_attention_heads)
        per_layer = []
        for layer in layers:
            if model_type in _CONFIG_WINDOW_MODEL_TYPES:
                w = getattr(cfg, "sliding_window", None)
            else:
                w = getattr(layer.self_attn, "sliding_window", None)
            per_layer.append(int(w) if w else None)
        windows = sorted(set(per_layer), key=lambda w: (w is not None, w or 0))  # None (global) first
        return dict(layers=len(layers), hq=cfg.num_attention_heads, hkv=cfg.num_key_value_heads, d=head_dim,
                    scale=attn.scaling, windows=windows, layer_window=[windows.index(w) for w in per_layer],
                    softcap=getattr(attn, "attn_logit_softcapping", None) or None,
                    final_softcap=getattr(cfg, "final_logit_softcapping", None) or None,
                    qkv_fused=hasattr(attn, "qkv_proj"), sandwich_norms=hasattr(layers[0], "pre_feedforward_layernorm"))

    # ------------------------------------------------------------------ session start
    def _start_session(self, input_ids, attention_mask):
        """Prefill all but the last token with the model's own forward, then move its cache into the pools."""
        from transformers import DynamicCache

        a = self._arch()
        B, T = input_ids.shape
        dev = input_ids.device
        dtype = self.model.dtype
        tpb = self.tokens_per_block
        cache = DynamicCache()
        prefix = input_ids[:, :-1]
        pmask = attention_mask[:, :-1]
        pos_all = self._position_ids_from_mask(attention_mask)
        for s in range(0, prefix.shape[1], self.prefill_chunk_tokens):
            e = min(s + self.prefill_chunk_tokens, prefix.shape[1])
            self.model(input_ids=prefix[:, s:e], attention_mask=pmask[:, :e], position_ids=pos_all[:, s:e],
                       past_key_values=cache, use_cache=True)
        n = prefix.shape[1]
        nfull = n // tpb
        if self.shared_pools is not None:
            if B != 1:
                raise ValueError("a session on shared pools is single-row")
            self._pools = self.shared_pools
        else:
            # Both tiers get a group for every block (plus the tail and room for new blocks): a
            # rebalance may demote blocks before its promotions free their host groups, and growing the
            # pinned host pool mid-decode (a new allocation of twice the size plus a copy) takes seconds.
            self._pools = KVPools(num_layers=a["layers"], kv_heads=a["hkv"], head_dim=a["d"], tokens_per_block=tpb,
                                  dtype=dtype, device=dev, rows_per_group=B, gpu_groups=max(nfull + 2, 2),
                                  cpu_groups=max(4, nfull + 2))
        self._store = KVBlockStore(tpb, self._ram_budget, pools=self._pools)
        keys = [layer.keys for layer in cache.layers]
        values = [layer.values for layer in cache.layers]
        for j in range(nfull):
            self._store.put_gpu_layers(j, [k[:, :, j * tpb:(j + 1) * tpb] for k in keys],
                                       [v[:, :, j * tpb:(j + 1) * tpb] for v in values])
        self._tail_group = self._pools.take_dev_group()
        rem = n - nfull * tpb
        tail = self._pools.dev_pool[self._pools.group_slots(self._tail_group)]
        for layer in range(a["layers"]):
            tail[:, layer, 0, :, :rem].copy_(keys[layer][:, :, nfull * tpb:])
            tail[:, layer, 1, :, :rem].copy_(values[layer][:, :, nfull * tpb:])
        del cache, keys, values
        self._num_layers = a["layers"]
        self._num_blocks = nfull
        self._tail_len = rem
        self._total = n
        self._pad = (attention_mask == 0).sum(dim=1).to(torch.int32)  # left padding per row
        import pager as _pager

        self._rust_pager = _pager.PyPager(**self._pager_kwargs)
        logger.info("Started PagedModel session: batch_size=%d prompt_tokens=%d layers=%d blocks=%d policy=%r",
                    B, T, a["layers"], nfull, self._pager_kwargs["policy"])

    # ------------------------------------------------------------------ one decode step
    def _block_attention(self) -> list[float]:
        n = self._num_blocks
        if n == 0 or self._mass_accum is None:
            return [1.0 / n] * n if n else []
        averaged = (self._mass_accum / self._num_layers).tolist()
        total = sum(averaged)
        if total <= 0:
            return [1.0 / n] * n
        return [x / total for x in averaged]

    def _forward_step(self, input_ids: torch.Tensor, attention_mask: torch.Tensor):
        """One token per row through the model with paged attention; then blocks, pager, tiers."""
        a = self._arch()
        B = input_ids.shape[0]
        dev = input_ids.device
        p = self._pools
        tpb = self.tokens_per_block
        nb = self._num_blocks
        total = self._total + 1  # columns including this step's token
        # block table: row b reads slot (group * B + b) of each block's group, then its tail slot
        table = torch.full((B, nb + 1), -1, dtype=torch.int32)
        if nb:
            table[:, :nb] = self._store.block_table(range(nb), device="cpu")
        table[:, nb] = torch.arange(self._tail_group * B, self._tail_group * B + B, dtype=torch.int32)
        pad = self._pad.to("cpu", torch.int32)
        # first attended column per row, one row of values per distinct sliding window
        los = [torch.tensor([window_lo(int(x), total, w) for x in pad], dtype=torch.int32) for w in a["windows"]]
        if self.decode_graphs:
            return self._graph_step(a, B, nb, table, los, total, input_ids, attention_mask)
        i32 = dict(dtype=torch.int32, device=dev)
        mass = torch.zeros(nb + 1, dtype=torch.float32, device=dev) if self._needs_attention else None
        table_dev = table.to(dev)
        plans = [PagedDecodePlan(
            batch=B, num_query_heads=a["hq"], dev_pool=p.dev_pool, host_pool=p.host_pool.tensor,
            num_layers=a["layers"], tokens_per_block=tpb, block_table=table_dev,
            num_blocks=torch.full((B,), nb + 1, **i32), max_row_tokens=(nb + 1) * tpb,
            valid_lo=lo.to(dev) if bool((lo > 0).any()) else None, valid_hi=torch.full((B,), total, **i32),
            scale=a["scale"], softcap=a["softcap"], mass_accum=mass,
            mass_mode="batch_mean" if mass is not None else "none", host_read=self.host_read,
            rounding=self._rounding(a), ref_group_tokens=self._ref_group_tokens(),
            ref_tail_start=torch.full((B,), nb * tpb, **i32)) for lo in los]
        self.last_host_read = plans[0].host_read
        slots = torch.arange(self._tail_group * B, self._tail_group * B + B, **i32)
        positions = torch.full((B,), self._tail_len, **i32)
        position_ids = self._position_ids_from_mask(attention_mask)[:, -1:]
        logits = run_decoder_step(self.model, a, [AttentionGroup(p, plans, slots, positions)], input_ids, position_ids)
        L.watch_for(dev).sync_and_check("PagedModel decode step")
        return logits, self._finish_token(None if mass is None else mass[:nb])

    def _graph_step(self, a, B, nb, table, los, total, input_ids, attention_mask):
        """``_forward_step`` through a captured graph (``_DecodeGraph``); same inputs, same result."""
        p = self._pools
        width = _DecodeGraph.width_for(nb)
        key = (B, width, id(p), p.version, self._needs_attention)
        if self._graph is None or self._graph.key != key:
            self._graph = None  # release the previous graph's memory before capturing the next
            self._graph = _DecodeGraph(self, a, key, B, width, input_ids.device)
        g = self._graph
        wide = torch.full((B, width), -1, dtype=torch.int32)
        wide[:, : nb + 1] = table
        ints = torch.cat([wide.reshape(-1), torch.full((B,), nb + 1, dtype=torch.int32),
                          torch.full((B,), total, dtype=torch.int32),
                          torch.arange(self._tail_group * B, self._tail_group * B + B, dtype=torch.int32),
                          torch.full((B,), self._tail_len, dtype=torch.int32),
                          torch.full((B,), nb * self.tokens_per_block, dtype=torch.int32)] + los)
        g.load(ints, input_ids, self._position_ids_from_mask(attention_mask)[:, -1:])
        logits = g.step().clone()  # the graph's logits buffer is overwritten by the next replay
        self.last_host_read = "zero_copy"
        L.watch_for(input_ids.device).sync_and_check("PagedModel decode step")
        return logits, self._finish_token(None if g.mass is None else g.mass[:nb])

    def _finish_token(self, mass_row):
        """After a decoded token (``paged_model.py:1210-1233, :785-798``): roll a full tail into a block
        (adopted in place), hand the step's block attention to the pager, move blocks to its tiers.
        ``mass_row``: this session's accumulated block mass over the layers (device tensor) or None."""
        p = self._pools
        dev = p.device
        nb = self._num_blocks
        self._total += 1
        self._tail_len += 1
        added = []
        if self._tail_len == self.tokens_per_block:
            self._store.adopt_gpu_group(nb, self._tail_group)
            added.append(nb)
            self._num_blocks = nb + 1
            self._tail_group = p.take_dev_group()
            self._tail_len = 0
        self._mass_accum = mass_row.cpu() if mass_row is not None else None
        step = {"new_blocks": len(added), "gpu_to_cpu_mb": 0.0, "cpu_to_gpu_mb": 0.0, "gpu_to_cpu_copies": 0,
                "cpu_to_gpu_copies": 0, "attention_in_gpu": 0.0}
        if self._num_blocks == 0:
            return step
        block_attention = (self._block_attention() if self._needs_attention
                           else [1.0 / self._num_blocks] * self._num_blocks)
        before = self._store.summary()
        query_block = self._num_blocks - 1
        self._rust_pager.on_step(query_block, 0, block_attention)
        if added:
            self._rust_pager.force_rebalance(query_block)
        self._store.apply_tiers(self._rust_pager.tiers(), dev)
        after = self._store.summary()
        step.update(gpu_to_cpu_mb=(after["gpu_to_cpu_bytes"] - before["gpu_to_cpu_bytes"]) / 1e6,
                    cpu_to_gpu_mb=(after["cpu_to_gpu_bytes"] - before["cpu_to_gpu_bytes"]) / 1e6,
                    gpu_to_cpu_copies=after["gpu_to_cpu_copies"] - before["gpu_to_cpu_copies"],
                    cpu_to_gpu_copies=after["cpu_to_gpu_copies"] - before["cpu_to_gpu_copies"],
                    attention_in_gpu=sum(block_attention[i] for i in self._store.gpu_block_ids()
                                         if i < len(block_attention)))
        return step

    def _reorder_rows(self, rows: list[int]) -> None:
        """Row i of the session continues old row ``rows[i]`` (``paged_model.py:612-622``): every block's
        rows on both tiers (``KVBlockStore.reorder_batch_rows``), the tail slots and the left padding."""
        self._store.reorder_batch_rows(rows)
        p = self._pools
        idx = torch.tensor(rows, dtype=torch.long, device=p.device)
        tail = p.dev_pool[p.group_slots(self._tail_group)]
        tail.copy_(tail.index_select(0, idx))
        self._pad = self._pad.index_select(0, idx.to(self._pad.device))

    def _extend_session(self, input_ids, attention_mask):
        total_len = input_ids.shape[-1]
        if total_len - 1 < self._primed_tokens:
            raise ValueError(
                "input_ids is shorter than the already-primed session "
                f"({total_len - 1} < {self._primed_tokens} tokens). "
                "Call reset() to start a new session instead of rewinding one.")
        if not torch.equal(input_ids[:, :self._primed_tokens].cpu(), self._primed_prefix):
            raise ValueError(
                "input_ids diverges from the already-primed session prefix. generate() expects each call to extend "
                "the same growing sequence (previous input + previously generated tokens + any new tokens). Call "
                "reset() to start a different session.")
        pending = input_ids[:, self._primed_tokens:total_len - 1]
        for i in range(pending.shape[-1]):
            self._forward_step(pending[:, i:i + 1], attention_mask[:, :self._primed_tokens + i + 1])

    # ------------------------------------------------------------------ public API
    @torch.inference_mode()
    def generate(self, input_ids: torch.Tensor, attention_mask: torch.Tensor, max_new_tokens: int, *,
                 do_sample: bool = False, temperature: float = 1.0, top_k: int | None = None,
                 top_p: float | None = None, generator: torch.Generator | None = None):
        """Generate up to max_new_tokens tokens, continuing any previous session on this model."""
        self._acquire_or_raise()
        try:
            batch_size = input_ids.shape[0]
            self._validate_left_padded(attention_mask)
            if do_sample:
                if temperature <= 0:
                    raise ValueError(f"temperature must be > 0 for sampling, got {temperature}.")
                if top_k is not None and top_k < 1:
                    raise ValueError(f"top_k must be >= 1, got {top_k}.")
                if top_p is not None and not (0.0 < top_p <= 1.0):
                    raise ValueError(f"top_p must be in (0, 1], got {top_p}.")
            fresh = self._store is None
            if fresh:
                self._start_session(input_ids, attention_mask)
            else:
                self._extend_session(input_ids, attention_mask)
            next_input_id = input_ids[:, -1:]
            mask = attention_mask
            generated: list[list[int]] = [[] for _ in range(batch_size)]
            stats = GenerationStats()
            in_gpu = []
            for _ in range(max_new_tokens):
                logits, step = self._forward_step(next_input_id, mask)
                if do_sample:
                    nxt = self._sample_next_token(logits[:, -1, :], temperature=temperature, top_k=top_k,
                                                  top_p=top_p, generator=generator)
                else:
                    nxt = torch.argmax(logits[:, -1, :], dim=-1, keepdim=True)
                for row, tok in zip(generated, nxt[:, 0].tolist()):
                    row.append(tok)
                stats.total_new_blocks += step["new_blocks"]
                stats.total_gpu_to_cpu_mb += step["gpu_to_cpu_mb"]
                stats.total_cpu_to_gpu_mb += step["cpu_to_gpu_mb"]
                stats.total_gpu_to_cpu_copies += step["gpu_to_cpu_copies"]
                stats.total_cpu_to_gpu_copies += step["cpu_to_gpu_copies"]
                in_gpu.append(step["attention_in_gpu"])
                next_input_id = nxt
                mask = torch.cat([mask, torch.ones((mask.shape[0], 1), dtype=mask.dtype, device=mask.device)], dim=1)
            full = torch.cat([input_ids, torch.tensor(generated, dtype=input_ids.dtype, device=input_ids.device)],
                             dim=1)
            self._primed_prefix = full[:, :-1].detach().cpu()
            self._primed_tokens = full.shape[-1] - 1
            stats.final_num_blocks = self._num_blocks
            if in_gpu:
                stats.mean_attention_in_gpu = sum(in_gpu) / len(in_gpu)
                stats.min_attention_in_gpu = min(in_gpu)
                stats.max_attention_in_gpu = max(in_gpu)
            self.last_run_stats = stats
            return generated[0] if batch_size == 1 else generated
        finally:
            self._lock.release()

    @torch.inference_mode()
    def generate_beam_search(self, input_ids: torch.Tensor, attention_mask: torch.Tensor, num_beams: int,
                             max_new_tokens: int, *, eos_token_id: int | None = None, length_penalty: float = 1.0,
                             num_return_sequences: int = 1, do_sample: bool = False, temperature: float = 1.0,
                             top_k: int | None = None, top_p: float | None = None,
                             generator: torch.Generator | None = None):
        """Beam search (``paged_model.py:409-610``): ``num_beams`` hypotheses per prompt, each a row of
        the session with its own KV history, advanced together one token per step; each step keeps the
        ``num_beams`` best continuations over all beams of a prompt (or samples them without replacement
        under ``do_sample``, after temperature / top-k / top-p), and the rows are reordered to their
        parents (``_reorder_rows``).  Only the first beam of a prompt starts live (the others at -inf);
        a beam that emitted ``eos_token_id`` may only repeat it at no score change.  Final candidates
        are ranked per prompt by score / length ** ``length_penalty``.  Every call starts a fresh
        session and ends it.  Returns, like ``generate``: one list of tokens for one prompt and one
        sequence, a list of lists for several prompts or several sequences, a list of lists of lists
        for both."""
        self._acquire_or_raise()
        try:
            batch = input_ids.shape[0]
            if num_beams < 1:
                raise ValueError(f"num_beams must be >= 1, got {num_beams}")
            if not 1 <= num_return_sequences <= num_beams:
                raise ValueError(f"num_return_sequences must be between 1 and num_beams ({num_beams}), got "
                                 f"{num_return_sequences}")
            if do_sample:
                if temperature <= 0:
                    raise ValueError(f"temperature must be > 0 for sampling, got {temperature}.")
                if top_k is not None and top_k < 1:
                    raise ValueError(f"top_k must be >= 1, got {top_k}.")
                if top_p is not None and not (0.0 < top_p <= 1.0):
                    raise ValueError(f"top_p must be in (0, 1], got {top_p}.")
            self._validate_left_padded(attention_mask)
            if self._store is not None:  # beam search starts its own session
                self._release_pools()
                self._clear_session()
            device = input_ids.device
            rows = batch * num_beams
            ids = input_ids.repeat_interleave(num_beams, dim=0)
            mask = attention_mask.repeat_interleave(num_beams, dim=0)
            self._start_session(ids, mask)
            try:
                nxt = ids[:, -1:]
                scores = torch.full((rows,), float("-inf"), dtype=torch.float32, device=device)
                scores[0::num_beams] = 0.0
                tokens: list[list[int]] = [[] for _ in range(rows)]
                finished = [False] * rows
                group_base = torch.arange(batch, device=device).unsqueeze(1) * num_beams
                for _ in range(max_new_tokens):
                    logits, _ = self._forward_step(nxt, mask)
                    logp = torch.log_softmax(logits[:, -1, :].float(), dim=-1)
                    vocab = logp.shape[-1]
                    if eos_token_id is not None and any(finished):
                        done = torch.tensor(finished, device=device)
                        frozen = torch.full((vocab,), float("-inf"), device=device)
                        frozen[eos_token_id] = 0.0
                        logp = torch.where(done[:, None], frozen[None, :], logp)
                    cand = logp
                    if do_sample:
                        cand = logp / temperature
                        if top_k is not None:
                            kth = torch.topk(cand, min(top_k, vocab), dim=-1).values[:, -1, None]
                            cand = cand.masked_fill(cand < kth, float("-inf"))
                        if top_p is not None:
                            srt, order = torch.sort(cand, descending=True, dim=-1)
                            pr = torch.softmax(srt, dim=-1)
                            srt = srt.masked_fill(torch.cumsum(pr, dim=-1) - pr > top_p, float("-inf"))
                            cand = torch.full_like(cand, float("-inf")).scatter(-1, order, srt)
                        cand = torch.log_softmax(cand, dim=-1)
                    joint = (scores[:, None] + cand).view(batch, num_beams * vocab)
                    if do_sample:
                        pick = torch.multinomial(torch.softmax(joint, dim=-1), num_beams, replacement=False,
                                                 generator=generator)
                        best = torch.gather(joint, 1, pick)
                    else:
                        best, pick = torch.topk(joint, num_beams, dim=-1)
                    parents = (pick // vocab + group_base).flatten().tolist()
                    chosen = (pick % vocab).flatten().tolist()
                    tokens = [tokens[par] + [tok] for par, tok in zip(parents, chosen)]
                    finished = [finished[par] or (eos_token_id is not None and tok == eos_token_id)
                                for par, tok in zip(parents, chosen)]
                    scores = best.flatten()
                    self._reorder_rows(parents)
                    nxt = torch.tensor(chosen, dtype=input_ids.dtype, device=device).unsqueeze(1)
                    mask = torch.cat([mask[parents], torch.ones((rows, 1), dtype=mask.dtype, device=device)], dim=1)
                    if all(finished):
                        break
            finally:
                self._release_pools()
                self._clear_session()
            results = []
            for g in range(batch):
                ranked = []
                for r in range(g * num_beams, (g + 1) * num_beams):
                    seq = tokens[r]
                    if eos_token_id is not None and eos_token_id in seq:
                        seq = seq[: seq.index(eos_token_id) + 1]
                    ranked.append((float(scores[r]) / (max(len(seq), 1) ** length_penalty), seq))
                ranked.sort(key=lambda item: item[0], reverse=True)
                results.append([seq for _, seq in ranked[:num_return_sequences]])
            if batch == 1:
                return results[0][0] if num_return_sequences == 1 else results[0]
            return [r[0] for r in results] if num_return_sequences == 1 else results
        finally:
            self._lock.release()
