"""Seeded input builders for the golden parity cases.

Shared by ``make_golden.py`` (which runs the reference's own kernels on these
inputs, on the CPU) and by the tests (which rebuild the same inputs from the
same seeds and compare the oracle / the CUDA path against the stored outputs).
Inputs are rebuilt from the torch CPU generator, so the fixtures only store
outputs plus a sha256 of the inputs to catch any drift in the generator.

Every case describes one call sequence the reference makes:

* ``steps``     -- repeated ``streaming_attention_step`` over fixed-size
                   groups (tests/test_streaming_attention.py:43-62 style);
* ``two_pass``  -- ``stats_step`` over groups + tail, then
                   ``accumulate_step`` over groups + ``fold_fixed_step`` on
                   the tail (pager_hf/paged_model.py:993-1039);
* ``batched``   -- the cross-session layout of pager_hf/batched_decode.py:
                   sessions with different block counts, front-padded with
                   all-invalid blocks in a shared numbering, ``active`` per
                   group, equal tail length (batched_decode.py:110-285).
"""

from __future__ import annotations

import hashlib

import torch

DT = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}


def _randn(shape, dtype, gen=None):
    return torch.randn(*shape, dtype=DT[dtype], generator=gen)


def input_digest(tensors) -> str:
    h = hashlib.sha256()
    for t in tensors:
        if t is None:
            h.update(b"none")
            continue
        t = t.contiguous()
        h.update(str(tuple(t.shape)).encode())
        h.update(str(t.dtype).encode())
        h.update(t.reshape(-1).view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


CASES = {
    # tests/test_streaming_attention.py:43-62
    "ref_single_pass": dict(kind="steps", seed=0, B=1, Hq=14, Hkv=2, D=64, T=200, group=48, dtype="f16"),
    # tests/test_streaming_attention.py:65-119
    "ref_two_pass_tail": dict(kind="two_pass", seed=0, B=1, Hq=14, Hkv=2, D=64, tpb=16, nb=9, tail=7,
                              group_blocks=2, dtype="f16"),
    # tests/test_streaming_attention.py:122-142
    "ref_batched_rows": dict(kind="steps", seed=1, B=2, Hq=14, Hkv=2, D=64, T=96, group=32, dtype="f16"),
    # tests/test_streaming_attention.py:145-171
    "ref_padding_mask": dict(kind="steps", seed=2, B=1, Hq=14, Hkv=2, D=64, T=64, group=64, dtype="f16",
                             pad_prefix=[20]),
    # tests/test_streaming_attention.py:174-207
    "ref_active_zero_step": dict(kind="steps", seed=4, B=2, Hq=14, Hkv=2, D=64, T=32, group=32, dtype="f16",
                                 active=[0, 1]),
    # tests/test_streaming_attention.py:210-240 (stats + accumulate, no tail)
    "ref_active_zero_two_pass": dict(kind="two_pass", seed=5, B=2, Hq=14, Hkv=2, D=64, tpb=16, nb=2, tail=0,
                                     group_blocks=2, dtype="f16", active=[0, 1]),
    # tests/test_streaming_attention.py:243-272 (softcap: dense reference)
    "ref_softcap": dict(kind="steps", seed=6, B=1, Hq=14, Hkv=2, D=64, T=96, group=32, dtype="f16",
                        scale=224.0**-0.5, softcap=50.0),
    # tests/test_streaming_attention.py:275-293
    "ref_default_scale": dict(kind="steps", seed=7, B=1, Hq=14, Hkv=2, D=64, T=64, group=64, dtype="f16"),
    # the CPU benchmark config: Qwen2.5-0.5B geometry, fp32, 4096 tokens in 64 blocks of 64, seed 0 (q, k, v)
    "cfg1_qwen05b_f32": dict(kind="two_pass", seed=0, B=1, Hq=14, Hkv=2, D=64, tpb=64, nb=64, tail=0,
                             group_blocks=64, dtype="f32", randn_order="qkv"),
    "cfg1_qwen05b_f32_onepass": dict(kind="steps", seed=0, B=1, Hq=14, Hkv=2, D=64, T=4096, group=4096,
                                     dtype="f32"),
    # Llama-3 / Mistral attention geometry, ragged left padding, several groups
    "gqa4_d128_f16_padded": dict(kind="two_pass", seed=11, B=3, Hq=32, Hkv=8, D=128, tpb=64, nb=5, tail=9,
                                 group_blocks=2, dtype="f16", pad_prefix=[0, 70, 200]),
    # bf16 data; the interpreter cannot run bf16, so the reference runs on fp32 copies of the bf16 values
    "gqa4_d128_bf16_as_f32": dict(kind="two_pass", seed=14, B=2, Hq=32, Hkv=8, D=128, tpb=64, nb=4, tail=5,
                                  group_blocks=3, dtype="bf16", pad_prefix=[0, 100]),
    # TinyLlama geometry (n_rep 8), a general 0/1 mask with holes, tpb 32
    "gqa8_d64_f16_holes": dict(kind="two_pass", seed=12, B=2, Hq=32, Hkv=4, D=64, tpb=32, nb=7, tail=3,
                               group_blocks=4, dtype="f16", holes=0.25),
    # Gemma geometry (head_dim 256, n_rep 2), left-padded rows, two-pass with block mass
    "gemma_d256_f16_padded": dict(kind="two_pass", seed=15, B=2, Hq=8, Hkv=4, D=256, tpb=16, nb=6, tail=5,
                                  group_blocks=2, dtype="f16", pad_prefix=[0, 20]),
    # the shapes the fused paged op's GPU parity cases compare with the oracle: GQA fan-out 16
    # (the most _validate_n_rep allows), plain MHA, head_dim 8 to 256 across fp16, bf16 and fp32
    "pin_n_rep_16_d128_f16": dict(kind="two_pass", seed=31, B=2, Hq=32, Hkv=2, D=128, tpb=64, nb=4, tail=7,
                                  group_blocks=2, dtype="f16", pad_prefix=[0, 90]),
    "pin_mha_d64_f16_holes": dict(kind="two_pass", seed=32, B=2, Hq=4, Hkv=4, D=64, tpb=32, nb=5, tail=11,
                                  group_blocks=2, dtype="f16", holes=0.2),
    "pin_d32_f16": dict(kind="two_pass", seed=33, B=2, Hq=6, Hkv=3, D=32, tpb=16, nb=9, tail=15,
                        group_blocks=4, dtype="f16"),
    "pin_d8_f32": dict(kind="two_pass", seed=34, B=3, Hq=4, Hkv=2, D=8, tpb=16, nb=5, tail=2,
                       group_blocks=2, dtype="f32"),
    "pin_d16_f32_steps": dict(kind="steps", seed=35, B=2, Hq=8, Hkv=2, D=16, T=80, group=40, dtype="f32"),
    "pin_d8_f16_steps": dict(kind="steps", seed=36, B=2, Hq=6, Hkv=2, D=8, T=72, group=24, dtype="f16"),
    "pin_d256_f32": dict(kind="two_pass", seed=37, B=1, Hq=4, Hkv=2, D=256, tpb=16, nb=3, tail=9,
                         group_blocks=2, dtype="f32"),
    "pin_d32_bf16_as_f32": dict(kind="two_pass", seed=38, B=2, Hq=8, Hkv=2, D=32, tpb=32, nb=4, tail=6,
                                group_blocks=3, dtype="bf16", pad_prefix=[0, 40]),
    # cross-session batched decode (batched_decode.py): block counts 6, 2, 0; tail 4 (+1 new token)
    "batched_sessions_f16": dict(kind="batched", seed=13, Hq=14, Hkv=2, D=64, tpb=16, nbs=[6, 2, 0], tail=4,
                                 group_blocks=4, dtype="f16"),
    # native bf16 (fixtures from the reference's Triton kernels on a B200, make_golden.py --gpu): the
    # reference's own rounding of p to bf16 is in these vectors
    "bf16_steps_gqa4_d128": dict(kind="steps", seed=41, B=2, Hq=32, Hkv=8, D=128, T=1100, group=512, dtype="bf16",
                                 pad_prefix=[0, 130], gpu_only=True),
    "bf16_two_pass_gqa8_d64": dict(kind="two_pass", seed=42, B=2, Hq=32, Hkv=4, D=64, tpb=64, nb=9, tail=17,
                                   group_blocks=4, dtype="bf16", pad_prefix=[0, 77], gpu_only=True),
    "bf16_batched_gqa4_d128": dict(kind="batched", seed=43, Hq=32, Hkv=8, D=128, tpb=16, nbs=[9, 3, 6], tail=5,
                                   group_blocks=4, dtype="bf16", gpu_only=True),
}

# cases whose reference outputs also exist as fixtures from the reference's kernels on a GPU, in the
# cases' native dtype (``<case>__gpu.npz``)
GPU_CASES = ("gqa4_d128_bf16_as_f32", "pin_d32_bf16_as_f32", "bf16_steps_gqa4_d128", "bf16_two_pass_gqa8_d64",
             "bf16_batched_gqa4_d128")


def build_contiguous(case):
    """Inputs for ``steps`` / ``two_pass`` cases: q [B,Hq,D], k/v [B,Hkv,T,D], valid [B,T], active [B]."""
    c = CASES[case] if isinstance(case, str) else case
    torch.manual_seed(c["seed"])
    B, Hq, Hkv, D, dt = c["B"], c["Hq"], c["Hkv"], c["D"], c["dtype"]
    T = c["T"] if c["kind"] == "steps" else c["nb"] * c["tpb"] + c["tail"]
    q = _randn((B, Hq, D), dt)
    k = _randn((B, Hkv, T, D), dt)
    v = _randn((B, Hkv, T, D), dt)
    valid = torch.ones(B, T, dtype=torch.int32)
    for row, pad in enumerate(c.get("pad_prefix", [])):
        valid[row, :pad] = 0
    if c.get("holes"):
        g = torch.Generator().manual_seed(c["seed"] + 1000)
        holes = torch.rand(B, T, generator=g) < c["holes"]
        valid[holes] = 0
        valid[:, -1] = 1  # the new token is always attended
    active = torch.tensor(c.get("active", [1] * B), dtype=torch.int32)
    return q, k, v, valid, active


def build_batched(case):
    """Inputs for a ``batched`` case.

    Returns per-session block K/V ([nb, Hkv, tpb, D] each) and tails
    ([Hkv, tail+1, D], the last token being the new one) plus q [S,Hq,D].
    """
    c = CASES[case] if isinstance(case, str) else case
    torch.manual_seed(c["seed"])
    S = len(c["nbs"])
    Hq, Hkv, D, tpb, dt = c["Hq"], c["Hkv"], c["D"], c["tpb"], c["dtype"]
    q = _randn((S, Hq, D), dt)
    blocks_k, blocks_v, tails_k, tails_v = [], [], [], []
    for nb in c["nbs"]:
        blocks_k.append(_randn((nb, Hkv, tpb, D), dt))
        blocks_v.append(_randn((nb, Hkv, tpb, D), dt))
        tails_k.append(_randn((Hkv, c["tail"] + 1, D), dt))
        tails_v.append(_randn((Hkv, c["tail"] + 1, D), dt))
    return q, blocks_k, blocks_v, tails_k, tails_v


def batched_combined_layout(case, blocks_k, blocks_v, tails_k, tails_v):
    """The combined front-padded layout batched_decode.py builds (:110-118, :183-236).

    Returns (k [S,Hkv,max_blocks*tpb,D], v, valid [S,max_blocks*tpb], pad_blocks,
    tail_k [S,Hkv,t,D], tail_v).  Padding blocks are zeros with valid 0
    (batched_decode.py:209-216).
    """
    c = CASES[case] if isinstance(case, str) else case
    tpb, Hkv, D = c["tpb"], c["Hkv"], c["D"]
    nbs = c["nbs"]
    max_blocks = max(nbs)
    S = len(nbs)
    dt = DT[c["dtype"]]
    k = torch.zeros(S, Hkv, max_blocks * tpb, D, dtype=dt)
    v = torch.zeros_like(k)
    valid = torch.zeros(S, max_blocks * tpb, dtype=torch.int32)
    pad_blocks = [max_blocks - nb for nb in nbs]
    for row, nb in enumerate(nbs):
        for j in range(nb):
            pos = pad_blocks[row] + j
            k[row, :, pos * tpb : (pos + 1) * tpb] = blocks_k[row][j]
            v[row, :, pos * tpb : (pos + 1) * tpb] = blocks_v[row][j]
            valid[row, pos * tpb : (pos + 1) * tpb] = 1
    tail_k = torch.stack(tails_k, 0)
    tail_v = torch.stack(tails_v, 0)
    return k, v, valid, pad_blocks, tail_k, tail_v


def group_row_active(pad_blocks, i, group_len):
    """batched_decode.py:222-236."""
    return torch.tensor([1 if p < i + group_len else 0 for p in pad_blocks], dtype=torch.int32)
