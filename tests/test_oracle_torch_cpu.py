"""The vectorised torch restatement used for model-level parity equals the numpy oracle.

``oracle/streaming_attention_torch.reference_decode`` must compute what the numpy restatement of
the reference's call sequences computes -- ``single_pass_decode`` (paged_model.py:1055-1072) for
the running-max rule, ``two_pass_decode`` (:993-1039) for the final-max rule -- on the same inputs:
outputs within fp32 rounding before the final cast (the torch form sums in another order), masses
within 1e-6 relative, and the rounded outputs equal in all but a sliver of elements.
"""

import numpy as np
import pytest
import torch

from oracle import streaming_attention_oracle as orc
from oracle import streaming_attention_torch as ort


def _case(seed, B, Hq, Hkv, D, nb, tpb, tail, dtype, pad=0, window=None):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, D, generator=g).to(dtype)
    k = torch.randn(B, Hkv, nb * tpb + tail, D, generator=g).to(dtype)
    v = torch.randn(B, Hkv, nb * tpb + tail, D, generator=g).to(dtype)
    valid = torch.ones(B, nb * tpb + tail, dtype=torch.int32)
    valid[:, :pad] = 0
    if window is not None:
        valid[:, : max(0, nb * tpb + tail - window)] = 0
    return q, k, v, valid


def _np(x):
    return x.float().numpy()


@pytest.mark.parametrize("dtype,vd", [(torch.bfloat16, "bf16"), (torch.float16, "f16"), (torch.float32, "f32")])
@pytest.mark.parametrize("gs,pad,window", [(2, 0, None), (64, 5, None), (3, 0, 50)])
def test_running_rule_matches_single_pass_sequence(dtype, vd, gs, pad, window):
    B, Hq, Hkv, D, nb, tpb, tail = 2, 8, 2, 64, 9, 16, 7
    q, k, v, valid = _case(1, B, Hq, Hkv, D, nb, tpb, tail, dtype, pad, window)
    full = nb * tpb
    out, m, l = orc.single_pass_decode(_np(q), _np(k[:, :, :full]), _np(v[:, :, :full]), _np(k[:, :, full:]),
                                       _np(v[:, :, full:]), nb, tpb, gs, valid=valid[:, :full].numpy(),
                                       tail_valid=valid[:, full:].numpy(), v_dtype=vd, out_dtype="f32")
    keys = ort.reference_tile_keys(full + tail, full, group_tokens=gs * tpb)[None].expand(B, -1)
    t_out, t_m, t_l, _ = ort.reference_decode(q, k, v, valid, keys, "running", out_dtype=torch.float32)
    np.testing.assert_allclose(t_out.numpy(), out, rtol=2e-6, atol=2e-6)
    np.testing.assert_allclose(t_m.numpy(), m, rtol=1e-6, atol=1e-6)  # the dot product sums in another order
    np.testing.assert_allclose(t_l.numpy(), l, rtol=2e-6)


@pytest.mark.parametrize("dtype,vd", [(torch.bfloat16, "bf16"), (torch.float16, "f16")])
def test_final_rule_matches_two_pass_sequence(dtype, vd):
    B, Hq, Hkv, D, nb, tpb, tail = 2, 16, 2, 128, 11, 16, 5
    q, k, v, valid = _case(2, B, Hq, Hkv, D, nb, tpb, tail, dtype, pad=9)
    full = nb * tpb
    out, mass, m, l = orc.two_pass_decode(_np(q), _np(k[:, :, :full]), _np(v[:, :, :full]), _np(k[:, :, full:]),
                                          _np(v[:, :, full:]), nb, tpb, 4, valid=valid[:, :full].numpy(),
                                          tail_valid=valid[:, full:].numpy(), v_dtype=vd, out_dtype="f32")
    keys = ort.reference_tile_keys(full + tail, full)[None].expand(B, -1)
    t_out, t_m, t_l, pl = ort.reference_decode(q, k, v, valid, keys, "final", out_dtype=torch.float32)
    np.testing.assert_allclose(t_out.numpy(), out, rtol=2e-6, atol=2e-6)
    np.testing.assert_allclose(t_m.numpy(), m, rtol=1e-6, atol=1e-6)  # the dot product sums in another order
    np.testing.assert_allclose(t_l.numpy(), l, rtol=2e-6)
    t_mass = pl[:, :, :full].reshape(B, Hq, nb, tpb).sum(-1)
    np.testing.assert_allclose(t_mass.numpy(), mass, rtol=1e-5, atol=1e-7)


def test_rounded_outputs_agree_bitwise_almost_everywhere():
    """In the output dtype the two restatements differ only where fp32 association moves a value
    across a rounding boundary."""
    B, Hq, Hkv, D, nb, tpb, tail = 4, 32, 8, 128, 8, 64, 20
    q, k, v, valid = _case(3, B, Hq, Hkv, D, nb, tpb, tail, torch.bfloat16)
    full = nb * tpb
    out, _, _ = orc.single_pass_decode(_np(q), _np(k[:, :, :full]), _np(v[:, :, :full]), _np(k[:, :, full:]),
                                       _np(v[:, :, full:]), nb, tpb, 64, v_dtype="bf16", out_dtype="bf16")
    keys = ort.reference_tile_keys(full + tail, full, group_tokens=64 * tpb)[None].expand(B, -1)
    t_out = ort.reference_decode(q, k, v, valid, keys, "running")[0]
    differ = (t_out.float().numpy() != out).mean()
    assert differ < 0.01, differ


def test_tile_keys_follow_the_reference_chunks():
    # groups of 48 tokens, then a tail from token 100: tiles [0,48) [48,96) [96,100) | [100,164) ...
    keys = ort.reference_tile_keys(200, 100, group_tokens=48)
    bounds = [0] + [j for j in range(1, 200) if keys[j] != keys[j - 1]]
    assert bounds == [0, 48, 96, 100, 164]
    assert bool((keys[1:] >= keys[:-1]).all())
    # a row sitting 40 tokens into the batched numbering: its first chunk ends at combined token 64
    keys = ort.reference_tile_keys(150, 130, shift=40, group_tokens=64)
    bounds = [0] + [j for j in range(1, 150) if keys[j] != keys[j - 1]]
    assert bounds == [0, 24, 88, 130]


def test_dense_reference_matches_the_numpy_dense_oracle():
    """The torch dense path the benchmark times on the host cores computes the numpy oracle's dense
    reference (both restate tests/test_streaming_attention.py:20-40 of the reference)."""
    B, Hq, Hkv, D, T, tpb = 2, 14, 2, 64, 300, 64
    q, k, v, valid = _case(5, B, Hq, Hkv, D, 4, tpb, T - 4 * tpb, torch.float16, pad=17)
    out, mass = ort.dense_reference(q, k, v, Hq // Hkv, tpb, valid=valid)
    ref_out, ref_mass = orc.dense_reference(_np(q), _np(k), _np(v), Hq // Hkv, tpb, valid=valid.numpy())
    np.testing.assert_allclose(out.numpy(), ref_out, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(mass.numpy(), ref_mass, rtol=1e-5, atol=1e-7)
