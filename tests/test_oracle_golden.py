"""Pin the CPU oracle against vectors produced by the reference's own kernels.

The fixtures under tests/golden/ were produced by tests/golden/make_golden.py,
which replays the reference's call sequences through its Triton kernels on the
CPU (interpreter).  The oracle (numpy restatement) must reproduce them to fp32
rounding.  The ``<case>__gpu`` fixtures were produced by the same script with
``--gpu``: the reference's kernels compiled for a B200 and run in the cases'
native dtype, so their bf16 vectors carry the reference's own rounding of p to
bf16; there the oracle must agree except where fp32 association moves a value
across a rounding boundary (within 2e-3 or one output ulp, at most 6 % of the
rounded outputs).
"""

import os

import numpy as np
import pytest

import golden_io as gio
from cases import (CASES, GPU_CASES, batched_combined_layout, build_batched, build_contiguous, group_row_active,
                   input_digest)
from oracle import streaming_attention_oracle as orc

TOL = dict(rtol=2e-5, atol=2e-6)


def _vdt(c):
    # bf16 fixtures ran the reference on fp32 copies, so P is not rounded to bf16 there
    return "f32" if c["dtype"] == "bf16" else c["dtype"]


def _run_steps(c, q, k, v, valid, active):
    B, Hq, D, T = c["B"], c["Hq"], c["D"], c["T"]
    m, l, acc = orc.state_init(B, Hq, D)
    g = c["group"]
    for s in range(0, T, g):
        e = min(s + g, T)
        orc.step(q, k[:, :, s:e], v[:, :, s:e], m, l, acc, valid=valid[:, s:e], active=active,
                 scale=c.get("scale"), softcap=c.get("softcap"), v_dtype=_vdt(c))
    return m, l, acc


def _run_two_pass(c, q, k, v, valid, active):
    B, Hq, D, tpb, nb, tail = c["B"], c["Hq"], c["D"], c["tpb"], c["nb"], c["tail"]
    full, gt = nb * tpb, c["group_blocks"] * tpb
    act = active if c.get("active") else None
    m, l, acc = orc.state_init(B, Hq, D)
    for s in range(0, full, gt):
        e = min(s + gt, full)
        orc.stats_step(q, k[:, :, s:e], m, l, valid=valid[:, s:e], active=act)
    if tail:
        orc.stats_step(q, k[:, :, full:], m, l, valid=valid[:, full:])
    bm = np.zeros((B, Hq, max(nb, 1)), np.float32)
    for s in range(0, full, gt):
        e = min(s + gt, full)
        orc.accumulate_step(q, k[:, :, s:e], v[:, :, s:e], m, l, acc, bm, s // tpb, tpb, valid=valid[:, s:e],
                            active=act, v_dtype=_vdt(c))
    if tail:
        orc.fold_fixed_step(q, k[:, :, full:], v[:, :, full:], m, l, acc, valid=valid[:, full:], v_dtype=_vdt(c))
    return m, l, acc, bm[:, :, :nb]


@pytest.mark.parametrize("name", [n for n, c in CASES.items() if c["kind"] in ("steps", "two_pass")
                                  and not c.get("gpu_only")])
def test_oracle_matches_reference_golden(name):
    c = CASES[name]
    g = gio.load(name)
    q, k, v, valid, active = build_contiguous(c)
    assert input_digest([q, k, v, valid, active]) == str(g["digest"]), "seeded input generator drifted"
    qn, kn, vn = gio.np32(q), gio.np32(k), gio.np32(v)
    validn, activen = valid.numpy(), active.numpy()
    if c.get("softcap"):
        out, _ = orc.dense_reference(qn, kn, vn, c["Hq"] // c["Hkv"], 16, valid=validn, scale=c["scale"],
                                     softcap=c["softcap"])
        np.testing.assert_allclose(orc.round_to(out, c["dtype"]), g["out"], rtol=1e-3, atol=1e-3)
        # and the online restatement agrees with the dense one on softcap
        m, l, acc = _run_steps(c, qn, kn, vn, validn, activen)
        np.testing.assert_allclose(orc.finalize(acc, l, c["dtype"]), g["out"], rtol=2e-3, atol=2e-3)
        return
    if c["kind"] == "steps":
        m, l, acc = _run_steps(c, qn, kn, vn, validn, activen)
    else:
        m, l, acc, bm = _run_two_pass(c, qn, kn, vn, validn, activen)
        np.testing.assert_allclose(bm, g["block_mass"], **TOL)
    np.testing.assert_allclose(m, g["m"], **TOL)
    np.testing.assert_allclose(l, g["l"], **TOL)
    # acc is unnormalised; single P->f16 rounding flips (one ulp of a 2^-11-relative cast) are expected
    np.testing.assert_allclose(acc, g["acc"], rtol=1e-4, atol=2e-3)
    out_dt = "f32" if c["dtype"] == "bf16" else c["dtype"]
    np.testing.assert_allclose(orc.finalize(acc, l, out_dt), g["out"], rtol=1e-3, atol=2e-4)


def _run_batched(c, g, vdt):
    q, bk, bv, tk, tv = build_batched(c)
    assert input_digest([q] + bk + bv + tk + tv) == str(g["digest"])
    k, v, valid, pad_blocks, tail_k, tail_v = batched_combined_layout(c, bk, bv, tk, tv)
    qn, kn, vn, tkn, tvn = map(gio.np32, (q, k, v, tail_k, tail_v))
    S, Hq, D, tpb, group = qn.shape[0], c["Hq"], c["D"], c["tpb"], c["group_blocks"]
    max_blocks = max(c["nbs"])
    m, l, acc = orc.state_init(S, Hq, D)
    validn = valid.numpy()
    for i in range(0, max_blocks, group):
        n = min(group, max_blocks - i)
        sl = slice(i * tpb, (i + n) * tpb)
        orc.stats_step(qn, kn[:, :, sl], m, l, valid=validn[:, sl], active=group_row_active(pad_blocks, i, n).numpy())
    orc.stats_step(qn, tkn, m, l)
    bm = np.zeros((S, Hq, max_blocks), np.float32)
    for i in range(0, max_blocks, group):
        n = min(group, max_blocks - i)
        sl = slice(i * tpb, (i + n) * tpb)
        orc.accumulate_step(qn, kn[:, :, sl], vn[:, :, sl], m, l, acc, bm, i, tpb, valid=validn[:, sl],
                            active=group_row_active(pad_blocks, i, n).numpy(), v_dtype=vdt)
    orc.fold_fixed_step(qn, tkn, tvn, m, l, acc, v_dtype=vdt)
    return m, l, acc, bm, pad_blocks


def test_oracle_matches_batched_sessions_golden():
    name = "batched_sessions_f16"
    c = CASES[name]
    g = gio.load(name)
    m, l, acc, bm, pad_blocks = _run_batched(c, g, "f16")
    np.testing.assert_allclose(m, g["m"], **TOL)
    np.testing.assert_allclose(l, g["l"], **TOL)
    np.testing.assert_allclose(acc, g["acc"], rtol=1e-4, atol=2e-3)
    np.testing.assert_allclose(orc.finalize(acc, l, "f16"), g["out"], rtol=1e-3, atol=1e-3)
    per_row = bm.mean(axis=1)
    for row, nb in enumerate(c["nbs"]):
        np.testing.assert_allclose(per_row[row, pad_blocks[row]:pad_blocks[row] + nb], g["session_mass"][row, :nb],
                                   **TOL)


def test_oracle_two_pass_equals_one_pass_and_dense():
    """Size-independent identities the oracle must satisfy: two-pass == one-pass == dense softmax."""
    rng = np.random.default_rng(3)
    q = rng.standard_normal((2, 8, 32)).astype(np.float32)
    k = rng.standard_normal((2, 2, 300, 32)).astype(np.float32)
    v = rng.standard_normal((2, 2, 300, 32)).astype(np.float32)
    m, l, acc = orc.state_init(2, 8, 32)
    orc.step(q, k, v, m, l, acc)
    out1 = orc.finalize(acc, l, "f32")
    out2, mass2, _, _ = orc.two_pass_decode(q, k[:, :, :256], v[:, :, :256], k[:, :, 256:], v[:, :, 256:],
                                            num_blocks=16, tokens_per_block=16, group_size_blocks=5)
    dense, dmass = orc.dense_reference(q, k, v, 4, 16)
    np.testing.assert_allclose(out1, dense, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(out2, dense, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(mass2, dmass[:, :, :16], rtol=1e-4, atol=1e-6)


def test_oracle_n_rep_guard():
    with pytest.raises(NotImplementedError):
        orc.validate_n_rep(17)


def test_dense_gqa_cpu_path_equals_two_pass():
    """The CPU timing path (dense, GQA-grouped) computes what the two-pass reference sequence computes."""
    rng = np.random.default_rng(9)
    q = rng.standard_normal((1, 8, 32)).astype(np.float32)
    k = rng.standard_normal((1, 2, 128, 32)).astype(np.float32)
    v = rng.standard_normal((1, 2, 128, 32)).astype(np.float32)
    tk = rng.standard_normal((1, 2, 5, 32)).astype(np.float32)
    tv = rng.standard_normal((1, 2, 5, 32)).astype(np.float32)
    valid = np.ones((1, 128), np.int32)
    valid[:, :20] = 0
    out, mass = orc.dense_decode_gqa(q, k, v, tk, tv, 16, valid=valid)
    out2, mass2, _, _ = orc.two_pass_decode(q, k, v, tk, tv, 8, 16, 8, valid=valid)
    np.testing.assert_allclose(out, out2, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(mass, mass2, rtol=1e-4, atol=1e-7)


def _agree_rounded(out, ref, dtype, what):
    """Within 2e-3, or one ulp of the output dtype where that is larger; at most 6 % of the rounded
    outputs different."""
    eps = {"bf16": 2.0 ** -7, "f16": 2.0 ** -10, "f32": 2.0 ** -23}[dtype]
    tol = np.maximum(2e-3, eps * np.abs(ref))
    worst = float((np.abs(out - ref) / tol).max())
    assert worst <= 1.0, f"{what}: {worst:.2f} x max(2e-3, 1 ulp)"
    differ = float((out != ref).mean())
    assert differ <= 0.06, f"{what}: {differ:.3f} of the rounded outputs differ"


@pytest.mark.parametrize("name", GPU_CASES)
def test_oracle_matches_the_reference_kernels_run_on_a_gpu(name):
    path = os.path.join(gio.GOLDEN_DIR, f"{name}__gpu.npz")
    if not os.path.exists(path):
        pytest.skip("fixture from the reference's kernels on a GPU not generated (make_golden.py --gpu)")
    c = CASES[name]
    g = gio.load(f"{name}__gpu")
    dt = c["dtype"]
    if c["kind"] == "batched":
        m, l, acc, bm, pad_blocks = _run_batched(c, g, dt)
        per_row = bm.mean(axis=1)
        for row, nb in enumerate(c["nbs"]):
            np.testing.assert_allclose(per_row[row, pad_blocks[row]:pad_blocks[row] + nb],
                                       g["session_mass"][row, :nb], rtol=1e-4, atol=1e-7)
    else:
        q, k, v, valid, active = build_contiguous(c)
        assert input_digest([q, k, v, valid, active]) == str(g["digest"]), "seeded input generator drifted"
        qn, kn, vn = gio.np32(q), gio.np32(k), gio.np32(v)
        if c["kind"] == "steps":
            m, l, acc = _run_native_steps(c, qn, kn, vn, valid.numpy(), active.numpy())
        else:
            m, l, acc, bm = _run_native_two_pass(c, qn, kn, vn, valid.numpy(), active.numpy())
            np.testing.assert_allclose(bm, g["block_mass"], rtol=1e-4, atol=1e-7)
    np.testing.assert_allclose(m, g["m"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(l, g["l"], rtol=1e-5)
    _agree_rounded(orc.finalize(acc, l, dt), g["out"], dt, name)


def _run_native_steps(c, q, k, v, valid, active):
    B, Hq, D, T = c["B"], c["Hq"], c["D"], c["T"]
    m, l, acc = orc.state_init(B, Hq, D)
    for s in range(0, T, c["group"]):
        e = min(s + c["group"], T)
        orc.step(q, k[:, :, s:e], v[:, :, s:e], m, l, acc, valid=valid[:, s:e], active=active, v_dtype=c["dtype"])
    return m, l, acc


def _run_native_two_pass(c, q, k, v, valid, active):
    B, Hq, D, tpb, nb, tail = c["B"], c["Hq"], c["D"], c["tpb"], c["nb"], c["tail"]
    full, gt = nb * tpb, c["group_blocks"] * tpb
    m, l, acc = orc.state_init(B, Hq, D)
    for s in range(0, full, gt):
        orc.stats_step(q, k[:, :, s:min(s + gt, full)], m, l, valid=valid[:, s:min(s + gt, full)])
    if tail:
        orc.stats_step(q, k[:, :, full:], m, l, valid=valid[:, full:])
    bm = np.zeros((B, Hq, max(nb, 1)), np.float32)
    for s in range(0, full, gt):
        e = min(s + gt, full)
        orc.accumulate_step(q, k[:, :, s:e], v[:, :, s:e], m, l, acc, bm, s // tpb, tpb, valid=valid[:, s:e],
                            v_dtype=c["dtype"])
    if tail:
        orc.fold_fixed_step(q, k[:, :, full:], v[:, :, full:], m, l, acc, valid=valid[:, full:], v_dtype=c["dtype"])
    return m, l, acc, bm[:, :, :nb]
