"""GPU parity of the drop-in streaming-attention functions (the C-ABI CUDA path).

Every golden case (tests/golden/, produced by the reference's own kernels) is
replayed through ``pager_hf.streaming_attention`` on the GPU and compared with
the reference's outputs:

* attention output: max-abs 2e-3 for fp16 / fp32 inputs (fp32 accumulate),
  5e-3 for bf16 (whose fixtures come from the reference run on fp32 copies,
  i.e. without its own P->bf16 rounding);
* per-block attention mass: 1e-4 relative (atol 1e-6 for near-zero masses);
* the online-softmax state (m, l) to fp32 rounding of the scores.

The ``<case>__gpu`` fixtures come from the reference's kernels compiled for a B200 and run in the
cases' native dtype (bf16 as bf16, with the reference's own rounding of p to bf16); against those the
rounded outputs must agree within 2e-3 or one output ulp, with at most 1 % of them different (both
backends round p as the reference does; what remains is fp32 association).

Both compute backends (tensor-core mma and CUDA-core fma) are checked.  The
reference's own test file (tests/test_streaming_attention.py) is mirrored by
the ``ref_*`` cases plus the must-differ checks below.
"""

import os

import numpy as np
import pytest
import torch

import golden_io as gio
from cases import CASES, GPU_CASES, build_contiguous
from replay import run_case

pytestmark = pytest.mark.gpu

OUT_ATOL = {"f16": 2e-3, "f32": 2e-3, "bf16": 5e-3}
MASS = dict(rtol=1e-4, atol=1e-6)


@pytest.fixture(scope="module")
def sa():
    from pager_hf import streaming_attention

    return streaming_attention


@pytest.fixture(params=["auto", "fma"])
def backend(request, sa):
    sa.set_backend(request.param)
    yield request.param
    sa.set_backend("auto")


@pytest.mark.parametrize("name", [n for n, c in CASES.items() if not c.get("gpu_only")])
def test_golden_case(sa, backend, name):
    c = CASES[name]
    g = gio.load(name)
    res = run_case(sa, name)
    atol = OUT_ATOL[c["dtype"]]
    np.testing.assert_allclose(res["out"].numpy(), g["out"], rtol=0, atol=atol)
    if "m" in g:
        np.testing.assert_allclose(res["m"].numpy(), g["m"], rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(res["l"].numpy(), g["l"], rtol=2e-4, atol=1e-6)
    if "block_mass" in g:
        np.testing.assert_allclose(res["block_mass"].numpy(), g["block_mass"], **MASS)
    if "session_mass" in g:
        np.testing.assert_allclose(res["session_mass"].numpy(), g["session_mass"], **MASS)


@pytest.mark.parametrize("name", GPU_CASES)
def test_golden_case_from_the_reference_on_a_gpu(sa, backend, name):
    if not os.path.exists(os.path.join(gio.GOLDEN_DIR, f"{name}__gpu.npz")):
        pytest.skip("fixture from the reference's kernels on a GPU not generated (make_golden.py --gpu)")
    c = CASES[name]
    g = gio.load(f"{name}__gpu")
    res = run_case(sa, name)
    out, ref = res["out"].numpy(), g["out"]
    eps = {"bf16": 2.0 ** -7, "f16": 2.0 ** -10, "f32": 2.0 ** -23}[c["dtype"]]
    worst = float((np.abs(out - ref) / np.maximum(2e-3, eps * np.abs(ref))).max())
    differ = float((out != ref).mean())
    print(f"{name} [{backend}]: {differ:.4f} of the rounded outputs differ; worst {worst:.2f} x max(2e-3, 1 ulp)")
    assert worst <= 1.0
    assert differ <= 0.01
    np.testing.assert_allclose(res["m"].numpy(), g["m"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(res["l"].numpy(), g["l"], rtol=2e-4, atol=1e-6)
    if "block_mass" in g:
        np.testing.assert_allclose(res["block_mass"].numpy(), g["block_mass"], **MASS)
    if "session_mass" in g:
        np.testing.assert_allclose(res["session_mass"].numpy(), g["session_mass"], **MASS)


def test_padding_mask_changes_result(sa):
    """tests/test_streaming_attention.py:170-171: masked != unmasked."""
    masked = run_case(sa, "ref_padding_mask")["out"]
    q, k, v, valid, active = (t.cuda() for t in build_contiguous("ref_padding_mask"))
    m, l, acc = sa.streaming_attention_state_init(1, 14, 64, "cuda")
    sa.streaming_attention_step(q, k, v, m, l, acc)
    unmasked = sa.streaming_attention_finalize(acc, l, q.dtype).float().cpu()
    assert not torch.allclose(masked, unmasked, rtol=2e-2, atol=2e-2)


def test_softcap_changes_result(sa):
    """tests/test_streaming_attention.py:270-272."""
    capped = run_case(sa, "ref_softcap")["out"]
    q, k, v, _, _ = (t.cuda() for t in build_contiguous("ref_softcap"))
    m, l, acc = sa.streaming_attention_state_init(1, 14, 64, "cuda")
    sa.streaming_attention_step(q, k, v, m, l, acc)
    plain = sa.streaming_attention_finalize(acc, l, q.dtype).float().cpu()
    assert not torch.allclose(capped, plain, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("fn", ["step", "stats", "accumulate"])
def test_active_zero_is_bit_exact_noop(sa, fn):
    """tests/test_streaming_attention.py:174-240: an inactive row's state is untouched, bit for bit."""
    torch.manual_seed(4)
    q = torch.randn(2, 14, 64, dtype=torch.float16, device="cuda")
    k = torch.randn(2, 2, 32, 64, dtype=torch.float16, device="cuda")
    v = torch.randn(2, 2, 32, 64, dtype=torch.float16, device="cuda")
    valid = torch.ones(2, 32, dtype=torch.int32, device="cuda")
    active = torch.tensor([0, 1], dtype=torch.int32, device="cuda")
    m, l, acc = sa.streaming_attention_state_init(2, 14, 64, "cuda")
    # a non-trivial prior state for the inactive row
    sa.streaming_attention_step(q, k, v, m, l, acc)
    m0, l0, acc0 = m.clone(), l.clone(), acc.clone()
    if fn == "step":
        sa.streaming_attention_step(q, k, v, m, l, acc, valid=valid, active=active)
        assert torch.equal(acc[0], acc0[0])
    elif fn == "stats":
        sa.streaming_attention_stats_step(q, k, m, l, valid=valid, active=active)
    else:
        bm = torch.zeros(2, 14, 2, device="cuda")
        sa.streaming_attention_accumulate_step(q, k, v, m, l, acc, bm, 0, 16, valid=valid, active=active)
        assert torch.equal(acc[0], acc0[0])
        assert torch.equal(bm[0], torch.zeros_like(bm[0]))
        assert bm[1].sum() > 0
    assert torch.equal(m[0], m0[0])
    assert torch.equal(l[0], l0[0])


def test_empty_chunk_is_noop(sa):
    q = torch.randn(1, 8, 64, dtype=torch.float16, device="cuda")
    k = torch.zeros(1, 2, 0, 64, dtype=torch.float16, device="cuda")
    m, l, acc = sa.streaming_attention_state_init(1, 8, 64, "cuda")
    sa.streaming_attention_step(q, k, k, m, l, acc)
    assert torch.isinf(m).all() and (l == 0).all() and (acc == 0).all()


def test_n_rep_guard_matches_reference(sa):
    q = torch.randn(1, 34, 64, dtype=torch.float16, device="cuda")
    k = torch.randn(1, 2, 16, 64, dtype=torch.float16, device="cuda")
    m, l, acc = sa.streaming_attention_state_init(1, 34, 64, "cuda")
    with pytest.raises(NotImplementedError):
        sa.streaming_attention_step(q, k, k, m, l, acc)
