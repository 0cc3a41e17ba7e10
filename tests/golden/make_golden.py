"""Generate the golden parity fixtures from the reference's own kernels.

Run where the reference checkout is available (its root is the only,
required, argument)::

    python tests/golden/make_golden.py /path/to/rust-llm-pager

It imports the reference's ``pager_hf.streaming_attention`` under Triton's
CPU interpreter (``TRITON_INTERPRET=1``, set before triton is imported) and
replays, on the seeded inputs of ``cases.py``, the call sequences the
reference itself makes (tests/test_streaming_attention.py,
pager_hf/paged_model.py:993-1039, pager_hf/batched_decode.py:238-277).  Two
limits of the interpreter are worked around and recorded in each fixture:

* ``softcap > 0`` fails in the interpreter (``tl_libdevice.tanh`` returns
  None, streaming_attention.py:160), so softcap cases use the reference's
  own dense test oracle ``_dense_reference``
  (tests/test_streaming_attention.py:20-40);
* bf16 tensors come back as garbage (numpy has no bf16), so bf16 cases run
  the reference on fp32 tensors holding the bf16 values; the P->bf16
  rounding at streaming_attention.py:178 is therefore not in those vectors.

Outputs go to ``tests/golden/<case>.npz``.

With ``--gpu`` (run on a GPU machine, against an install of the reference such as
``baseline/_ref``), the reference's kernels compile for the GPU instead and run the cases of
``GPU_CASES`` on CUDA tensors in their native dtype -- bf16 as bf16, so the reference's own rounding
of p to bf16 (streaming_attention.py:178, :347, :428) is in the vectors -- writing
``tests/golden/<case>__gpu.npz`` (or to the directory given by ``--out``)::

    python tests/golden/make_golden.py --gpu baseline/_ref [--out DIR] [case ...]

The tests only read the stored fixtures; none of them runs the reference.
"""

from __future__ import annotations

import os
import sys

GPU = "--gpu" in sys.argv
if not GPU:
    os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from cases import (CASES, GPU_CASES, batched_combined_layout, build_batched, build_contiguous,  # noqa: E402
                   group_row_active, input_digest)

DEV = "cuda" if GPU else "cpu"


def _load_reference(ref_root):
    import importlib.util

    # the kernel module alone: the package's __init__ also imports the compiled pager core
    spec = importlib.util.spec_from_file_location("reference_streaming_attention",
                                                  os.path.join(ref_root, "pager_hf", "streaming_attention.py"))
    sa = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(sa)
    sys.path.insert(0, ref_root)
    sys.path.insert(0, os.path.join(ref_root, "tests"))

    try:
        import test_streaming_attention as ref_tests  # noqa: E402  (a checkout has the tests; an install may not)
    except ImportError:
        ref_tests = None
    return sa, ref_tests


def _as_ref_dtype(t, c):
    """The interpreter cannot run bf16: it gets fp32 copies of the bf16 values; the GPU runs bf16."""
    t = t.to(DEV)
    return t.float() if c["dtype"] == "bf16" and not GPU else t


def _note(c):
    if GPU:
        import torch as _t

        return f"reference triton kernels on {_t.cuda.get_device_name(0)}, native {c['dtype']}"
    return "reference triton kernels (interpreter)" + (" on fp32 copies of bf16 data" if c["dtype"] == "bf16" else "")


def _np(t):
    return t.float().cpu().numpy()


def run_steps(sa, ref_tests, name, c):
    q, k, v, valid, active = build_contiguous(c)
    digest = input_digest([q, k, v, valid, active])
    B, Hq, D, T = c["B"], c["Hq"], c["D"], c["T"]
    note = "reference triton kernels (interpreter)"
    if c.get("softcap"):
        out, _ = ref_tests._dense_reference(
            q, k, v, n_rep=Hq // c["Hkv"], tokens_per_block=16, valid=valid, scale=c.get("scale"),
            softcap=c.get("softcap"),
        )
        note = "reference dense test oracle (interpreter cannot run softcap)"
        return dict(out=out.float().numpy(), digest=digest, note=note)
    qr, kr, vr = _as_ref_dtype(q, c), _as_ref_dtype(k, c), _as_ref_dtype(v, c)
    valid, active = valid.to(DEV), active.to(DEV)
    m, l, acc = sa.streaming_attention_state_init(B, Hq, D, DEV)
    g = c["group"]
    for s in range(0, T, g):
        e = min(s + g, T)
        sa.streaming_attention_step(qr, kr[:, :, s:e], vr[:, :, s:e], m, l, acc, valid=valid[:, s:e], active=active,
                                    scale=c.get("scale"), softcap=c.get("softcap"))
    out = sa.streaming_attention_finalize(acc, l, qr.dtype)
    return dict(out=_np(out), m=_np(m), l=_np(l), acc=_np(acc), digest=digest, note=_note(c))


def run_two_pass(sa, ref_tests, name, c):
    q, k, v, valid, active = build_contiguous(c)
    digest = input_digest([q, k, v, valid, active])
    q, k, v = _as_ref_dtype(q, c), _as_ref_dtype(k, c), _as_ref_dtype(v, c)
    valid, active = valid.to(DEV), active.to(DEV)
    B, Hq, D, tpb, nb, tail = c["B"], c["Hq"], c["D"], c["tpb"], c["nb"], c["tail"]
    full = nb * tpb
    gt = c["group_blocks"] * tpb
    act = active if c.get("active") else None
    m, l, _ = sa.streaming_attention_state_init(B, Hq, D, DEV)
    for s in range(0, full, gt):
        e = min(s + gt, full)
        sa.streaming_attention_stats_step(q, k[:, :, s:e], m, l, valid=valid[:, s:e], active=act)
    if tail:
        sa.streaming_attention_stats_step(q, k[:, :, full:], m, l, valid=valid[:, full:])
    acc = torch.zeros(B, Hq, D, dtype=torch.float32, device=DEV)
    block_mass = torch.zeros(B, Hq, max(nb, 1), dtype=torch.float32, device=DEV)
    for s in range(0, full, gt):
        e = min(s + gt, full)
        sa.streaming_attention_accumulate_step(q, k[:, :, s:e], v[:, :, s:e], m, l, acc, block_mass, s // tpb, tpb,
                                               valid=valid[:, s:e], active=act)
    if tail:
        sa.streaming_attention_fold_fixed_step(q, k[:, :, full:], v[:, :, full:], m, l, acc, valid=valid[:, full:])
    out = sa.streaming_attention_finalize(acc, l, q.dtype)
    return dict(out=_np(out), m=_np(m), l=_np(l), acc=_np(acc), block_mass=_np(block_mass[:, :, :nb]), digest=digest,
                note=_note(c))


def run_batched(sa, ref_tests, name, c):
    q, bk, bv, tk, tv = build_batched(c)
    digest = input_digest([q] + bk + bv + tk + tv)
    k, v, valid, pad_blocks, tail_k, tail_v = batched_combined_layout(c, bk, bv, tk, tv)
    q, k, v, tail_k, tail_v = (_as_ref_dtype(t, c) for t in (q, k, v, tail_k, tail_v))
    valid = valid.to(DEV)
    S, Hq, D, tpb = q.shape[0], c["Hq"], c["D"], c["tpb"]
    max_blocks = max(c["nbs"])
    group = c["group_blocks"]
    m, l, acc = sa.streaming_attention_state_init(S, Hq, D, DEV)
    tail_valid = torch.ones(S, tail_k.shape[2], dtype=torch.int32, device=DEV)
    positions = list(range(max_blocks))
    for i in range(0, max_blocks, group):
        n = len(positions[i:i + group])
        sl = slice(i * tpb, (i + n) * tpb)
        sa.streaming_attention_stats_step(q, k[:, :, sl], m, l, valid=valid[:, sl],
                                          active=group_row_active(pad_blocks, i, n).to(DEV))
    sa.streaming_attention_stats_step(q, tail_k, m, l, valid=tail_valid)
    block_mass = torch.zeros(S, Hq, max(max_blocks, 1), dtype=torch.float32, device=DEV)
    for i in range(0, max_blocks, group):
        n = len(positions[i:i + group])
        sl = slice(i * tpb, (i + n) * tpb)
        sa.streaming_attention_accumulate_step(q, k[:, :, sl], v[:, :, sl], m, l, acc, block_mass, i, tpb,
                                               valid=valid[:, sl], active=group_row_active(pad_blocks, i, n).to(DEV))
    sa.streaming_attention_fold_fixed_step(q, tail_k, tail_v, m, l, acc, valid=tail_valid)
    out = sa.streaming_attention_finalize(acc, l, q.dtype)
    per_row = block_mass.mean(dim=1).cpu()  # batched_decode.py:273
    session_mass = np.zeros((S, max(max_blocks, 1)), dtype=np.float32)
    for row, nb in enumerate(c["nbs"]):
        session_mass[row, :nb] = per_row[row, pad_blocks[row]:pad_blocks[row] + nb].numpy()
    return dict(out=_np(out), m=_np(m), l=_np(l), acc=_np(acc), session_mass=session_mass, digest=digest,
                note=_note(c))


def main():
    args = [a for a in sys.argv[1:] if a != "--gpu"]
    out_dir = HERE
    if "--out" in args:
        i = args.index("--out")
        out_dir = args[i + 1]
        del args[i:i + 2]
    if not args:
        sys.exit("usage: python tests/golden/make_golden.py [--gpu] [--out DIR] /path/to/rust-llm-pager [case ...]")
    ref_root = args[0]
    only = set(args[1:])
    unknown = only - set(CASES)
    if unknown:
        sys.exit(f"unknown cases: {sorted(unknown)}")
    sa, ref_tests = _load_reference(ref_root)
    runners = {"steps": run_steps, "two_pass": run_two_pass, "batched": run_batched}
    os.makedirs(out_dir, exist_ok=True)
    for name, c in CASES.items():
        if only and name not in only:
            continue
        if (GPU and name not in GPU_CASES) or (not GPU and c.get("gpu_only")):
            continue
        res = runners[c["kind"]](sa, ref_tests, name, c)
        fname = f"{name}__gpu.npz" if GPU else f"{name}.npz"
        np.savez_compressed(os.path.join(out_dir, fname), **res)
        print(f"{fname}: {sorted(res)}")


if __name__ == "__main__":
    main()
