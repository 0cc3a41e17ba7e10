"""Host-side logic of ``bench.py``: workload placement and byte accounting, the config both arms
print, and the one-JSON-line stdout under torchrun."""

import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_cfg5_layout_respects_the_hbm_budget_and_counts_every_token_once():
    lay = bench.WorkloadLayout("cfg5-32k", seed=1234)
    w = bench.WORKLOADS["cfg5-32k"]
    assert lay.dev_slots * lay.slot_bytes <= w["hbm_budget_gb"] * 1e9
    assert lay.dev_slots + lay.host_slots == lay.B * lay.nb
    # no window: every block token is attended, on one tier or the other
    assert lay.dev_tokens + lay.host_tokens == lay.B * lay.nb * lay.tpb
    kv_tok = 2 * lay.Hkv * lay.D * 2
    assert lay.host_bytes == lay.L * lay.host_tokens * kv_tok
    # recent_only: each row's device blocks are its newest ones
    for b in range(lay.B):
        row = lay.table[b]
        on_dev = [(int(e) & 0x40000000) == 0 for e in row]
        first_dev = on_dev.index(True)
        assert all(on_dev[first_dev:]) and not any(on_dev[:first_dev])


def test_window_counts_only_tokens_inside_the_window():
    lay = bench.WorkloadLayout("cfg4-32k-window", seed=1234)
    window = bench.WORKLOADS["cfg4-32k-window"]["window"]
    # per row, the attended block tokens are the last `window` tokens minus the tail
    per_row = [min(window, lay.nb * lay.tpb + t) - t for t in lay.tails]
    assert lay.dev_tokens + lay.host_tokens == sum(per_row)
    assert all(lo == lay.nb * lay.tpb + t - window for lo, t in zip(lay.lo, lay.tails))


def test_both_arms_report_the_same_config():
    """The config is the workload's alone (the host-tier read mode is a key of its own), so the GPU
    arm and the CPU reference arm report identical configs."""
    cfg = bench.WorkloadLayout("cfg5-32k", seed=1234).config(2)
    assert cfg["global_batch"] == 2 * cfg["batch_per_gpu"]
    for key in ("workload", "model", "context", "hbm_bytes_per_step", "host_bytes_per_step", "l2", "parallelism"):
        assert key in cfg
    assert "host_read" not in cfg
    assert cfg == bench.WorkloadLayout("cfg5-32k", seed=1234).config(2)


def test_cpu_torch_arm_times_the_reference_dense_path(monkeypatch):
    """The CPU baseline runs the reference's dense torch path on one (request, layer) unit with every
    host thread, and reports the attended KV bytes of each call."""
    monkeypatch.setitem(bench.WORKLOADS, "tiny", dict(model="tiny", layers=2, hq=8, hkv=2, d=64, dtype="bf16",
                                                     tpb=64, batch=2, context=1024, hbm_budget_gb=1.0, window=None))
    arm = bench.CpuTorchArm("tiny", threads=2, reps=3)
    b, t = arm.sample()
    assert b == 3 * (1024 + 32) * 2 * 2 * 64 * 2 and t > 0
    assert "torch.set_num_threads(2)" in bench.sample_desc(arm)


def test_json_line_is_alone_on_stdout_under_torchrun():
    code = (
        "import os, sys; sys.path.insert(0, %r); import bench\n"
        "out = bench._json_stdout(2)\n"
        "os.write(1, b'NCCL version banner\\n'); print('library noise')\n"
        "print('{\"metric\": 1}', file=out, flush=True)\n" % ROOT)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)
    assert r.stdout == '{"metric": 1}\n'
    assert "NCCL version banner" in r.stderr and "library noise" in r.stderr


@pytest.mark.parametrize("name", sorted(bench.WORKLOADS))
def test_every_workload_lays_out(name):
    lay = bench.WorkloadLayout(name, seed=7)
    assert lay.bytes_per_step == lay.hbm_bytes + lay.host_bytes > 0
    assert lay.launches_per_step == 2 * lay.L


def test_reference_gpu_arm_reports_unavailable_without_the_install(tmp_path, monkeypatch, capsys):
    """Without the reference installed under baseline/_ref, the GPU comparison arm prints one
    ``unavailable`` line and succeeds, leaving the import path alone."""
    import argparse
    import json

    monkeypatch.setattr(bench, "REF_INSTALL", str(tmp_path / "missing"))
    before = list(sys.path)
    args = argparse.Namespace(workload="hbm-32k", steps=1, warmup=1, gpus=1)
    assert bench.run_reference_gpu_arm(args) == 0
    line = json.loads(capsys.readouterr().out.strip())
    assert line["impl"] == "reference-gpu" and "baseline/_ref" in line["unavailable"]
    assert sys.path == before


def test_reference_arms_do_no_work_on_ranks_other_than_zero(monkeypatch, capsys):
    """Under torchrun only rank 0 runs and prints the reference arms; the other ranks exit 0 at once."""
    import argparse

    monkeypatch.setenv("WORLD_SIZE", "2")
    monkeypatch.setenv("RANK", "1")
    monkeypatch.setenv("LOCAL_RANK", "1")
    monkeypatch.setattr(bench, "CpuOracleArm", lambda *a, **k: pytest.fail("rank 1 started the CPU arm"))
    monkeypatch.setattr(bench, "CpuTorchArm", lambda *a, **k: pytest.fail("rank 1 started the CPU arm"))
    args = argparse.Namespace(workload="cfg5-32k", gpus=2, steps=3, warmup=3, cpu_arm="torch")
    assert bench.run_reference_arm(args) == 0
    assert bench.run_reference_gpu_arm(args) == 0
    assert capsys.readouterr().out == ""
