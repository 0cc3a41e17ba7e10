#!/usr/bin/env python
"""Decode-attention benchmark: effective KV GB/s against the HBM + host-link roofline.

One *step* is one decode step of attention over every layer of a model for a
batch of requests at long context: per layer, one fused paged decode-attention
call (split-KV kernel, then one combine/mass kernel) walks each request's block table over
the device KV pool (HBM) and the pinned host pool (read zero-copy over the
host link), plus its tail, and writes the attention output and the per-block
attention mass the heavy-hitter policies consume.

Default workload ("cfg5-32k"): the Llama-3-8B attention geometry of the
reference's serving config (32 layers, 32 query / 8 KV heads, head_dim 128,
bf16, 64-token blocks) with 12 concurrent requests at a 32,768-token context
per GPU and a 40 GB per-GPU HBM KV budget; the most recent blocks of each
request stay in HBM (recent_only placement) and the rest sit in the pinned
host pool.  KV values are seeded synthetic data (no checkpoints offline).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]
                    [--rounding running|final|one_pass] [--no-extras]

N > 1 runs one process per GPU (torchrun); requests are sharded across GPUs
(weak scaling, no collective on the data path); the timed region is bracketed
by barriers and its time is the max over ranks.

``--rounding``: how p is rounded before P.V.  "running" (default) rounds exactly
as the reference's one-pass path does for this workload's recent_only placement
(a K pass, a scan and a V pass); "one_pass" is the fused one-pass kernel.  At
N = 1 the line also carries, unless ``--no-extras``: the HBM-resident ``hbm-32k``
workload timed on its own (``kernel_hbm_32k``, against the measured HBM peak)
and model-level decode tokens/s of ``PagedModel.generate`` on BASELINE config 4
at 32k (``model_decode``).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "rust-llm-pager_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "decode-attn effective KV GB/s (HBM + host tiers) at 32k ctx"
# DRAM bytes (read + written) per algorithmic K/V byte of one layer's kernels, from ncu captures
# with caches left warm between kernels (--cache-control none) on prof-b8, one layer of hbm-32k
# (the prof-b8 traffic summary under profiles/): the one-pass kernel + combine/mass, 1051.87 MB read +
# 4.94 MB written; the reference-rounding passes (scores, reference-max scan, values,
# combine/mass), 1070.60 MB + 14.74 MB, the scores mostly staying in L2 between the passes.
# Algorithmic bytes per layer: 1073.74 MB.
NCU_DRAM_PER_HBM_BYTE = {"one_pass": (1051.87 + 4.94) / 1073.74, "exact": (1070.60 + 14.74) / 1073.74}

WORKLOADS = {
    # the serving config's Llama-3-8B geometry at 32k: 40 GB HBM budget, overflow in the pinned host pool
    "cfg5-32k": dict(model="Llama-3-8B attention (L32, Hq32, Hkv8, D128)", layers=32, hq=32, hkv=8, d=128,
                     dtype="bf16", tpb=64, batch=12, context=32768, hbm_budget_gb=40.0, window=None),
    # same geometry, everything resident in HBM (8 x 4 GiB < 40 GB)
    "hbm-32k": dict(model="Llama-3-8B attention (L32, Hq32, Hkv8, D128)", layers=32, hq=32, hkv=8, d=128,
                    dtype="bf16", tpb=64, batch=8, context=32768, hbm_budget_gb=40.0, window=None),
    # small HBM-only case for ncu captures (two requests, four layers: 1 GB of KV, 268 MB per launch > L2)
    "prof-hbm": dict(model="Llama-3-8B attention (L4 slice, Hq32, Hkv8, D128)", layers=4, hq=32, hkv=8, d=128,
                     dtype="bf16", tpb=64, batch=2, context=32768, hbm_budget_gb=40.0, window=None),
    # one layer of hbm-32k for ncu captures: the same launch (8 rows x 32k, 256 CTAs of 128 tiles each),
    # 1.07 GB of KV on the device
    "prof-b8": dict(model="Llama-3-8B attention (L1 slice, Hq32, Hkv8, D128)", layers=1, hq=32, hkv=8, d=128,
                    dtype="bf16", tpb=64, batch=8, context=32768, hbm_budget_gb=40.0, window=None),
    # BASELINE config 3's attention geometry (TinyLlama: 8 query heads per KV head, head_dim 64, fp16),
    # 16 rows x 16k, all in HBM: the kernel-bound case of the n_rep-8 values pass
    "cfg3-hbm-16k": dict(model="TinyLlama-1.1B attention (L22, Hq32, Hkv4, D64)", layers=22, hq=32, hkv=4, d=64,
                         dtype="f16", tpb=64, batch=16, context=16384, hbm_budget_gb=40.0, window=None),
    # small tiered case for ncu captures: two requests, four layers, 20% of each row's blocks in HBM, the
    # rest in the host pool (staged per layer by the copy engines when the link favours it)
    "prof-tiered": dict(model="Llama-3-8B attention (L4 slice, Hq32, Hkv8, D128)", layers=4, hq=32, hkv=8, d=128,
                        dtype="bf16", tpb=64, batch=2, context=32768, resident_frac=0.2, sinks=0, window=None),
    # the sliding-window config: Mistral-7B, B8 x 32k, window 4096, 5% resident (sinks + recent)
    "cfg4-32k-window": dict(model="Mistral-7B attention (L32, Hq32, Hkv8, D128, window 4096)", layers=32, hq=32,
                            hkv=8, d=128, dtype="bf16", tpb=64, batch=8, context=32768, resident_frac=0.05,
                            sinks=4, window=4096),
}


# ----------------------------------------------------------------------------- helpers
def _json_stdout(world: int):
    """Where the one JSON line goes.  Under torchrun, native libraries (NCCL's version banner) write to
    file descriptor 1 too; that descriptor is pointed at stderr and the JSON line goes to a saved copy
    of the original stdout, so stdout carries exactly one line."""
    if world <= 1:
        return sys.stdout
    sys.stdout.flush()
    saved = os.dup(1)
    os.dup2(2, 1)
    return os.fdopen(saved, "w", buffering=1)


def _dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        import torch

        p = torch.cuda.get_device_properties(device)
        self.gpu = f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json)"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback 6.65 TB/s"


# ----------------------------------------------------------------------------- workload
class WorkloadLayout:
    """Placement and byte accounting of one GPU's share (CPU only): tails, which blocks of each row
    live in HBM or in the host pool, the block table, the attended range, the bytes per step.
    Shared by the GPU workload and by the reference arm, which reports the same configuration."""

    def __init__(self, name: str, seed: int):
        import torch

        w = WORKLOADS[name]
        self.name, self.w = name, w
        self.L, self.Hq, self.Hkv, self.D, self.tpb = w["layers"], w["hq"], w["hkv"], w["d"], w["tpb"]
        self.B, self.ctx = w["batch"], w["context"]
        elt = 2
        nb = self.ctx // self.tpb
        self.nb = nb
        self.slot_bytes = self.L * 2 * self.Hkv * self.tpb * self.D * elt
        g = torch.Generator(device="cpu").manual_seed(seed)
        self.tails = torch.randint(1, self.tpb + 1, (self.B,), generator=g).tolist()
        resident = []  # per row: block indices that live in HBM
        if "hbm_budget_gb" in w:
            per_row = min(nb, int(w["hbm_budget_gb"] * 1e9 // self.slot_bytes) // self.B)
            for _ in range(self.B):
                resident.append(set(range(nb - per_row, nb)))  # recent_only: newest blocks
        else:
            per_row = max(1, int(math.ceil(w["resident_frac"] * nb)))
            sinks = min(w.get("sinks", 0), per_row)
            for _ in range(self.B):
                resident.append(set(range(sinks)) | set(range(nb - (per_row - sinks), nb)))
        self.dev_slots = sum(len(r) for r in resident)
        self.host_slots = self.B * nb - self.dev_slots
        host_bit = 0x40000000
        table = torch.full((self.B, nb), -1, dtype=torch.int32)
        d_next = h_next = 0
        self.dev_tokens = self.host_tokens = 0
        window = w.get("window")
        self.window = window
        self.lo = []
        for b in range(self.B):
            ntok = nb * self.tpb + self.tails[b]
            row_lo = max(0, ntok - window) if window else 0
            self.lo.append(row_lo)
            for j in range(nb):
                on_dev = j in resident[b]
                if on_dev:
                    table[b, j] = d_next
                    d_next += 1
                else:
                    table[b, j] = h_next | host_bit
                    h_next += 1
                # tokens of this block that the window keeps (all of them without a window)
                t0, t1 = j * self.tpb, (j + 1) * self.tpb
                n_valid = max(0, t1 - max(t0, row_lo))
                if on_dev:
                    self.dev_tokens += n_valid
                else:
                    self.host_tokens += n_valid
        self.table = table
        self.tail_tokens = sum(self.tails)
        # algorithmic bytes per step (only attended tokens are counted)
        kv_tok = 2 * self.Hkv * self.D * elt
        qo = 2 * self.B * self.Hq * self.D * elt
        mass_b = self.B * nb * 4 * 2  # read-modify-write of the mass accumulator
        self.hbm_bytes = self.L * ((self.dev_tokens + self.tail_tokens) * kv_tok + qo + mass_b)
        self.host_bytes = self.L * self.host_tokens * kv_tok
        self.bytes_per_step = self.hbm_bytes + self.host_bytes
        self.launches_per_step = self.L * 2  # split kernel + combine/mass kernel per layer

    def config(self, world: int) -> dict:
        w = self.w
        return {
            "workload": self.name, "model": w["model"], "batch_per_gpu": self.B, "global_batch": self.B * world,
            "context": self.ctx, "tokens_per_block": self.tpb, "layers": self.L,
            "hbm_kv_gb": round(max(self.dev_slots, 1) * self.slot_bytes / 1e9, 2),
            "host_pool_gb": round(self.host_slots * self.slot_bytes / 1e9, 2),
            "hbm_bytes_per_step": self.hbm_bytes, "host_bytes_per_step": self.host_bytes,
            "l2": "inputs larger than L2 (KV per step >> 126 MB), no flush",
            "parallelism": f"request-sharded x{world}, no collectives on the data path",
        }


class Workload(WorkloadLayout):
    """Device pool, pinned host pool, block tables, tails and queries for one GPU's share."""

    def __init__(self, name: str, device, seed: int):
        import torch

        from pager_hf.host_pool import HostPool

        super().__init__(name, seed)
        self.device = device
        self.dtype = {"bf16": torch.bfloat16, "f16": torch.float16}[self.w["dtype"]]
        shape = (self.L, 2, self.Hkv, self.tpb, self.D)
        self.dev_pool = torch.empty((max(self.dev_slots, 1),) + shape, dtype=self.dtype, device=device)
        self.dev_pool.normal_(generator=torch.Generator(device=device).manual_seed(seed + 1))
        self.host = HostPool((max(self.host_slots, 1),) + shape, self.dtype) if self.host_slots else None
        if self.host is not None:
            self._fill_host(seed + 2)
        self.table = self.table.to(device)
        nb = self.nb
        self.num_blocks = torch.full((self.B,), nb, dtype=torch.int32, device=device)
        self.tail_len = torch.tensor(self.tails, dtype=torch.int32, device=device)
        self.valid_lo = torch.tensor(self.lo, dtype=torch.int32, device=device) if self.window else None
        gd = torch.Generator(device=device).manual_seed(seed + 3)
        self.tail_k = torch.randn(self.B, self.Hkv, self.tpb, self.D, generator=gd, device=device).to(self.dtype)
        self.tail_v = torch.randn(self.B, self.Hkv, self.tpb, self.D, generator=gd, device=device).to(self.dtype)
        self.q = torch.randn(self.L, self.B, self.Hq, self.D, generator=gd, device=device).to(self.dtype)
        self.out = torch.empty_like(self.q)
        self.mass = torch.zeros(self.B, nb, dtype=torch.float32, device=device)
        self.max_row_tokens = nb * self.tpb + self.tpb
        self.plan = None

    def _fill_host(self, seed):
        import torch

        flat = self.host.tensor.view(-1)
        chunk = 1 << 27
        src = torch.empty(chunk, dtype=self.dtype, device=self.device)
        src.normal_(generator=torch.Generator(device=self.device).manual_seed(seed))
        for s in range(0, flat.numel(), chunk):
            n = min(chunk, flat.numel() - s)
            flat[s:s + n].copy_(src[:n], non_blocking=False)

    def build_plan(self, host_read: str, rounding: str = "running"):
        from pager_hf.streaming_attention import PagedDecodePlan

        # the reference's chunks for its rounding: groups of 64 blocks (PagedModel's default
        # streaming_group_size_blocks), then the tail
        self.plan = PagedDecodePlan(
            batch=self.B, num_query_heads=self.Hq, dev_pool=self.dev_pool,
            host_pool=None if self.host is None else self.host.tensor, num_layers=self.L, tokens_per_block=self.tpb,
            block_table=self.table, num_blocks=self.num_blocks, max_row_tokens=self.max_row_tokens,
            tail_k=self.tail_k, tail_v=self.tail_v, tail_len=self.tail_len, valid_lo=self.valid_lo,
            mass_accum=self.mass, mass_mode="row_mean", host_read=host_read, prefetch_next_step=True,
            rounding=rounding, ref_group_tokens=64 * self.tpb)
        # kernels per layer: split + combine/mass, or scores + reference max + values + combine/mass
        self.launches_per_step = self.L * (2 if self.plan.rounding == 0 else 4)

    def invalidate_staging(self):
        if self.plan.staging is not None:
            self.plan.staging.invalidate()

    def step(self, events=None):
        self.mass.zero_()
        for layer in range(self.L):
            if events is not None:
                events[layer][0].record()
            self.plan.run(self.q[layer], layer, self.out[layer])
            if events is not None:
                events[layer][1].record()

    def close(self):
        if self.host is not None:
            self.host.close()
            self.host = None


def probe_link(wl, device):
    """Measured host->device link: best of pinned cudaMemcpyAsync and zero-copy kernel reads (GB/s)."""
    import ctypes

    import torch

    from pager_hf import _lib

    if wl.host is None:
        return {"copy_gbs": None, "zero_copy_gbs": None}
    nbytes = min(1 << 30, wl.host.nbytes) // 16 * 16
    dst = torch.empty(nbytes, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device).cuda_stream
    c, z = ctypes.c_double(), ctypes.c_double()
    _lib.check(_lib.lib().pager_probe_h2d_copy_gbs(wl.host.data_ptr, dst.data_ptr(), nbytes, 5, stream, ctypes.byref(c)))
    _lib.check(_lib.lib().pager_probe_zero_copy_gbs(wl.host.data_ptr, dst.data_ptr(), nbytes, 5, stream,
                                                    ctypes.byref(z)))
    del dst
    return {"copy_gbs": c.value, "zero_copy_gbs": z.value, "probe_bytes": nbytes}


# ----------------------------------------------------------------------------- CPU oracle arm
_CPU_UNIT = None


def _cpu_unit_init(args):
    """Pool initializer: build one (request, layer) unit of the workload in this process (untimed)."""
    import numpy as np

    global _CPU_UNIT
    sys.path.insert(0, ROOT)
    from oracle import streaming_attention_oracle as orc

    hkv, hq, d, tpb, nb, tail, lo, seed = args
    rng = np.random.default_rng(seed)
    t = nb * tpb
    mk = lambda *shape: orc.round_to(rng.standard_normal(shape, dtype=np.float32), "bf16")  # noqa: E731
    valid = np.ones((1, t), np.int32)
    valid[:, :lo] = 0
    _CPU_UNIT = dict(q=mk(1, hq, d), k=mk(1, hkv, t, d), v=mk(1, hkv, t, d), tk=mk(1, hkv, tail, d),
                     tv=mk(1, hkv, tail, d), valid=valid, tpb=tpb,
                     bytes=(t - lo + tail) * 2 * hkv * d * 2)


def _cpu_unit_run(reps):
    """Time `reps` decode-attention calls of this process's unit through the CPU oracle."""
    from oracle import streaming_attention_oracle as orc

    u = _CPU_UNIT
    t0 = time.perf_counter()
    for _ in range(reps):
        orc.dense_decode_gqa(u["q"], u["k"], u["v"], u["tk"], u["tv"], u["tpb"], valid=u["valid"])
    return u["bytes"] * reps, time.perf_counter() - t0


class CpuOracleArm:
    """The reference's decode attention restated on the CPU (oracle/), one single-threaded process per host core.

    Each process holds one (request, layer) unit of the workload at the full
    context and times ``reps`` calls; a sample runs every process at once and
    reports KV bytes over wall time.
    """

    def __init__(self, wl_name: str, procs: int | None = None, reps: int = 4):
        import multiprocessing as mp

        w = WORKLOADS[wl_name]
        self.w = w
        self.reps = reps
        self.procs = procs or os.cpu_count() or 1
        nb = w["context"] // w["tpb"]
        window = w.get("window")
        lo = max(0, nb * w["tpb"] + 32 - window) if window else 0
        for var in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
            os.environ[var] = "1"  # one core per process; the processes provide the parallelism
        ctx = mp.get_context("spawn")
        self.pool = ctx.Pool(self.procs, initializer=_cpu_unit_init,
                             initargs=((w["hkv"], w["hq"], w["d"], w["tpb"], nb, 32, lo, 1000),))
        self.pool.map(_cpu_unit_run, [1] * self.procs)  # warm-up

    def sample(self):
        t0 = time.perf_counter()
        res = self.pool.map(_cpu_unit_run, [self.reps] * self.procs, chunksize=1)
        wall = time.perf_counter() - t0
        return sum(r[0] for r in res), wall

    def close(self):
        self.pool.terminate()
        self.pool.join()


class CpuTorchArm:
    """The reference's torch decode-attention path on the host cores: its dense test oracle
    (tests/test_streaming_attention.py:20-40, restated in oracle/streaming_attention_torch.py) on one
    (request, layer) unit of the workload at the full context, with ``torch.set_num_threads`` = every
    host core.  A sample is ``reps`` calls."""

    def __init__(self, wl_name: str, threads: int | None = None, reps: int = 2):
        import torch

        from oracle import streaming_attention_torch as ort

        w = WORKLOADS[wl_name]
        self.w, self.reps, self.ort = w, reps, ort
        self.procs = threads or os.cpu_count() or 1
        torch.set_num_threads(self.procs)
        nb = w["context"] // w["tpb"]
        T = nb * w["tpb"] + 32  # the blocks plus a 32-token tail
        window = w.get("window")
        lo = max(0, T - window) if window else 0
        dt = torch.bfloat16 if w["dtype"] == "bf16" else torch.float16
        g = torch.Generator().manual_seed(1000)
        self.q = torch.randn(1, w["hq"], w["d"], generator=g).to(dt)
        self.k = torch.randn(1, w["hkv"], T, w["d"], generator=g).to(dt)
        self.v = torch.randn(1, w["hkv"], T, w["d"], generator=g).to(dt)
        self.valid = torch.ones(1, T, dtype=torch.int32)
        self.valid[:, :lo] = 0
        self.n_rep, self.tpb = w["hq"] // w["hkv"], w["tpb"]
        self.bytes = (T - lo) * 2 * w["hkv"] * w["d"] * 2  # attended K and V bytes
        self.units = reps
        self._call()  # warm-up

    def _call(self):
        self.ort.dense_reference(self.q, self.k, self.v, self.n_rep, self.tpb, valid=self.valid)

    def sample(self):
        t0 = time.perf_counter()
        for _ in range(self.reps):
            self._call()
        return self.bytes * self.reps, time.perf_counter() - t0

    def close(self):
        pass


def sample_desc(arm):
    w = arm.w
    if isinstance(arm, CpuTorchArm):
        return (f"{arm.reps} calls per sample, each one (request, layer) of the workload at {w['context']} tokens: "
                f"the reference's dense torch decode attention with per-block mass (its test oracle restated), "
                f"torch.set_num_threads({arm.procs})")
    return (f"{arm.procs} processes x {arm.reps} calls, each one (request, layer) of the workload at "
            f"{w['context']} tokens; numpy restatement of the reference's dense decode attention with "
            f"per-block mass, 1 BLAS thread per process")


def cpu_arm(wl_name: str, kind: str):
    return CpuTorchArm(wl_name) if kind == "torch" else CpuOracleArm(wl_name)


# ----------------------------------------------------------------------------- arms
def run_reference_arm(args):
    world, rank, _ = _dist_env()
    if world > 1 and rank != 0:
        return 0
    arm = cpu_arm(args.workload, args.cpu_arm)
    try:
        for _ in range(args.warmup):
            arm.sample()
        tot_b, tot_t = 0, 0.0
        for _ in range(args.steps):
            b, t = arm.sample()
            tot_b += b
            tot_t += t
    finally:
        arm.close()
    gbs = tot_b / tot_t / 1e9
    w = WORKLOADS[args.workload]
    lay = WorkloadLayout(args.workload, seed=1234)
    line = {
        "impl": "reference", "metric": METRIC, "value": gbs, "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup,
        # one step = the whole workload step (every request and layer), at the rate the samples measured
        "ms_per_step": 1000 * lay.bytes_per_step / (gbs * 1e9), "sample_ms": 1000 * tot_t / args.steps,
        "units_per_step": lay.B * lay.L, "units_per_sample": getattr(arm, "units", arm.procs * arm.reps),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": w["dtype"],
        "data": "synthetic (seeded random KV)", "config": lay.config(args.gpus), "host_read": "n/a (CPU)",
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": arm.procs, "kind": "port", "sample": sample_desc(arm)},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference path = the reference's torch decode attention (its dense test oracle, "
                "tests/test_streaming_attention.py:20-40) on the host cores; the reference ships no compiled CPU "
                "implementation",
    }
    print(json.dumps(line), flush=True)
    return 0


REF_INSTALL = os.path.join(ROOT, "baseline", "_ref")


class ReferenceGpuWorkload:
    """The same workload driven through the reference's own GPU path (the installed, unmodified
    `pager_hf` package under baseline/_ref): its `KVBlockStore` holds each block as per-layer
    `[L, B, tpb, Hkv, D]` K/V tensors, on the GPU or, for host-tier blocks, in the pageable CPU
    tensors `offload_to_cpu` makes; per layer, `PagedModel._gather_layer_kv_group` gathers each
    64-block group and the Triton `streaming_attention_step` folds it, then the tail (previous tail
    + the new token, `torch.cat` as the reference does), then `streaming_attention_finalize`.  That is
    the single-pass sequence of `paged_model.py:1055-1072`, which the reference runs for the
    workloads' placements (recent_only / sinks_recent need no attention mass, `paged_model.py:40`).

    Rows share one store and one tail length (the reference's batch layout): a row with a shorter
    tail is left-padded by a zero `valid` prefix, and a sliding window is folded into the mask per
    layer (`paged_model.py:975-980`), so every row attends to exactly the tokens it does in the
    fused op and the algorithmic bytes are the same.
    """

    def __init__(self, name: str, device, seed: int, sa, gather):
        import torch

        from pager_hf.kv_block_store import KVBlockStore  # the reference's (sys.path set by the caller)

        lay = WorkloadLayout(name, seed)
        self.lay, self.sa, self.gather, self.device = lay, sa, gather, device
        w = lay.w
        self.dtype = {"bf16": torch.bfloat16, "f16": torch.float16}[w["dtype"]]
        L, B, Hkv, D, tpb, nb = lay.L, lay.B, lay.Hkv, lay.D, lay.tpb, lay.nb
        host_bit = 0x40000000
        resident = [bool(int(lay.table[0, j]) & host_bit) is False for j in range(nb)]
        self.store = KVBlockStore(tokens_per_block=tpb)
        g = torch.Generator(device=device).manual_seed(seed + 1)
        for j in range(nb):
            k = torch.randn(L, B, tpb, Hkv, D, generator=g, device=device).to(self.dtype)
            v = torch.randn(L, B, tpb, Hkv, D, generator=g, device=device).to(self.dtype)
            self.store.put_gpu(j, k, v)
            del k, v
            if not resident[j]:
                self.store.offload_to_cpu(j)
        self.block_ids = list(range(nb))
        self.group = 64  # PagedModel's default streaming_group_size_blocks
        t_max = max(lay.tails)
        gd = torch.Generator(device=device).manual_seed(seed + 3)
        self.tail_k = torch.randn(L, B, Hkv, t_max - 1, D, generator=gd, device=device).to(self.dtype)
        self.tail_v = torch.randn(L, B, Hkv, t_max - 1, D, generator=gd, device=device).to(self.dtype)
        self.new_k = torch.randn(L, B, Hkv, 1, D, generator=gd, device=device).to(self.dtype)
        self.new_v = torch.randn(L, B, Hkv, 1, D, generator=gd, device=device).to(self.dtype)
        self.q = torch.randn(L, B, lay.Hq, D, generator=gd, device=device).to(self.dtype)
        self.out = torch.empty_like(self.q)
        cols = nb * tpb + t_max
        mask = torch.ones(B, cols, dtype=torch.int32)
        for b in range(B):
            mask[b, : t_max - lay.tails[b]] = 0  # left padding of the shorter tails
        self.full_tokens = nb * tpb
        self.padding_mask = mask.to(device)
        self.window = lay.window
        self.cols = cols
        self.scale = 1.0 / math.sqrt(D)
        self.two_pass = False
        self.mass_accum = torch.zeros(nb, dtype=torch.float32, device=device)

    def _layer(self, layer: int):
        import torch

        sa, lay, device = self.sa, self.lay, self.device
        q = self.q[layer]
        m, l, acc = sa.streaming_attention_state_init(lay.B, lay.Hq, lay.D, device)
        padding_mask = self.padding_mask
        if self.window is not None:  # paged_model.py:975-980
            current_pos = self.cols - 1
            col_positions = torch.arange(padding_mask.shape[1], device=device)
            window_valid = (col_positions > (current_pos - self.window)).unsqueeze(0)
            padding_mask = padding_mask.to(torch.int32) * window_valid.to(torch.int32)
        full_tail_key = torch.cat([self.tail_k[layer], self.new_k[layer]], dim=2)
        full_tail_value = torch.cat([self.tail_v[layer], self.new_v[layer]], dim=2)
        tail_valid = padding_mask[:, self.full_tokens:].to(torch.int32)
        ids, G, tpb = self.block_ids, self.group, lay.tpb
        for i in range(0, len(ids), G):
            group_ids = ids[i: i + G]
            gk, gv, _, _ = self.gather(layer_idx=layer, block_ids=group_ids, device=device)
            gvalid = padding_mask[:, i * tpb: (i + len(group_ids)) * tpb].to(torch.int32)
            sa.streaming_attention_step(q, gk, gv, m, l, acc, valid=gvalid, scale=self.scale)
            del gk, gv
        sa.streaming_attention_step(q, full_tail_key, full_tail_value, m, l, acc, valid=tail_valid, scale=self.scale)
        self.out[layer] = sa.streaming_attention_finalize(acc, l, q.dtype)

    def _layer_two_pass(self, layer: int):
        """The two-pass sequence the reference runs for mass-scoring placements (heavy_hitter,
        sinks_heavy_hitter; ``paged_model.py:993-1050``): a stats pass over every gathered group and
        the tail, then each group gathered again for ``accumulate_step`` (writing ``block_mass``), the
        tail folded with the final statistics, and the batch-and-head mean of the mass accumulated."""
        import torch

        sa, lay, device = self.sa, self.lay, self.device
        q = self.q[layer]
        m, l, acc = sa.streaming_attention_state_init(lay.B, lay.Hq, lay.D, device)
        padding_mask = self.padding_mask
        if self.window is not None:
            col_positions = torch.arange(padding_mask.shape[1], device=device)
            window_valid = (col_positions > (self.cols - 1 - self.window)).unsqueeze(0)
            padding_mask = padding_mask.to(torch.int32) * window_valid.to(torch.int32)
        full_tail_key = torch.cat([self.tail_k[layer], self.new_k[layer]], dim=2)
        full_tail_value = torch.cat([self.tail_v[layer], self.new_v[layer]], dim=2)
        tail_valid = padding_mask[:, self.full_tokens:].to(torch.int32)
        ids, G, tpb = self.block_ids, self.group, lay.tpb
        for i in range(0, len(ids), G):
            group_ids = ids[i: i + G]
            gk, gv, _, _ = self.gather(layer_idx=layer, block_ids=group_ids, device=device)
            gvalid = padding_mask[:, i * tpb: (i + len(group_ids)) * tpb].to(torch.int32)
            sa.streaming_attention_stats_step(q, gk, m, l, valid=gvalid, scale=self.scale)
            del gk, gv
        sa.streaming_attention_stats_step(q, full_tail_key, m, l, valid=tail_valid, scale=self.scale)
        block_mass = torch.zeros(lay.B, lay.Hq, max(len(ids), 1), dtype=torch.float32, device=device)
        for i in range(0, len(ids), G):
            group_ids = ids[i: i + G]
            gk, gv, _, _ = self.gather(layer_idx=layer, block_ids=group_ids, device=device)
            gvalid = padding_mask[:, i * tpb: (i + len(group_ids)) * tpb].to(torch.int32)
            sa.streaming_attention_accumulate_step(q, gk, gv, m, l, acc, block_mass, i, tpb, valid=gvalid,
                                                   scale=self.scale)
            del gk, gv
        sa.streaming_attention_fold_fixed_step(q, full_tail_key, full_tail_value, m, l, acc, valid=tail_valid,
                                               scale=self.scale)
        self.mass_accum += block_mass.mean(dim=(0, 1))[: len(ids)]
        self.out[layer] = sa.streaming_attention_finalize(acc, l, q.dtype)

    def step(self):
        if self.two_pass:
            self.mass_accum.zero_()
        for layer in range(self.lay.L):
            (self._layer_two_pass if self.two_pass else self._layer)(layer)


def _import_reference_gpu_path():
    """The installed reference package (`pip install --target baseline/_ref`), unmodified.  Its
    `paged_model` imports the Rust `pager` extension at module level; that crate cannot be built
    offline and the block placement it decides is fixed by the workload here, so a bare module
    stands in for it and nothing on the timed path touches it."""
    import types

    if not os.path.isdir(os.path.join(REF_INSTALL, "pager_hf")):
        raise RuntimeError("reference not installed under baseline/_ref (pip install --target baseline/_ref)")
    for p in (ROOT, os.path.join(ROOT, "rust-llm-pager_b200")):
        while p in sys.path:
            sys.path.remove(p)
    sys.path.insert(0, REF_INSTALL)
    for mod in [m for m in sys.modules if m == "pager_hf" or m.startswith("pager_hf.") or m == "pager"]:
        del sys.modules[mod]
    sys.modules["pager"] = types.ModuleType("pager")
    import pager_hf.paged_model as ref_pm
    from pager_hf import streaming_attention as ref_sa

    if not ref_sa.__file__.startswith(REF_INSTALL):
        raise RuntimeError(f"imported {ref_sa.__file__}, not the installed reference")
    return ref_pm, ref_sa


def run_reference_gpu_arm(args):
    """GPU comparison: the reference's own Triton path on the same GPU, workload and byte accounting."""
    import types

    import torch

    world, rank, _ = _dist_env()
    if world > 1 and rank != 0:
        return 0
    w = WORKLOADS[args.workload]
    try:
        ref_pm, ref_sa = _import_reference_gpu_path()
    except Exception as e:  # noqa: BLE001 - reported as the line's reason
        print(json.dumps({"impl": "reference-gpu", "unavailable": f"{type(e).__name__}: {e}"}), flush=True)
        return 0
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    holder = types.SimpleNamespace(_store=None)

    def gather(**kw):
        return ref_pm.PagedModel._gather_layer_kv_group(holder, **kw)

    wl = ReferenceGpuWorkload(args.workload, device, seed=1234, sa=ref_sa, gather=gather)
    wl.two_pass = bool(getattr(args, "ref_mass", False))
    holder._store = wl.store
    for _ in range(max(args.warmup, 1)):
        wl.step()
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device) as clk:
        start.record()
        for _ in range(args.steps):
            wl.step()
        end.record()
        end.synchronize()
    ms_step = start.elapsed_time(end) / args.steps
    lay = wl.lay
    q_host = wl.q.cpu().pin_memory()
    out_host = torch.empty(wl.out.shape, dtype=wl.out.dtype).pin_memory()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        wl.q.copy_(q_host, non_blocking=True)
        wl.step()
        out_host.copy_(wl.out, non_blocking=True)
    e1.record()
    e1.synchronize()
    e2e_step = e0.elapsed_time(e1) / args.steps
    value = lay.bytes_per_step / (ms_step / 1000) / 1e9
    line = {
        "impl": "reference-gpu", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": w["dtype"], "data": "synthetic: seeded random KV in the workload's geometry",
        "config": lay.config(1), "host_read": "reference: pageable CPU blocks gathered with synchronous .to(device)",
        "decode_tokens_per_s": lay.B / (ms_step / 1000),
        "e2e": {"value": lay.bytes_per_step / (e2e_step / 1000) / 1e9, "unit": "GB/s", "ms_per_step": e2e_step,
                "h2d_bytes_per_step": q_host.numel() * q_host.element_size(),
                "d2h_bytes_per_step": out_host.numel() * out_host.element_size()},
        "clocks": clk.summary(),
        "reference_path": ("two-pass with block mass (paged_model.py:993-1050)" if wl.two_pass
                           else "single pass, no mass (paged_model.py:1055-1072)"),
        "note": "the reference's KVBlockStore, PagedModel._gather_layer_kv_group and Triton streaming_attention_* "
                "from the unmodified package in baseline/_ref, in the per-layer order of the reference_path; "
                "the Rust pager is not on this path",
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    import torch
    import torch.distributed as dist

    world, rank, local = _dist_env()
    out = _json_stdout(world)
    from pager_hf.request_shard import device_for_local_rank

    local = device_for_local_rank(local, int(os.environ.get("LOCAL_WORLD_SIZE", world)), torch.cuda.device_count())
    if world > 1:
        torch.cuda.set_device(local)
        from datetime import timedelta

        dist.init_process_group("nccl", init_method="env://", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    from pager_hf.request_shard import local_requests, max_over_ranks, shard_requests

    w = WORKLOADS[args.workload]
    # world x batch requests of equal length, routed by least load: each rank owns `batch` of them
    owners = shard_requests(world * w["batch"], world)
    mine = local_requests(owners, rank)
    assert len(mine) == w["batch"], (len(mine), w["batch"])
    wl = Workload(args.workload, device, seed=1234 + 7919 * mine[0])

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(device)

    # all ranks probe the host link at once: with N GPUs the pinned pools share host DRAM bandwidth;
    # the host tier's read mode ("auto") is then chosen from this concurrent measurement
    barrier()
    link = probe_link(wl, device)
    if link.get("copy_gbs"):
        from pager_hf.host_staging import record_link_bandwidth

        record_link_bandwidth(device, link["copy_gbs"], link["zero_copy_gbs"])
    wl.build_plan(args.host_read, args.rounding)

    # warm-up (also first-call setup: occupancy queries, smem attributes)
    for _ in range(max(args.warmup, 1)):
        wl.step()
    barrier()
    # The timed region is bracketed by two events on the launching stream.  Per-layer events are
    # not recorded inside it: an event between two kernels ends the programmatic (overlapped)
    # launch of the next layer's kernel, so the per-launch duration is the region's time divided
    # by the layer launches in it (they run back to back on one stream).
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    wl.invalidate_staging()  # no host-block copy made before the timed region counts inside it
    with ClockSampler(device) as clk:
        barrier()
        start.record()
        for _ in range(args.steps):
            wl.step()
        end.record()
        barrier()
    ms_local = start.elapsed_time(end)
    per_launch = [ms_local / (args.steps * wl.L)]
    ms_total = max_over_ranks(ms_local, device)
    # each rank's own view of the host side: its concurrently measured link and where the pages of its
    # pinned host pool sit relative to its GPU's NUMA node
    from pager_hf.host_pool import device_numa_node, numa_pages

    mine_host = {"rank": rank, "host_link": link, "gpu_numa_node": device_numa_node(local),
                 "host_pool_pages_by_numa_node": ({str(k): v for k, v in numa_pages(wl.host.data_ptr,
                                                                                    wl.host.nbytes).items()}
                                                  if wl.host is not None else {})}
    per_rank_host = [mine_host]
    if world > 1:
        per_rank_host = [None] * world
        dist.all_gather_object(per_rank_host, mine_host)
    ms_step = ms_total / args.steps
    value = world * wl.bytes_per_step / (ms_step / 1000) / 1e9
    tokens_per_s = world * wl.B / (ms_step / 1000)

    # end-to-end through the public API with host buffers: q from pinned host memory in, output + mass out
    q_host = wl.q.cpu().pin_memory()
    out_host = torch.empty(wl.out.shape, dtype=wl.out.dtype).pin_memory()
    mass_host = torch.empty(wl.mass.shape, dtype=torch.float32).pin_memory()
    wl.invalidate_staging()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        wl.q.copy_(q_host, non_blocking=True)
        wl.step()
        out_host.copy_(wl.out, non_blocking=True)
        mass_host.copy_(wl.mass, non_blocking=True)
    e1.record()
    barrier()
    e2e_step = max_over_ranks(e0.elapsed_time(e1), device) / args.steps
    e2e_value = world * wl.bytes_per_step / (e2e_step / 1000) / 1e9

    hbm_peak, peak_src = measured_peaks()
    h2d = max([x for x in (link.get("copy_gbs"), link.get("zero_copy_gbs")) if x] or [0.0])
    launch_ms = statistics.mean(per_launch)
    bytes_per_launch = wl.bytes_per_step / wl.L
    achieved = bytes_per_launch / (launch_ms / 1000) / 1e9
    t_hbm = wl.hbm_bytes / wl.L / (hbm_peak * 1e9)
    t_link = wl.host_bytes / wl.L / (h2d * 1e9) if wl.host_bytes else 0.0
    t_roof = t_hbm + t_link  # combined roofline: HBM time plus host-link time
    combined_peak = bytes_per_launch / t_roof / 1e9
    # DRAM traffic per launch: the ncu capture of the split kernel on the small HBM-resident case read
    # and wrote NCU_DRAM_PER_HBM_BYTE bytes per algorithmic HBM byte; scaled here to the bytes this
    # launch's kernels read from DRAM -- the HBM tier, plus the staged copies of host blocks when the
    # host tier is staged (zero-copy host reads cross the link, not DRAM) -- and to those copies
    # themselves: the copy engines write every staged host byte into device memory first.
    staged = wl.plan.host_read == "staged"
    dram_ratio = NCU_DRAM_PER_HBM_BYTE["one_pass" if wl.plan.rounding == 0 else "exact"]
    kernel_dram_bytes = (wl.hbm_bytes + (wl.host_bytes if staged else 0)) / wl.L * dram_ratio
    copy_engine_writes = wl.host_bytes / wl.L if staged else 0.0
    traffic = kernel_dram_bytes + copy_engine_writes
    clocks = clk.summary()
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": w["dtype"],
        "data": "synthetic: seeded random KV in the workload's geometry (no checkpoints offline)",
        "config": wl.config(world), "host_read": wl.plan.host_read, "rounding": args.rounding,
        "decode_tokens_per_s": tokens_per_s,
        "roofline": {
            "bound": "hbm", "achieved": achieved, "peak": combined_peak, "unit": "GB/s",
            "frac": achieved / combined_peak, "traffic": traffic,
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one layer's kernels on prof-b8 "
                              f"(caches warm between kernels; {dram_ratio:.4f} B per algorithmic HBM byte) scaled to "
                              "the bytes this "
                              "launch reads from DRAM (HBM tier + staged copies), plus the copy engines' writes of "
                              f"the staged host blocks ({copy_engine_writes:.0f} B per launch)",
            "traffic_per_algorithmic_byte": traffic / (wl.bytes_per_step / wl.L),
            "kernel": ("paged decode attention per layer: " + ("split-KV kernel + combine/mass kernel"
                       if wl.plan.rounding == 0 else "scores pass + reference-max scan + values pass + combine/mass")
                       + ", back to back"),
            "peak_kind": f"combined roofline: HBM {hbm_peak:.0f} GB/s ({peak_src}) + host link {h2d:.1f} GB/s "
                         f"(measured live); peak = bytes / (hbm_bytes/HBM + host_bytes/link)",
            "launch_ms": launch_ms, "bytes_per_launch": bytes_per_launch,
            # staged host reads overlap the link with the HBM reads (the next layer's copies run
            # during this layer's kernel), so the tighter bound is the slower of the two
            "frac_of_overlapped_bound": achieved / (bytes_per_launch / max(t_hbm, t_link) / 1e9),
        },
        "host_link": link,
        "host_per_rank": per_rank_host,
        "e2e": {"value": e2e_value, "unit": "GB/s", "ms_per_step": e2e_step,
                "h2d_bytes_per_step": q_host.numel() * q_host.element_size(),
                "d2h_bytes_per_step": out_host.numel() * out_host.element_size() + mass_host.numel() * 4},
        "gpu_launches": wl.launches_per_step * args.steps,
        "clocks": clocks,
    }
    wl.close()
    del wl
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank == 0:
        if world == 1 and not args.no_extras:
            if args.workload != "hbm-32k":
                line["kernel_hbm_32k"] = kernel_only_measurement("hbm-32k", device, args.rounding, hbm_peak, peak_src)
                if args.rounding != "one_pass":
                    line["kernel_hbm_32k_one_pass"] = kernel_only_measurement("hbm-32k", device, "one_pass", hbm_peak,
                                                                              peak_src)
            line["model_decode"] = model_level_decode(device)
        if world == 1 and not args.no_cpu_baseline:
            arm = cpu_arm(args.workload, args.cpu_arm)
            try:
                arm.sample()
                b, t_cpu = arm.sample()
            finally:
                arm.close()
            line["cpu_baseline"] = {"value": b / t_cpu / 1e9, "unit": "GB/s", "cores": arm.procs, "kind": "port",
                                    "sample": sample_desc(arm)}
        print(json.dumps(line), file=out, flush=True)
    return 0


def kernel_only_measurement(name: str, device, rounding: str, hbm_peak: float, peak_src: str, steps: int = 5):
    """The fused op alone on an HBM-resident workload (no host tier), against the measured HBM peak:
    the kernel-bound figure beside a headline that the host link bounds."""
    import torch

    wl = Workload(name, device, seed=4321)
    try:
        wl.build_plan("zero_copy", rounding)
        for _ in range(2):
            wl.step()
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            wl.step()
        e1.record()
        e1.synchronize()
        ms = e0.elapsed_time(e1) / steps
        gbs = wl.bytes_per_step / (ms / 1000) / 1e9
        return {"workload": name, "value": gbs, "unit": "GB/s", "ms_per_step": ms, "launch_ms": ms / wl.L,
                "peak": hbm_peak, "frac": gbs / hbm_peak, "peak_kind": f"HBM copy peak, {peak_src}",
                "rounding": rounding, "decode_tokens_per_s": wl.B / (ms / 1000), "steps": steps}
    finally:
        wl.close()
        del wl
        torch.cuda.empty_cache()


def model_level_decode(device, config: str = "cfg4", new_tokens: int = 32):
    """Model-level decode through ``PagedModel.generate``: BASELINE config 4 (random-init Mistral-7B
    architecture, 8 rows x 32,768 tokens, window 4096, 5 % of blocks resident, sinks_recent, bf16),
    ``new_tokens`` greedy tokens after the prompt's prefill, with the default reference rounding and
    CUDA-graph steps.  Wall clock around the decode call, device synchronised on both sides; every
    step reads its argmax back to the host, as generate() does."""
    import torch

    from pager_hf import generate_bench as gb

    c = gb.CONFIGS[config]
    model = gb.build_model(c)
    try:
        ids, mask, lens = gb.build_prompt(c)
        toks, dt, peak, prefill_s, stats, resident, nb, host_read = gb.paged_decode(model, c, ids, mask, new_tokens)
        B = ids.shape[0]
        return {"config": f"{config}: random-init {c['family']} ({c['num_hidden_layers']} layers, hidden "
                          f"{c['hidden_size']}), {B} rows x {max(lens)} tokens, window {c.get('sliding_window')}, "
                          f"{c['policy']}, {int(100 * c['resident'])}% of blocks resident",
                "decode_tokens_per_s": B * new_tokens / dt, "ms_per_step": 1000 * dt / new_tokens,
                "new_tokens": new_tokens, "kv_gbs": gb.kv_bytes_per_step(c, lens, new_tokens // 2) / (dt / new_tokens) / 1e9,
                "prefill_s": prefill_s, "peak_gpu_gb": peak / 1e9, "host_read": host_read,
                "rounding": "reference (running max per 64-token tile)", "dtype": c.get("dtype", "f16")}
    finally:
        del model
        torch.cuda.empty_cache()


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="cfg5-32k", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference-gpu"],
                    help="ours; reference = the reference's algorithm on the host cores; reference-gpu = the "
                         "reference's own Triton path from baseline/_ref on the same GPU (comparison)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the kernel-only hbm-32k figure and the model-level decode of config 4 (N = 1 only)")
    ap.add_argument("--rounding", default="running", choices=["running", "final", "one_pass"],
                    help="rounding of p before P.V: the reference's one-pass rule (running max per 64-token tile), "
                         "its two-pass rule (final max), or the fused one-pass kernel")
    ap.add_argument("--cpu-arm", default="torch", choices=["torch", "numpy"],
                    help="CPU baseline: the reference's dense torch path with all host threads, or the numpy "
                         "restatement in one single-threaded process per core")
    ap.add_argument("--ref-mass", action="store_true",
                    help="reference-gpu: the reference's two-pass path that also writes the per-block mass "
                         "(what its heavy-hitter placements run; ours always emits the mass)")
    ap.add_argument("--host-read", default="auto", choices=["auto", "zero_copy", "staged"],
                    help="host tier: zero-copy kernel reads, copy-engine staging, or pick from the measured link")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference_arm(args)
    if args.impl == "reference-gpu":
        return run_reference_gpu_arm(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
