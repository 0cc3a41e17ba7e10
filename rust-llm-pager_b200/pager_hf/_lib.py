"""ctypes binding of ``libpager_b200.so`` (declared in include/pager_b200.h).

The library is the product: there is no Python or torch fallback.  Loading
fails loudly (``ImportError``) when the shared library has not been built,
and every call's status code is turned into the exception the reference
raises for the same condition (``ValueError`` for bad arguments,
``NotImplementedError`` for unsupported GQA fan-out / head_dim, ``RuntimeError``
for CUDA failures).
"""

from __future__ import annotations

import ctypes
import os
import re
import threading

import torch

PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# The in-tree build, unless PAGER_B200_LIB points elsewhere (e.g. when these modules are dropped
# into the reference's own pager_hf package).
LIB_PATH = os.environ.get("PAGER_B200_LIB") or os.path.join(PKG_ROOT, "libpager_b200.so")
HEADER_PATH = os.path.join(os.path.dirname(PKG_ROOT), "include", "pager_b200.h")

PAGER_OK = 0
PAGER_ERR_INVALID = 1
PAGER_ERR_UNSUPPORTED = 2
PAGER_ERR_CUDA = 3
PAGER_ERR_SCRATCH = 4
PAGER_ERR_TIMEOUT = 5

# block-table entry tags (include/pager_b200.h PAGER_HOST_SLOT_BIT / PAGER_STAGE_SLOT_BIT)
HOST_SLOT_BIT = 0x40000000
STAGE_SLOT_BIT = 0x20000000

BACKEND_AUTO, BACKEND_MMA, BACKEND_FMA = 0, 1, 2
# rounding of p before P.V (include/pager_b200.h PAGER_ROUND_*): the one-pass kernel, or the reference's
# own rounding against its running max per 64-token tile (its one-pass path) / its final max (two-pass)
ROUND_ONE_PASS, ROUND_RUNNING, ROUND_FINAL = 0, 1, 2
ROUNDING_CODE = {"one_pass": ROUND_ONE_PASS, "running": ROUND_RUNNING, "final": ROUND_FINAL}
MASS_NONE, MASS_ROW_MEAN, MASS_BATCH_MEAN = 0, 1, 2

DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}

_vp = ctypes.c_void_p
_i = ctypes.c_int
_f = ctypes.c_float
_sz = ctypes.c_size_t
_i64 = ctypes.c_int64

_SIGNATURES = {
    "pager_last_error": (ctypes.c_char_p, []),
    "pager_version": (_i, []),
    "pager_device_status": (_i, [_i, ctypes.POINTER(_i)]),
    "pager_status_snapshot_async": (_i, [_vp, _vp]),
    "pager_attn_state_init": (_i, [_vp, _vp, _vp, _i64, _i, _vp]),
    "pager_attn_finalize": (_i, [_vp, _vp, _vp, _i, _i64, _i, _vp]),
    "pager_attn_chunk_scratch_bytes": (_sz, [_i, _i, _i, _i, _i, _i, _i, _i]),
    "pager_attn_step": (_i, [_vp, _i, _vp, _vp, _i, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _f, _f, _i, _vp,
                             _sz, _vp]),
    "pager_attn_stats_step": (_i, [_vp, _i, _vp, _i, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _f, _f, _i, _vp, _sz,
                                   _vp]),
    "pager_attn_accumulate_step": (_i, [_vp, _i, _vp, _vp, _i, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i,
                                        _i, _i, _f, _f, _i, _vp, _sz, _vp]),
    "pager_attn_fold_fixed_step": (_i, [_vp, _i, _vp, _vp, _i, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _f, _f, _i,
                                        _vp, _sz, _vp]),
    "pager_paged_decode_scratch_bytes": (_sz, [_i, _i, _i, _i, _i, _i, _i, _i]),
    "pager_paged_decode_attention": (_i, [_vp, _i, _vp, _i, _vp, _i, _i, _i, _i, _i, _i, _i, _vp, _i, _vp, _vp,
                                          _vp, _vp, _i, _vp, _vp, _vp, _i, _i, _f, _f, _i, _vp, _i, _vp, _vp, _i,
                                          _i, _vp, _sz, _vp]),
    "pager_paged_decode_attention_noalloc": (_i, [_vp, _i, _vp, _i, _vp, _i, _i, _i, _i, _i, _i, _i, _vp, _i, _vp,
                                                  _vp, _vp, _vp, _i, _vp, _vp, _vp, _i, _i, _f, _f, _i, _vp, _i,
                                                  _vp, _vp, _i, _i, _vp]),
    "pager_append_tokens": (_i, [_vp, _i, _i, _i, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _i, _vp]),
    "pager_paged_decode_attention_staged": (_i, [_vp, _i, _vp, _i, _vp, _i, _vp, _i, _i, _i, _i, _i, _i, _i, _vp,
                                                 _i, _vp, _vp, _vp, _vp, _i, _vp, _vp, _vp, _i, _i, _f, _f, _i,
                                                 _vp, _i, _vp, _vp, _i, _i, _vp, _sz, _vp]),
    "pager_paged_decode_scratch_bytes_rounded": (_sz, [_i, _i, _i, _i, _i, _i, _i, _i]),
    "pager_paged_decode_attention_rounded": (_i, [_vp, _i, _vp, _i, _vp, _i, _vp, _i, _i, _i, _i, _i, _i, _i, _vp,
                                                  _i, _vp, _vp, _vp, _vp, _i, _vp, _vp, _vp, _i, _i, _f, _f, _i,
                                                  _vp, _i, _vp, _vp, _i, _i, _i, _i, _vp, _vp, _vp, _sz, _vp]),
    "pager_stage_host_blocks": (_i, [_vp, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _i, _vp]),
    "pager_selftest_bounded_wait": (_i, [ctypes.c_ulonglong, ctypes.POINTER(ctypes.c_ulonglong), _vp]),
    "pager_host_pool_alloc": (_i, [_sz, ctypes.POINTER(_vp)]),
    "pager_host_pool_free": (_i, [_vp]),
    "pager_probe_h2d_copy_gbs": (_i, [_vp, _vp, _sz, _i, _vp, ctypes.POINTER(ctypes.c_double)]),
    "pager_probe_zero_copy_gbs": (_i, [_vp, _vp, _sz, _i, _vp, ctypes.POINTER(ctypes.c_double)]),
}

_lock = threading.Lock()
_lib = None


def declared_symbols(header_path: str = HEADER_PATH) -> list[str]:
    """Every function name declared in the C header (for the export check)."""
    text = open(header_path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(pager_[a-z0-9_]+)\s*\(", text)))


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the shared library and declare every entry point's signature."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise ImportError(
                f"{path} is missing: build it with `python rust-llm-pager_b200/build_lib.py` "
                "(or __graft_entry__.build()). There is no CPU fallback."
            )
        lib = ctypes.CDLL(path)
        for name, (restype, argtypes) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = lib
        return lib


def lib() -> ctypes.CDLL:
    return _lib if _lib is not None else load_library()


def last_error() -> str:
    msg = lib().pager_last_error()
    return msg.decode() if msg else ""


def check(rc: int) -> None:
    if rc == PAGER_OK:
        return
    msg = last_error()
    if rc == PAGER_ERR_INVALID:
        raise ValueError(msg)
    if rc == PAGER_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise RuntimeError(f"libpager_b200 error {rc}: {msg}")


def device_status(device: int) -> int:
    """Read and clear the device status word (non-zero after a bounded wait ran out or a bad block entry)."""
    out = _i(0)
    check(lib().pager_device_status(device, ctypes.byref(out)))
    return out.value


STATUS_TIMEOUT = 5
STATUS_BAD_SLOT = 6
_STATUS_TEXT = {
    STATUS_TIMEOUT: "a bounded wait in a decode kernel ran out (a copy or a stage never arrived); the step's "
                    "attention is incomplete",
    STATUS_BAD_SLOT: "a block-table entry or a tail write named a slot outside its pool; that block was skipped, so "
                     "the step's attention is wrong",
}


class DeviceStatusError(RuntimeError):
    """A decode step's kernels reported a fault through the device status word (``code``: 5 for a
    timed-out wait, 6 for a slot outside its pool).  The kernels never dereference such a slot and
    always finish, so the CUDA context stays usable; the step's result must not be used."""

    def __init__(self, code: int, where: str = "decode step"):
        self.code = int(code)
        super().__init__(f"{where}: device status {self.code}: {_STATUS_TEXT.get(self.code, 'unknown fault')}")


class StatusWatch:
    """Per-step check of a device's status word at a synchronisation the step already has.

    ``enqueue(stream)`` queues, behind the step's kernels, a copy of the word into a page-locked
    host int and a reset of the word (``pager_status_snapshot_async``); once the stream has been
    synchronised, ``check()`` raises ``DeviceStatusError`` if the step set it.  One watch per
    (thread, device): ``watch_for(device)``."""

    def __init__(self, device: torch.device):
        self.device = torch.device(device)
        self.host = torch.zeros(1, dtype=torch.int32).pin_memory()

    def enqueue(self, stream: int | None = None) -> None:
        with torch.cuda.device(self.device):
            s = torch.cuda.current_stream(self.device).cuda_stream if stream is None else stream
            check(lib().pager_status_snapshot_async(self.host.data_ptr(), s))

    def check(self, where: str = "decode step") -> None:
        code = int(self.host[0])
        if code:
            self.host[0] = 0
            raise DeviceStatusError(code, where)

    def sync_and_check(self, where: str = "decode step") -> None:
        """Enqueue, wait for the current stream, check: for a step with no later synchronisation."""
        self.enqueue()
        torch.cuda.current_stream(self.device).synchronize()
        self.check(where)


_watches = threading.local()


def watch_for(device) -> StatusWatch:
    device = torch.device(device)
    if device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    table = getattr(_watches, "table", None)
    if table is None:
        table = _watches.table = {}
    w = table.get(device.index)
    if w is None:
        w = table[device.index] = StatusWatch(device)
    return w


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream
