"""``pager``: the block-placement pager, bound from ``libpager_core.so``.

Same module name and class surface as the reference's pyo3 extension
(``pager/src/lib.rs:9-74``, ``pager/src/metrics.rs:4-27``), so
``import pager`` / ``pager.PyPager(...)`` in ``pager_hf/paged_model.py:13``
and its callers work unchanged:

    PyPager(vram, ram, recent, rebalance_interval=32, promote_margin=0.10,
            ram_promote_margin=0.20, policy="heavy_hitter")
    .on_step(token_idx, layer, attention)   # attention: sequence of floats
    .force_rebalance(token_idx)
    .metrics() -> Metrics                   # tokens, vram_peak, ram_peak, swap_vram_ram,
                                            # swap_ram_ssd, attention_mass_total, attention_mass_vram
    .tiers() -> list[int]                   # 0 VRAM, 1 RAM, 2 SSD per block
    .vram_block_ids() -> list[int]

Argument conversion follows pyo3's: integers must be ints (``TypeError``
otherwise) and fit the Rust type (``OverflowError`` for negatives or too large
values); margins accept any real number; ``policy`` must be a ``str``.  A
rebalance that falls due with ``rebalance_interval=0`` raises
``PanicException`` where the Rust code panics on the modulo.
"""

from __future__ import annotations

import ctypes
import operator
import os

import numpy as np

__all__ = ["PyPager", "Metrics", "PanicException"]

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("PAGER_CORE_LIB", os.path.join(os.path.dirname(_HERE), "libpager_core.so"))
_U64 = (1 << 64) - 1
_U32 = (1 << 32) - 1


class PanicException(BaseException):
    """Raised where the Rust pager panics (pyo3 maps a panic to a BaseException)."""


class _CMetrics(ctypes.Structure):
    _fields_ = [("tokens", ctypes.c_uint64), ("vram_peak", ctypes.c_uint64), ("ram_peak", ctypes.c_uint64),
                ("swap_vram_ram", ctypes.c_uint64), ("swap_ram_ssd", ctypes.c_uint64),
                ("attention_mass_total", ctypes.c_double), ("attention_mass_vram", ctypes.c_double)]


_lib = None


def lib():
    """Load ``libpager_core.so`` once (raises OSError with the path if it is not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"libpager_core.so not found at {LIB_PATH}; build it with "
                          "`python rust-llm-pager_b200/build_lib.py`")
        L = ctypes.CDLL(LIB_PATH)
        vp, u64, sz = ctypes.c_void_p, ctypes.c_uint64, ctypes.c_size_t
        sigs = {
            "pager_core_last_error": (ctypes.c_char_p, []),
            "pager_core_policy_code": (ctypes.c_int, [ctypes.c_char_p]),
            "pager_core_new": (vp, [u64, u64, u64, u64, ctypes.c_float, ctypes.c_float, ctypes.c_char_p]),
            "pager_core_free": (None, [vp]),
            "pager_core_on_step": (ctypes.c_int, [vp, u64, ctypes.c_uint32, vp, sz]),
            "pager_core_force_rebalance": (ctypes.c_int, [vp, u64]),
            "pager_core_metrics_get": (ctypes.c_int, [vp, ctypes.POINTER(_CMetrics)]),
            "pager_core_num_blocks": (sz, [vp]),
            "pager_core_tiers": (sz, [vp, vp, sz]),
            "pager_core_vram_block_ids": (sz, [vp, vp, sz]),
            "pager_core_scores": (sz, [vp, vp, sz]),
        }
        for name, (res, args) in sigs.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
        _lib = L
    return _lib


def _uint(value, name, hi=_U64):
    if isinstance(value, float):
        raise TypeError(f"'{type(value).__name__}' object cannot be interpreted as an integer ({name})")
    v = operator.index(value)
    if v < 0 or v > hi:
        raise OverflowError(f"{name}={v} out of range for an unsigned {hi.bit_length()}-bit integer")
    return v


def _real(value, name):
    try:
        return float(value)
    except (TypeError, ValueError):
        raise TypeError(f"{name} must be a real number, got {type(value).__name__}") from None


class Metrics:
    """Snapshot of the pager's counters (``metrics.rs:4-27``), read-only attributes."""

    __slots__ = ("_v",)

    def __init__(self, c: _CMetrics):
        object.__setattr__(self, "_v", {f: getattr(c, f) for f, _ in _CMetrics._fields_})

    def __getattr__(self, name):
        try:
            return self._v[name]
        except KeyError:
            raise AttributeError(name) from None

    def __setattr__(self, name, value):
        raise AttributeError(f"Metrics.{name} is read-only")

    def __repr__(self):
        return "Metrics(" + ", ".join(f"{k}={v}" for k, v in self._v.items()) + ")"


class PyPager:
    """Block-placement pager over VRAM / RAM / SSD tiers (``lib.rs:9-67``)."""

    def __init__(self, vram, ram, recent, rebalance_interval=32, promote_margin=0.10, ram_promote_margin=0.20,
                 policy="heavy_hitter"):
        if not isinstance(policy, str):
            raise TypeError(f"policy must be str, got {type(policy).__name__}")
        args = (_uint(vram, "vram"), _uint(ram, "ram"), _uint(recent, "recent"),
                _uint(rebalance_interval, "rebalance_interval"), _real(promote_margin, "promote_margin"),
                _real(ram_promote_margin, "ram_promote_margin"), policy.encode())
        self._h = None
        h = lib().pager_core_new(*args)
        if not h:
            raise MemoryError("pager_core_new failed")
        self._h = h

    def __del__(self):
        h, self._h = getattr(self, "_h", None), None
        if h and _lib is not None:
            _lib.pager_core_free(h)

    def _check(self, rc):
        if rc:
            raise PanicException(lib().pager_core_last_error().decode())

    def on_step(self, token_idx, layer, attention):
        if isinstance(attention, (str, bytes)):
            raise TypeError("Can't extract `str` to `Vec`")
        a = np.ascontiguousarray(np.asarray(attention, dtype=np.float32).reshape(-1))
        self._check(lib().pager_core_on_step(self._h, _uint(token_idx, "token_idx"), _uint(layer, "layer", _U32),
                                             a.ctypes.data if a.size else None, a.size))

    def force_rebalance(self, token_idx):
        self._check(lib().pager_core_force_rebalance(self._h, _uint(token_idx, "token_idx")))

    def metrics(self) -> Metrics:
        c = _CMetrics()
        self._check(lib().pager_core_metrics_get(self._h, ctypes.byref(c)))
        return Metrics(c)

    def tiers(self) -> list[int]:
        n = lib().pager_core_num_blocks(self._h)
        out = np.empty(n, dtype=np.uint8)
        lib().pager_core_tiers(self._h, out.ctypes.data if n else None, n)
        return out.tolist()

    def vram_block_ids(self) -> list[int]:
        n = lib().pager_core_num_blocks(self._h)
        out = np.empty(n, dtype=np.uint64)
        k = lib().pager_core_vram_block_ids(self._h, out.ctypes.data if n else None, n)
        return out[:k].tolist()

    def scores(self) -> list[float]:
        """Per-block smoothed attention scores (f32), an inspection helper the pyo3 class does not have."""
        n = lib().pager_core_num_blocks(self._h)
        out = np.empty(n, dtype=np.float32)
        lib().pager_core_scores(self._h, out.ctypes.data if n else None, n)
        return out.tolist()
