"""CPU checks of the drop-in boundary: the C-ABI library loads, exports every
symbol include/pager_b200.h declares, and the Python wrappers reject bad input
with the reference's exception types before any device work."""

import ctypes

import pytest
import torch


def test_library_exports_every_declared_symbol():
    from pager_hf import _lib

    names = _lib.declared_symbols()
    assert len(names) >= 16
    raw = ctypes.CDLL(_lib.LIB_PATH)
    missing = [n for n in names if not hasattr(raw, n)]
    assert not missing, f"symbols declared in include/pager_b200.h but not exported: {missing}"
    # every declared symbol also has a ctypes signature
    assert set(names) <= set(_lib._SIGNATURES), set(names) - set(_lib._SIGNATURES)


def test_version_and_status_codes():
    from pager_hf import _lib

    assert _lib.lib().pager_version() == 1
    with pytest.raises(ValueError):
        _lib.check(_lib.PAGER_ERR_INVALID)
    with pytest.raises(NotImplementedError):
        _lib.check(_lib.PAGER_ERR_UNSUPPORTED)
    with pytest.raises(RuntimeError):
        _lib.check(_lib.PAGER_ERR_CUDA)
    _lib.check(_lib.PAGER_OK)


def test_n_rep_guard_raises_not_implemented():
    """streaming_attention.py:69-74: n_rep > 16 -> NotImplementedError (checked before device work)."""
    from pager_hf import streaming_attention as sa

    q = torch.zeros(1, 34, 8)
    k = torch.zeros(1, 2, 4, 8)
    m, l, acc = torch.zeros(1, 34), torch.zeros(1, 34), torch.zeros(1, 34, 8)
    with pytest.raises(NotImplementedError, match="n_rep up to 16"):
        sa.streaming_attention_step(q, k, k, m, l, acc)
    with pytest.raises(NotImplementedError):
        sa.streaming_attention_stats_step(q, k, m, l)


def test_cpu_tensors_rejected_no_fallback():
    from pager_hf import streaming_attention as sa

    q = torch.zeros(1, 8, 8)
    k = torch.zeros(1, 2, 4, 8)
    m, l, acc = torch.zeros(1, 8), torch.zeros(1, 8), torch.zeros(1, 8, 8)
    with pytest.raises(ValueError, match="CUDA"):
        sa.streaming_attention_step(q, k, k, m, l, acc)


def test_module_surface_matches_reference():
    """The six public functions and the tuning constants of streaming_attention.py:11-74, :444-670."""
    from pager_hf import streaming_attention as sa

    for name in ("streaming_attention_state_init", "streaming_attention_step", "streaming_attention_stats_step",
                 "streaming_attention_accumulate_step", "streaming_attention_fold_fixed_step",
                 "streaming_attention_finalize", "_validate_n_rep", "_default_valid", "_default_active"):
        assert callable(getattr(sa, name))
    assert sa._BLOCK_KV == 64 and sa._M_TILE == 16 and sa._MIN_DOT_DIM == 16


def test_python_constants_match_the_header():
    """Status codes, dtype / backend / mass-mode codes and block-table tags of ``_lib`` equal the
    values ``include/pager_b200.h`` defines, so the ctypes binding and the C ABI cannot drift."""
    import re

    from pager_hf import _lib as L
    from pager_hf import host_staging, kv_block_store

    hdr = open(L.HEADER_PATH).read()
    defined = {name: int(val, 0) for name, val in re.findall(r"\b(PAGER_[A-Z0-9_]+)\s*=\s*(\w+)", hdr)}
    defined.update({name: int(val, 0) for name, val in re.findall(r"#define (PAGER_\w+_BIT) (0x[0-9a-fA-F]+)", hdr)})
    for name in ("PAGER_OK", "PAGER_ERR_INVALID", "PAGER_ERR_UNSUPPORTED", "PAGER_ERR_CUDA", "PAGER_ERR_SCRATCH",
                 "PAGER_ERR_TIMEOUT"):
        assert getattr(L, name) == defined[name], name
    assert (L.BACKEND_AUTO, L.BACKEND_MMA, L.BACKEND_FMA) == (
        defined["PAGER_BACKEND_AUTO"], defined["PAGER_BACKEND_MMA"], defined["PAGER_BACKEND_FMA"])
    assert (L.MASS_NONE, L.MASS_ROW_MEAN, L.MASS_BATCH_MEAN) == (
        defined["PAGER_MASS_NONE"], defined["PAGER_MASS_ROW_MEAN"], defined["PAGER_MASS_BATCH_MEAN"])
    assert L.DTYPE_CODE == {torch.float32: defined["PAGER_DTYPE_F32"], torch.float16: defined["PAGER_DTYPE_F16"],
                            torch.bfloat16: defined["PAGER_DTYPE_BF16"]}
    assert L.HOST_SLOT_BIT == host_staging.HOST_SLOT_BIT == kv_block_store.HOST_SLOT_BIT == defined["PAGER_HOST_SLOT_BIT"]
    assert L.STAGE_SLOT_BIT == host_staging.STAGE_SLOT_BIT == defined["PAGER_STAGE_SLOT_BIT"]
