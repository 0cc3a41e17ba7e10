"""The allocation-free entry point, checked against the regular one.

``pager_paged_decode_attention_noalloc`` serves callers that cannot allocate
device memory -- a client binding the C ABI from a host language without a
CUDA allocator, or a serving loop that allocates nothing after start-up.  It
takes the same arguments as ``pager_paged_decode_attention`` minus the scratch
buffer and uses a fixed array of device memory built into the library instead.

This file is named to be collected last: a failure here never hides the rest of
the suite in a run that stops at the first failure.  It must pass both on its
own in a fresh process and after the other tests (the array keeps whatever the
previous call left in it; nothing in it needs to start at zero).
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

HOST = 0x40000000


def _setup(seed, B, Hq, Hkv, D, tpb, L, nbs, tails, dtype):
    from pager_hf.host_pool import HostPool

    g = torch.Generator().manual_seed(seed)
    slots = sum(nbs) + 2
    dev = torch.randn(slots, L, 2, Hkv, tpb, D, generator=g).to(dtype).cuda()
    host = HostPool((slots, L, 2, Hkv, tpb, D), dtype)
    host.tensor.copy_(torch.randn(slots, L, 2, Hkv, tpb, D, generator=g).to(dtype))
    table = torch.full((B, max(nbs)), -1, dtype=torch.int32)
    nxt = 0
    for b, nb in enumerate(nbs):
        for j in range(nb):
            table[b, j] = (nxt | HOST) if j % 3 == 2 else nxt
            nxt += 1
    tail_cap = max(tails)
    return dict(
        q=torch.randn(B, Hq, D, generator=g).to(dtype).cuda(), dev=dev, host=host, table=table.cuda(),
        nbs=torch.tensor(nbs, dtype=torch.int32).cuda(), tails=torch.tensor(tails, dtype=torch.int32).cuda(),
        tk=torch.randn(B, Hkv, tail_cap, D, generator=g).to(dtype).cuda(),
        tv=torch.randn(B, Hkv, tail_cap, D, generator=g).to(dtype).cuda(),
        B=B, Hq=Hq, Hkv=Hkv, D=D, tpb=tpb, L=L, max_row=max(nb * tpb + t for nb, t in zip(nbs, tails)),
        dtype=dtype)


def _args(s, layer, out, block_mass, accum, backend=0):
    from pager_hf import _lib

    code = _lib.DTYPE_CODE[s["dtype"]]
    return [s["q"].data_ptr(), code, s["dev"].data_ptr(), s["dev"].shape[0], s["host"].data_ptr,
            s["host"].shape[0], code, s["L"], layer, s["Hkv"], s["tpb"], s["D"], s["table"].data_ptr(),
            s["table"].shape[1], s["nbs"].data_ptr(), s["tk"].data_ptr(), s["tv"].data_ptr(), s["tails"].data_ptr(),
            s["tk"].shape[2], None, None, None, s["B"], s["Hq"], 1.0 / s["D"] ** 0.5, 0.0, s["max_row"],
            out.data_ptr(), code, block_mass.data_ptr(), accum.data_ptr(), _lib.MASS_ROW_MEAN, backend]


def _regular(s, layer, backend=0):
    from pager_hf import _lib

    lib = _lib.lib()
    out = torch.empty(s["B"], s["Hq"], s["D"], dtype=s["dtype"], device="cuda")
    bm = torch.zeros(s["B"], s["Hq"], s["table"].shape[1], device="cuda")
    acc = torch.zeros(s["B"], s["table"].shape[1], device="cuda")
    nbytes = lib.pager_paged_decode_scratch_bytes(s["B"], s["Hq"], s["Hkv"], s["D"], _lib.DTYPE_CODE[s["dtype"]],
                                                  s["tpb"], s["table"].shape[1], s["max_row"])
    scratch = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.pager_paged_decode_attention(*_args(s, layer, out, bm, acc, backend), scratch.data_ptr(), nbytes,
                                                stream))
    torch.cuda.synchronize()
    return out.float().cpu(), bm.cpu(), acc.cpu()


def _noalloc(s, layer, backend=0):
    from pager_hf import _lib

    out = torch.empty(s["B"], s["Hq"], s["D"], dtype=s["dtype"], device="cuda")
    bm = torch.zeros(s["B"], s["Hq"], s["table"].shape[1], device="cuda")
    acc = torch.zeros(s["B"], s["table"].shape[1], device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(_lib.lib().pager_paged_decode_attention_noalloc(*_args(s, layer, out, bm, acc, backend), stream))
    torch.cuda.synchronize()
    return out.float().cpu(), bm.cpu(), acc.cpu()


def test_noalloc_matches_regular_entry_on_two_calls_in_a_row():
    from pager_hf import _lib

    first = _setup(31, 3, 32, 8, 128, 64, 2, [9, 4, 6], [7, 64, 1], torch.bfloat16)
    second = _setup(32, 2, 14, 2, 64, 16, 3, [11, 3], [5, 16], torch.float16)
    try:
        for s, layer, atol in ((first, 1, 5e-3), (second, 2, 2e-3)):  # the test suite's bf16 / fp16 tolerances
            ref_out, ref_bm, ref_acc = _regular(s, layer)
            out, bm, acc = _noalloc(s, layer)
            np.testing.assert_allclose(out.numpy(), ref_out.numpy(), rtol=0, atol=atol)
            np.testing.assert_allclose(bm.numpy(), ref_bm.numpy(), rtol=1e-4, atol=1e-6)
            np.testing.assert_allclose(acc.numpy(), ref_acc.numpy(), rtol=1e-4, atol=1e-6)
            assert float(bm.sum()) > 0
        assert _lib.device_status(0) == 0
    finally:
        first["host"].close()
        second["host"].close()


def test_noalloc_with_an_explicit_backend_matches_regular_entry():
    """The size check follows the backend a call asks for: tensor-core and CUDA-core calls both run
    and agree with the regular entry on the same backend."""
    from pager_hf import _lib

    s = _setup(34, 2, 14, 2, 64, 16, 3, [11, 3], [5, 16], torch.float16)
    try:
        for backend in (_lib.BACKEND_MMA, _lib.BACKEND_FMA):
            ref_out, ref_bm, ref_acc = _regular(s, 1, backend)
            out, bm, acc = _noalloc(s, 1, backend)
            np.testing.assert_allclose(out.numpy(), ref_out.numpy(), rtol=0, atol=2e-3)
            np.testing.assert_allclose(bm.numpy(), ref_bm.numpy(), rtol=1e-4, atol=1e-6)
            np.testing.assert_allclose(acc.numpy(), ref_acc.numpy(), rtol=1e-4, atol=1e-6)
        assert _lib.device_status(0) == 0
    finally:
        s["host"].close()


def test_noalloc_rejects_calls_beyond_its_scratch_array():
    """64 rows x 32 heads at 65,536 tokens need more scratch than the built-in 32 MiB array holds."""
    from pager_hf import _lib

    B, Hq, Hkv, D, tpb, nb = 64, 32, 8, 128, 64, 1024
    dtype = torch.bfloat16
    s = _setup(33, 1, Hq, Hkv, D, tpb, 1, [4], [1], dtype)
    try:
        lib = _lib.lib()
        need = lib.pager_paged_decode_scratch_bytes(B, Hq, Hkv, D, _lib.DTYPE_CODE[dtype], tpb, nb, nb * tpb + 1)
        assert need > (32 << 20)
        # every row names the same four device blocks, so the buffers are valid for the claimed shape
        s.update(B=B, q=torch.randn(B, Hq, D, device="cuda").to(dtype),
                 table=torch.arange(nb, dtype=torch.int32, device="cuda").remainder(4).repeat(B, 1).contiguous(),
                 nbs=torch.full((B,), nb, dtype=torch.int32, device="cuda"),
                 tails=torch.ones(B, dtype=torch.int32, device="cuda"),
                 tk=torch.randn(B, Hkv, 1, D, device="cuda").to(dtype),
                 tv=torch.randn(B, Hkv, 1, D, device="cuda").to(dtype), max_row=nb * tpb + 1)
        out = torch.empty(B, Hq, D, dtype=dtype, device="cuda")
        bm = torch.zeros(B, Hq, nb, device="cuda")
        acc = torch.zeros(B, nb, device="cuda")
        rc = lib.pager_paged_decode_attention_noalloc(*_args(s, 0, out, bm, acc), torch.cuda.current_stream().cuda_stream)
        assert rc == _lib.PAGER_ERR_SCRATCH
        assert "scratch" in _lib.last_error()
    finally:
        s["host"].close()
