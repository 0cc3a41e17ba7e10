"""A decode step's per-layer loop through ``PagedDecodePlan`` captured in a CUDA graph.

Every per-layer call is one ctypes call that launches on the current stream, so
a step (zero the mass accumulator, then one ``run`` per layer) can be captured
once and replayed with new queries written into the same buffers; the replay
must give the eager result bit for bit.  (The staged host tier orders its copies
with events on a second stream and is used eagerly.)
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

HOST = 0x40000000


def test_captured_step_replays_the_eager_result():
    from pager_hf.host_pool import HostPool
    from pager_hf.streaming_attention import PagedDecodePlan

    g = torch.Generator().manual_seed(21)
    L, B, Hq, Hkv, D, tpb, nb = 3, 2, 16, 4, 128, 32, 6
    dt = torch.bfloat16
    dev = torch.randn(B * nb, L, 2, Hkv, tpb, D, generator=g).to(dt).cuda()
    host = HostPool((B * nb, L, 2, Hkv, tpb, D), dt)
    host.tensor.copy_(torch.randn(host.shape, generator=g).to(dt))
    table = torch.tensor([[j if j % 2 == 0 else (j | HOST) for j in range(b * nb, (b + 1) * nb)] for b in range(B)],
                         dtype=torch.int32).cuda()
    tk = torch.randn(B, Hkv, tpb, D, generator=g).to(dt).cuda()
    tv = torch.randn(B, Hkv, tpb, D, generator=g).to(dt).cuda()
    mass = torch.zeros(B, nb, device="cuda")
    plan = PagedDecodePlan(batch=B, num_query_heads=Hq, dev_pool=dev, host_pool=host.tensor, num_layers=L,
                           tokens_per_block=tpb, block_table=table,
                           num_blocks=torch.full((B,), nb, dtype=torch.int32, device="cuda"),
                           max_row_tokens=nb * tpb + tpb, tail_k=tk, tail_v=tv,
                           tail_len=torch.tensor([5, 17], dtype=torch.int32, device="cuda"), mass_accum=mass,
                           mass_mode="row_mean", host_read="zero_copy")
    q = torch.randn(L, B, Hq, D, generator=g).to(dt).cuda()
    out = torch.empty_like(q)

    def step():
        mass.zero_()
        for layer in range(L):
            plan.run(q[layer], layer, out[layer])

    try:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            step()  # warm-up outside capture (kernel attributes, occupancy)
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        for trial in range(2):
            q.copy_(torch.randn(q.shape, generator=g).to(dt))
            step()
            torch.cuda.synchronize()
            eager_out, eager_mass = out.clone(), mass.clone()
            out.zero_()
            graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(out, eager_out), trial
            assert torch.equal(mass, eager_mass), trial
            assert float(mass.sum()) > 0
    finally:
        host.close()
