"""Request sharding across ranks: routing (as the reference's MultiGpuScheduler tests
check it, ``tests/test_multi_gpu_scheduler.py``) and the multi-rank host logic of
``bench.py --gpus N`` run as two ``gloo`` ranks on the CPU."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from pager_hf.request_shard import (RequestRouter, SessionCapacityError, aggregate_rate, local_requests,
                                    max_over_ranks, shard_requests)


def test_submit_routes_to_least_loaded_rank():
    r = RequestRouter(2)
    r.submit(weight=5)  # rank 0 busy
    assert r.submit() == 1


def test_ties_go_to_lowest_rank_and_requests_spread_evenly():
    owners = shard_requests(24, 4)
    assert owners[:4] == [0, 1, 2, 3]
    assert [owners.count(k) for k in range(4)] == [6, 6, 6, 6]
    assert local_requests(owners, 2) == [2, 6, 10, 14, 18, 22]


def test_weighted_routing_balances_tokens():
    # one long request then short ones: the short ones fill the other rank first
    owners = shard_requests(5, 2, weights=[64, 16, 16, 16, 16])
    assert owners == [0, 1, 1, 1, 1]


def test_create_session_falls_back_when_least_loaded_rank_is_full():
    r = RequestRouter(2, session_capacity=1)
    a = r.create_session()
    b = r.create_session()
    assert {r.owner(a), r.owner(b)} == {0, 1}
    with pytest.raises(SessionCapacityError):
        r.create_session()
    r.delete_session(a)
    c = r.create_session()
    assert r.owner(c) == 0


def test_session_affinity_and_unknown_session():
    r = RequestRouter(3)
    sid = r.create_session()
    for _ in range(5):
        r.submit()
    assert r.owner(sid) == 0
    with pytest.raises(KeyError):
        r.owner("nope")


def test_finish_rejects_more_than_the_load():
    r = RequestRouter(1)
    r.submit()
    r.finish(0)
    with pytest.raises(ValueError):
        r.finish(0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, batch, result_dir):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, init_method="env://")
    try:
        owners = shard_requests(world * batch, world)
        mine = local_requests(owners, rank)
        views = [None] * world
        dist.all_gather_object(views, (owners, mine))
        # every rank reaches the same routing, the shares are disjoint and cover all requests
        assert all(v[0] == owners for v in views)
        got = sorted(i for v in views for i in v[1])
        assert got == list(range(world * batch))
        assert all(len(v[1]) == batch for v in views)
        # the slowest rank's time is what every rank sees
        t = max_over_ranks(10.0 + 5.0 * rank)
        assert t == 10.0 + 5.0 * (world - 1)
        # weak scaling: whole-job rate = all ranks' units / the slowest rank's time
        units = float(len(mine))
        total = [None] * world
        dist.all_gather_object(total, units)
        rate = aggregate_rate(total, t)
        assert rate == pytest.approx(aggregate_rate(units, t, world))
        with open(os.path.join(result_dir, f"rank{rank}.ok"), "w") as f:
            f.write(f"{rate}\n")
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_shard_requests_and_reduce_time(tmp_path):
    world, batch = 2, 12
    mp.start_processes(_rank_main, args=(world, _free_port(), batch, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    rates = {open(tmp_path / f"rank{k}.ok").read() for k in range(world)}
    assert len(rates) == 1  # identical aggregate on every rank
    assert float(rates.pop()) == pytest.approx(world * batch / 15.0)


def test_max_over_ranks_without_process_group_is_identity():
    assert max_over_ranks(3.5) == 3.5
    assert torch.distributed.is_available()


def test_ranks_spread_over_the_visible_gpus():
    from pager_hf.request_shard import device_for_local_rank

    assert [device_for_local_rank(r, 4, 8) for r in range(4)] == [0, 2, 4, 6]
    assert [device_for_local_rank(r, 2, 8) for r in range(2)] == [0, 4]
    assert [device_for_local_rank(r, 8, 8) for r in range(8)] == list(range(8))
    assert [device_for_local_rank(r, 3, 8) for r in range(3)] == [0, 2, 4]
    assert device_for_local_rank(0, 1, 8) == 0
    assert [device_for_local_rank(r, 4, 4) for r in range(4)] == [0, 1, 2, 3]  # one GPU per rank: identity
