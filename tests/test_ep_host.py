"""Expert-parallel host logic on CPU: placement and the handle exchange over
gloo with two ranks (no GPU), including a rank that sends a malformed handle and
a rank that never joins (both end in an error on the other rank, not a hang)."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from nebula_b200 import ep


def test_snake_owner_balances_hot_experts():
    rng = np.random.default_rng(5)
    ranking = rng.permutation(512)
    for world in (1, 2, 4, 8):
        owner = ep.snake_owner(ranking, world)
        counts = np.bincount(owner, minlength=world)
        assert counts.tolist() == [512 // world] * world
        # the hottest 2*world experts land two per rank
        hot = np.bincount(owner[ranking[:2 * world]], minlength=world)
        assert hot.tolist() == [2] * world
        for r in range(world):
            loc, experts = ep.local_map(owner, r)
            assert len(experts) == 512 // world
            assert (loc[experts] == np.arange(len(experts))).all()
            assert (loc[owner != r] == -1).all()


def test_snake_owner_rejects_bad_input():
    with pytest.raises(ValueError):
        ep.snake_owner(np.arange(511), 2)
    with pytest.raises(ValueError):
        ep.snake_owner(np.arange(512), 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _exchange_worker(rank, world, port, results, bad_rank):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        h = bytes([rank]) * (ep.IPC_HANDLE_BYTES if rank != bad_rank else 8)
        if rank == bad_rank:  # a rank that sends a malformed handle: everyone must raise, not hang
            import torch.distributed as d
            hs = [None] * world
            d.all_gather_object(hs, h)
            results[rank] = "sent-bad"
            return
        try:
            hs = ep.exchange_handles(h, world)
            results[rank] = [x[0] for x in hs]
        except RuntimeError as e:
            results[rank] = "error:" + str(e)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("bad_rank", [-1, 1])
def test_handle_exchange_gloo(bad_rank):
    world = 2
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_exchange_worker, args=(world, _free_port(), results, bad_rank), nprocs=world,
                       start_method="spawn", join=True)
    if bad_rank < 0:
        assert [results[r] for r in range(world)] == [[0, 1], [0, 1]]
    else:
        assert results[bad_rank] == "sent-bad"
        assert str(results[0]).startswith("error:")


def _absent_worker(rank, world, port, results):
    """Rank 1 never joins the exchange; rank 0's exchange must end with an error
    within the process group's timeout instead of waiting for good."""
    import time
    from datetime import timedelta

    import torch.distributed as dist
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    try:
        if rank == 1:
            t_end = time.monotonic() + 120
            while 0 not in results and time.monotonic() < t_end:
                time.sleep(0.1)
            results[1] = "absent"
            return
        t0 = time.monotonic()
        try:
            ep.exchange_handles(bytes(ep.IPC_HANDLE_BYTES), world)
            results[0] = "returned"
        except RuntimeError as e:
            results[0] = ("error", time.monotonic() - t0, type(e).__name__)
    finally:
        dist.destroy_process_group()


def test_handle_exchange_with_an_absent_rank_times_out():
    world = 2
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_absent_worker, args=(world, _free_port(), results), nprocs=world,
                       start_method="spawn", join=True)
    assert results[1] == "absent"
    kind, waited, _ = results[0]
    assert kind == "error" and waited < 60
