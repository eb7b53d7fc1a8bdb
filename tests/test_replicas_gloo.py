"""Multi-rank host logic of the replica decode (``rwkv_b200.replicas``) with two
``gloo`` ranks on the CPU: session split, per-session seeds, max-over-ranks
timing, rank-ordered gathers, and a rank that fails before a collective."""

from __future__ import annotations

import datetime
import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from rwkv_b200 import replicas


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank: int, world: int, port: int, timeout_s: float = 30.0) -> None:
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _worker_logic(rank: int, world: int, port: int, q) -> None:
    sys.path[:0] = [p for p in os.environ.get("RWKVB_TEST_PATH", "").split(os.pathsep) if p]
    try:
        _init(rank, world, port)
        r, w = replicas.world()
        sess = replicas.session_range(3, r, w)
        seeds = [replicas.session_seed(2026, s) for s in sess]
        # a fake per-rank step time: the job time is the slowest rank's
        t = replicas.max_over_ranks(1.5 + r)
        ids = replicas.gather_ranks(list(sess))
        uneven = replicas.gather_ranks(list(range(r + 1)))
        q.put((r, w, list(sess), seeds, t, ids, uneven))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported through the queue
        q.put(("error", rank, repr(e)))


def _worker_fail(rank: int, world: int, port: int, q) -> None:
    sys.path[:0] = [p for p in os.environ.get("RWKVB_TEST_PATH", "").split(os.pathsep) if p]
    store = dist.TCPStore("127.0.0.1", port, world, is_master=rank == 0, timeout=datetime.timedelta(seconds=30))
    # step 0: everyone present
    q.put((rank, 0, replicas.missing_peers(store, 0, rank, world, timeout_s=10.0)))
    if rank == 1:
        q.close()
        q.join_thread()  # flush the queued message before leaving
        os._exit(0)  # this rank leaves between steps, with nothing in flight
    # step 1: the survivor sees the missing rank on the host before any collective
    q.put((rank, 1, replicas.missing_peers(store, 1, rank, world, timeout_s=1.0)))


def _spawn(target, world: int):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    os.environ["RWKVB_TEST_PATH"] = os.pathsep.join(sys.path)
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():  # pragma: no cover
            p.kill()
    return out


def test_session_split_and_seeds_single_process():
    assert list(replicas.session_range(4, 0, 1)) == [0, 1, 2, 3]
    blocks = [list(replicas.session_range(4, r, 3)) for r in range(3)]
    assert sum(blocks, []) == list(range(12))
    assert replicas.session_seed(1, 5) == replicas.session_seed(1, 5)
    assert replicas.session_seed(1, 5) != replicas.session_seed(1, 6)
    with pytest.raises(ValueError):
        replicas.session_range(2, 3, 3)
    assert replicas.max_over_ranks(2.5) == 2.5
    assert replicas.gather_ranks([1, 2]) == [[1, 2]]


def test_two_gloo_ranks_split_time_and_gather():
    out = _spawn(_worker_logic, 2)
    assert not any(o[0] == "error" for o in out), out
    by_rank = {o[0]: o for o in out}
    for r in (0, 1):
        _, w, sess, seeds, t, ids, uneven = by_rank[r]
        assert w == 2
        assert sess == [3 * r, 3 * r + 1, 3 * r + 2]
        assert seeds == [replicas.session_seed(2026, s) for s in sess]
        assert t == 2.5  # max over ranks of 1.5 + rank
        assert ids == [[0, 1, 2], [3, 4, 5]]  # every session exactly once, in rank order
        assert uneven == [[0], [0, 1]]


def test_rank_leaving_is_seen_through_the_store_heartbeat():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    os.environ["RWKVB_TEST_PATH"] = os.pathsep.join(sys.path)
    procs = [ctx.Process(target=_worker_fail, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(3):  # rank 0: steps 0 and 1; rank 1: step 0 only
        r, step, miss = q.get(timeout=60)
        got[(r, step)] = miss
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():  # pragma: no cover
            p.kill()
    assert got[(0, 0)] == [] and got[(1, 0)] == []
    assert got[(0, 1)] == [1]
