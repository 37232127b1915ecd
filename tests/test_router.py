"""Session placement across GPUs (host logic, CPU): the least-loaded rule,
page accounting, agreement of all ranks under world_size 2 over gloo, and a
rank that dies being detected by the others through a host collective timeout
(no GPU involved)."""
import datetime
import os
import socket

import pytest
import torch.multiprocessing as mp

from orator_b200.router import SessionRouter


def test_least_loaded_with_room():
    r = SessionRouter(world=3, pages_per_rank=10)
    assert r.place(0, 100) == 0      # 7 pages on rank 0
    assert r.place(1, 20) == 1
    assert r.place(2, 20) == 2
    assert r.place(3, 10) == 1       # ranks 1 and 2 tie at 20 tokens: lowest rank
    assert r.loads() == [100, 30, 20]
    # rank 2 is least loaded but a 200-token session needs 13 pages: nobody has them
    with pytest.raises(RuntimeError):
        r.place(4, 200)
    # 9 pages: only rank 2 (8 free) cannot, rank 1 (7 free) cannot, rank 0 (3) cannot
    with pytest.raises(RuntimeError):
        r.place(5, 130)
    r.release(0)
    assert r.place(5, 130) == 0
    assert r.sessions_on(0) == [5]


def test_grow_takes_pages():
    r = SessionRouter(world=1, pages_per_rank=4, page=16)
    r.place(7, 16)
    assert r.ranks[0].free_pages == 3
    r.grow(7)          # 17 tokens -> second page
    assert r.ranks[0].free_pages == 2 and r.loads() == [17]
    r.release(7)
    assert r.ranks[0].free_pages == 4 and r.loads() == [0]


def test_grow_without_pages_raises_and_keeps_state():
    r = SessionRouter(world=1, pages_per_rank=2, page=16)
    r.place(1, 32)                 # both pages
    with pytest.raises(RuntimeError):
        r.grow(1)
    assert r.ranks[0].free_pages == 0 and r.lens[1] == 32 and r.loads() == [32]


def _release_worker(rank, world, port, q):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=30))
    r = SessionRouter(world, pages_per_rank=100, page=16)
    a, b = r.place(10, 64), r.place(11, 64)       # one session per rank
    # each rank's session really holds 20 tokens (it was truncated): report it
    mine = 10 if rank == a else 11
    r.gather_loads(rank, kv_tokens=20, free_pages=100 - 2, lens={mine: 20})
    r.release(10)
    r.release(11)
    q.put((rank, r.loads(), [ld.free_pages for ld in r.ranks], a, b))
    dist.destroy_process_group()


def test_gather_loads_then_release_is_consistent():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_release_worker, args=(i, 2, port, q)) for i in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in ps]
    for p in ps:
        p.join(timeout=60)
    for rank, loads, free, a, b in res:
        assert (a, b) == (0, 1)
        assert loads == [0, 0]          # the reported 20 tokens come back, not the modelled 64
        assert free == [100, 100]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _agree_worker(rank, world, port, q):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=30))
    r = SessionRouter(world, pages_per_rank=1000)
    # each rank reports a different measured load; placements follow the reports
    r.gather_loads(rank, kv_tokens=[5000, 100][rank], free_pages=1000)
    placed = [r.place(s, 300) for s in range(6)]
    got = [None] * world
    dist.all_gather_object(got, placed)
    q.put((rank, placed, got[0] == got[1]))
    dist.destroy_process_group()


def test_ranks_agree_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_agree_worker, args=(i, 2, port, q)) for i in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in ps]
    for p in ps:
        p.join(timeout=60)
    for rank, placed, same in res:
        assert same
        # rank 1 reported 100 tokens vs 5000: it takes new sessions until it catches up
        assert placed[:6] == [1] * 6


def _dying_worker(rank, world, port, q):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)  # leaves between steps, before the next load exchange
    r = SessionRouter(world, pages_per_rank=100)
    try:
        r.gather_loads(rank, 0, 100)
        q.put("no error")
    except Exception as e:  # timeout or closed connection
        q.put(type(e).__name__)


def test_dead_rank_detected_by_timeout():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_dying_worker, args=(i, 2, port, q)) for i in range(2)]
    for p in ps:
        p.start()
    msg = q.get(timeout=120)
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert msg != "no error"
