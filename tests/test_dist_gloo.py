"""The N > 1 host path (shard ranges + all-gather of per-image scores) on CPU with gloo."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n_total, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import __graft_entry__ as ge
    pkg = ge.load_package()
    sh = __import__(pkg.__name__ + ".sharded", fromlist=["x"])
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    try:
        lo, hi = sh.shard_range(n_total, world, rank)
        local = torch.arange(lo, hi, dtype=torch.float32) * 0.5
        full = sh.gather_scores(local, n_total)
        q.put((rank, full.tolist()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n_total", [(2, 5), (2, 8), (3, 7)])
def test_gather_scores_unequal_shards(world, n_total):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n_total, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    expect = [0.5 * i for i in range(n_total)]
    for r in range(world):
        assert results[r] == expect


def _deadline_worker(rank, world, port, q, absent_rank):
    """Rank `absent_rank` never joins the all-gather (it stays away, then exits);
    the others must see CollectiveTimeout within their host deadline."""
    import time
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import __graft_entry__ as ge
    pkg = ge.load_package()
    sh = __import__(pkg.__name__ + ".sharded", fromlist=["x"])
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    if rank == absent_rank:
        time.sleep(3.0)
        q.put((rank, "absent", 0.0))
    else:
        lo, hi = sh.shard_range(8, world, rank)
        t0 = time.monotonic()
        try:
            sh.gather_scores(torch.arange(lo, hi, dtype=torch.float32), 8, deadline_s=1.0)
            q.put((rank, "completed", time.monotonic() - t0))
        except sh.CollectiveTimeout as e:
            q.put((rank, "timeout: " + str(e), time.monotonic() - t0))
        sh.abort_group()
    q.close()
    q.join_thread()
    os._exit(0)


@pytest.mark.parametrize("world", [2, 3])
def test_gather_deadline_detects_a_rank_that_never_joins(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_deadline_worker, args=(r, world, port, q, world - 1)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        r, what, dt = q.get(timeout=120)
        results[r] = (what, dt)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results[world - 1][0] == "absent"
    for r in range(world - 1):
        what, dt = results[r]
        assert what.startswith("timeout: all-gather of per-image scores: not completed within 1 s"), what
        assert 1.0 <= dt < 2.9, dt        # detected at the deadline, before the absent rank leaves


def _deadline_ok_worker(rank, world, port, n_total, q):
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import __graft_entry__ as ge
    pkg = ge.load_package()
    sh = __import__(pkg.__name__ + ".sharded", fromlist=["x"])
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    try:
        lo, hi = sh.shard_range(n_total, world, rank)
        full = sh.gather_scores(torch.arange(lo, hi, dtype=torch.float32), n_total, deadline_s=30.0)
        q.put((rank, full.tolist()))
    finally:
        dist.destroy_process_group()


def test_gather_with_deadline_when_every_rank_joins():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_deadline_ok_worker, args=(r, 2, port, 7, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results[0] == results[1] == [float(i) for i in range(7)]


def _score_gather_worker(rank, world, port, n_total, q):
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import __graft_entry__ as ge
    pkg = ge.load_package()
    sh = __import__(pkg.__name__ + ".sharded", fromlist=["x"])
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    try:
        g = sh.ScoreGather(n_total, torch.float32, torch.device("cpu"))
        lo, hi = sh.shard_range(n_total, world, rank)
        rounds = []
        for k in range(2):   # the same gatherer, reused: the second round overwrites the first
            work = g.start(torch.arange(lo, hi, dtype=torch.float32) + 100.0 * k)
            rounds.append(g.finish(work, deadline_s=30.0).tolist())
        q.put((rank, rounds, g.equal))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n_total", [(2, 8), (3, 7), (2, 5)])
def test_score_gather_reused_across_steps(world, n_total):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_score_gather_worker, args=(r, world, port, n_total, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        r, rounds, equal = q.get(timeout=120)
        results[r] = (rounds, equal)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        rounds, equal = results[r]
        assert equal == (n_total % world == 0)
        for k in range(2):
            assert rounds[k] == [float(i) + 100.0 * k for i in range(n_total)]
