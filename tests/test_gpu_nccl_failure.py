"""A rank that leaves between steps, on two GPUs over NCCL.

Two child processes, one per GPU, run a sharded SSIM + gradient step (the kernel on
their own shard, then the NCCL all-gather of the per-image scores).  After the first
step rank 1 leaves: it waits for its own work, destroys its process group and exits,
with no kernel or collective in flight.  Rank 0 then runs the next step.  Its
all-gather can never complete, so ``gather_scores(..., deadline_s=1)`` must raise
``CollectiveTimeout`` at the deadline; ``abort_group`` then aborts the communicator
(ncclCommAbort) and the process exits 0.  NVLS is off (NCCL_NVLS_ENABLE=0), as for
every test where a rank leaves.  Skipped on machines with fewer than two GPUs.
"""
import os
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, q, left):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import sys
    from datetime import timedelta
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import torch.distributed as dist
    import __graft_entry__ as ge
    pkg = ge.load_package()
    sh = __import__(pkg.__name__ + ".sharded", fromlist=["x"])
    syn = __import__(pkg.__name__ + ".synthetic", fromlist=["x"])
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=2, timeout=timedelta(seconds=30), device_id=dev)
    n_total = 6
    lo, hi = sh.shard_range(n_total, 2, rank)
    x, y = syn.device_pair((3, 64, 48, hi - lo), 0.1, seed=50 + rank, device=dev)

    # step 1: both ranks
    scores, _ = sh.sharded_with_gradient(x, y, n_total, deadline_s=20.0)
    torch.cuda.synchronize(dev)
    q.put((rank, "step1", scores.cpu().tolist()))
    if rank == 1:
        dist.destroy_process_group()   # nothing in flight: the step above is complete
        left.set()
        q.close()
        q.join_thread()
        os._exit(0)

    # step 2: rank 0 alone, after rank 1 has gone
    left.wait(timeout=60)
    t0 = time.monotonic()
    try:
        sh.sharded_with_gradient(x, y, n_total, deadline_s=1.0)
        q.put((rank, "completed", time.monotonic() - t0))
    except sh.CollectiveTimeout as e:
        q.put((rank, "timeout: " + str(e), time.monotonic() - t0))
    sh.abort_group()
    q.put((rank, "aborted", time.monotonic() - t0))
    q.close()
    q.join_thread()
    os._exit(0)


def test_rank_leaving_between_steps_is_detected_and_the_communicator_aborted():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    left = ctx.Event()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q, left)) for r in range(2)]
    for p in procs:
        p.start()
    msgs = []
    try:
        for _ in range(4):
            msgs.append(q.get(timeout=180))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():   # never expected; a child that outlives the test is ended here
                p.kill()
                p.join(timeout=30)
    step1 = {r: v for r, what, v in msgs if what == "step1"}
    assert step1[0] == step1[1] and len(step1[0]) == 6     # the all-gather worked while both ranks ran
    rank0 = [(what, v) for r, what, v in msgs if r == 0 and what != "step1"]
    assert rank0[0][0].startswith("timeout: all-gather of per-image scores: not completed within 1 s"), rank0
    assert 1.0 <= rank0[0][1] < 5.0, rank0
    assert rank0[1][0] == "aborted"
    for p in procs:
        assert p.exitcode == 0
