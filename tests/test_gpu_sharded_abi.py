"""The multi-GPU C ABI on two GPUs: fssim_comm_*, fssim_fwd_bwd_sharded, fssim_comm_wait.

Two child processes, one per GPU, build an NCCL communicator through the library
(rank 0 makes the unique id and passes it on), run their shard of a batch through
fssim_fwd_bwd_sharded and wait with fssim_comm_wait.  Every rank must end with the
full vector of per-image values, equal to the oracle's, and its own gradient slice,
for unequal shards (5 images, gathered through padded buffers) and equal shards (6,
gathered in place).  Then rank 1 leaves between steps (its work finished, the process
exits); rank 0's next gather cannot finish, so fssim_comm_wait must end it by the
deadline with CommTimeout or a communicator error, after aborting the communicator.
NVLS stays off.  Skipped with fewer than two GPUs.
"""
import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")]


def _worker(rank, q_id, q_out, left):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import sys
    import time
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    sys.path.insert(0, os.path.join(root, "oracle"))
    import __graft_entry__ as ge
    import oracle
    pkg = ge.load_package()
    nat = pkg._native
    syn = __import__(pkg.__name__ + ".synthetic", fromlist=["x"])
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    stream = torch.cuda.current_stream(dev).cuda_stream
    if rank == 0:
        uid = nat.comm_unique_id()
        q_id.put(uid)
    else:
        uid = q_id.get(timeout=60)
    comm = nat.comm_init(2, rank, uid, deadline_s=60.0)

    def run(n_total, seed, deadline_s=30.0):
        xa, ya = syn.host_pair(seed, (3, 40, 36, n_total), 0.1)
        base, rem = divmod(n_total, 2)
        lo = rank * base + min(rank, rem)
        cnt = base + (1 if rank < rem else 0)
        xs = pkg.jl_from_numpy(np.asfortranarray(xa[..., lo:lo + cnt]))
        ys = pkg.jl_from_numpy(np.asfortranarray(ya[..., lo:lo + cnt]))
        g = pkg.jl_empty((3, 40, 36, cnt), torch.float32)
        out = torch.zeros(n_total, dtype=torch.float32, device=dev)
        flags = nat.SHOULD_ZERO
        wsb = nat.sharded_workspace_size(3, 40, 36, n_total, 2, rank, flags, nat.FLOAT32)
        ws = torch.zeros(max(wsb, 1), dtype=torch.uint8, device=dev)
        nat.fwd_bwd_sharded(out.data_ptr(), nat.FLOAT32, n_total, g.data_ptr(), nat.FLOAT32, xs.data_ptr(),
                            nat.FLOAT32, ys.data_ptr(), nat.FLOAT32, 3, 40, 36, cnt, flags, comm, 2, rank,
                            ws.data_ptr(), wsb, stream)
        nat.comm_wait(comm, stream, deadline_s)
        rv, rg = oracle.ssim(xa, ya, precision="f64")
        err_v = float(np.max(np.abs(out.double().cpu().numpy() - rv)))
        gl = pkg.jl_to_numpy(g).astype(np.float64)
        rl = rg[..., lo:lo + cnt]
        err_g = float(np.linalg.norm(gl - rl) / np.linalg.norm(rl))
        return err_v, err_g

    for n_total, seed in ((5, 81), (6, 82)):
        q_out.put((rank, f"n{n_total}", run(n_total, seed)))
    if rank == 1:
        left.set()
        q_out.close()
        q_out.join_thread()
        os._exit(0)                      # leaves between steps, nothing in flight
    left.wait(timeout=60)
    time.sleep(1.0)
    t0 = time.monotonic()
    try:
        run(6, 83, deadline_s=3.0)
        q_out.put((rank, "completed", time.monotonic() - t0))
    except nat.CommTimeout as e:
        q_out.put((rank, "timeout: " + str(e), time.monotonic() - t0))
    except nat.FastSSIMError as e:
        q_out.put((rank, "comm error: " + str(e), time.monotonic() - t0))
    q_out.close()
    q_out.join_thread()
    os._exit(0)


def test_sharded_entry_gathers_every_image_and_a_leaving_rank_is_detected():
    ctx = mp.get_context("spawn")
    q_id, q_out, left = ctx.Queue(), ctx.Queue(), ctx.Event()
    procs = [ctx.Process(target=_worker, args=(r, q_id, q_out, left)) for r in range(2)]
    for p in procs:
        p.start()
    msgs = []
    try:
        for _ in range(5):
            msgs.append(q_out.get(timeout=240))
    finally:
        for p in procs:
            p.join(timeout=90)
            if p.is_alive():
                p.kill()
                p.join(timeout=30)
    for r, what, v in msgs:
        if what in ("n5", "n6"):
            err_v, err_g = v
            assert err_v <= 1e-5, (r, what, err_v)
            assert err_g <= 1e-4, (r, what, err_g)
    last = [(what, v) for r, what, v in msgs if r == 0 and what not in ("n5", "n6")]
    assert len(last) == 1
    what, dt = last[0]
    assert what.startswith("timeout:") or what.startswith("comm error:"), what
    assert dt < 15.0, dt
    for p in procs:
        assert p.exitcode == 0
