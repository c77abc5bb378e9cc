"""Stream, thread and graph use of the library: calls on two streams at once, calls from
several host threads at once, and a call captured in a CUDA graph and replayed with new
inputs (the per-image counters in the workspace reset themselves, so every replay starts
from a zeroed workspace)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _syn(pkg):
    return __import__(pkg.__name__ + ".synthetic", fromlist=["x"])


def test_two_streams_at_once_match_one_stream(pkg):
    syn = _syn(pkg)
    shape = (3, 300, 260, 6)
    pairs = [syn.device_pair(shape, 0.1, seed=s) for s in (1, 2)]
    ref = [pkg.dssim_with_gradient(x, y, True) for x, y in pairs]
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    outs = [None, None]
    for _ in range(3):
        for i, ((x, y), st) in enumerate(zip(pairs, streams)):
            st.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(st):
                outs[i] = pkg.dssim_with_gradient(x, y, True)
        torch.cuda.synchronize()
        for (v, g), (rv, rg) in zip(outs, ref):
            assert torch.equal(v, rv) and torch.equal(g, rg)   # deterministic: bitwise equal


def test_captured_call_replays_with_new_inputs(pkg, orc):
    syn = _syn(pkg)
    shape = (3, 120, 100, 4)
    x = pkg.jl_empty(shape, torch.float32)
    y = pkg.jl_empty(shape, torch.float32)
    s = torch.empty(4, dtype=torch.float32, device="cuda")
    g = pkg.jl_empty(shape, torch.float32)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):               # warm-up on the capture stream: kernel attributes, workspace
        pkg.ssim_with_gradient_(s, g, x.zero_(), y.zero_(), None, True)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        pkg.ssim_with_gradient_(s, g, x, y, None, True)
    for seed in (3, 4, 5):
        hx, hy = syn.host_pair(seed, shape, 0.1)
        x.copy_(pkg.jl_from_numpy(hx))
        y.copy_(pkg.jl_from_numpy(hy))
        graph.replay()
        torch.cuda.synchronize()
        rv, rg = orc.ssim(hx, hy, precision="f32")
        assert np.max(np.abs(s.double().cpu().numpy() - rv)) <= 1e-5
        gv = pkg.jl_to_numpy(g).astype(np.float64)
        assert np.linalg.norm(gv - rg) / np.linalg.norm(rg) <= 1e-4
    del graph


def test_host_threads_call_at_once(pkg):
    """Four host threads call the library at the same time (ctypes releases the GIL for
    the call), each on its own stream with its own outputs and workspace, while a fifth
    makes calls that the library refuses.  Every result is bitwise the one-thread result,
    and each thread reads only its own errors: the error channel is per thread."""
    import threading
    nat = pkg._native
    syn = _syn(pkg)
    shape = (3, 200, 180, 5)
    pairs = [syn.device_pair(shape, 0.1, seed=20 + i) for i in range(4)]
    ref = [pkg.dssim_with_gradient(x, y, True) for x, y in pairs]
    torch.cuda.synchronize()
    results, failures = [None] * 4, []
    start = threading.Barrier(5)

    def good(i):
        try:
            st = torch.cuda.Stream()
            x, y = pairs[i]
            start.wait()
            outs = []
            for _ in range(25):
                with torch.cuda.stream(st):
                    outs.append(pkg.dssim_with_gradient(x, y, True))
            st.synchronize()
            results[i] = outs
        except Exception as e:   # reported below, in the main thread
            failures.append(repr(e))

    def bad():
        try:
            start.wait()
            for k in range(200):
                with pytest.raises(nat.FastSSIMError, match="sizes must be positive"):
                    nat.fwd_bwd(0, 0, 1, 0, 0, 0, 0, 0, 0, 0, 0, 8, 8, 1, nat.SHOULD_ZERO, 0, 0, 0)
        except Exception as e:
            failures.append(repr(e))

    threads = [threading.Thread(target=good, args=(i,)) for i in range(4)] + [threading.Thread(target=bad)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=120)
    assert not any(t.is_alive() for t in threads)
    assert not failures, failures
    for outs, (rv, rg) in zip(results, ref):
        for v, g in outs:
            assert torch.equal(v, rv) and torch.equal(g, rg)
    assert nat.last_error()[0] == nat.OK   # this thread made no failing call
