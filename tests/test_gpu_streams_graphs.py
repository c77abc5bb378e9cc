"""Stream and graph use of the library: calls on two streams at once, and a call
captured in a CUDA graph and replayed with new inputs (the per-image counters in
the workspace reset themselves, so every replay starts from a zeroed workspace)."""
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
