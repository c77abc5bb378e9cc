"""The C ABI from a plain C program (tests/c_client/fssim_client.c): built with gcc
against include/fastssim.h and libfastssim.so, it allocates with the CUDA runtime
and calls fssim_fwd_bwd as the Julia ccall shim would.  Its outputs are checked
against the oracle."""
import os
import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


@pytest.fixture(scope="module")
def client(tmp_path_factory):
    out = str(tmp_path_factory.mktemp("c_client") / "fssim_client")
    lib_dir = os.path.join(ROOT, "fastcudassim.jl_b200", "lib")
    cmd = ["gcc", "-O2", "-std=c11", "-o", out, os.path.join(ROOT, "tests", "c_client", "fssim_client.c"),
           "-I", os.path.join(ROOT, "include"), "-I", os.path.join(CUDA, "include"),
           "-L", lib_dir, "-lfastssim", "-L", os.path.join(CUDA, "lib64"), "-lcudart", "-Wl,-rpath," + lib_dir]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return out


@pytest.mark.parametrize("flags", [0, 4 | 8])   # SSIM + gradient; DSSIM/2 + gradient
def test_c_client_matches_the_oracle(client, pkg, orc, tmp_path, flags):
    shape = (3, 70, 53, 2)
    x, y = __import__(pkg.__name__ + ".synthetic", fromlist=["x"]).host_pair(21, shape, 0.1)
    xf, yf = tmp_path / "x.bin", tmp_path / "y.bin"
    sf, gf = tmp_path / "s.bin", tmp_path / "g.bin"
    x.ravel(order="F").astype(np.float32).tofile(xf)
    y.ravel(order="F").astype(np.float32).tofile(yf)
    r = subprocess.run([client, *map(str, shape), str(flags), str(xf), str(yf), str(sf), str(gf)],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "fastssim" in r.stdout and r.stdout.strip().endswith("ok")
    s = np.fromfile(sf, dtype=np.float32).astype(np.float64)
    g = np.fromfile(gf, dtype=np.float32).reshape(shape, order="F").astype(np.float64)
    rs, rg = orc.ssim(x, y, flags=flags, precision="f32")
    assert np.max(np.abs(s - rs)) <= 1e-5
    assert np.linalg.norm(g - rg) / np.linalg.norm(rg) <= 1e-4


@pytest.mark.parametrize("channels", [1, 3])
def test_c_abi_call_cost(channels):
    """The per-call cost program builds and runs: SSIM of two zero images is 1, and one call
    with the read of its value takes longer on the host than the call alone."""
    import json
    import sys
    sys.path.insert(0, ROOT)
    import bench
    r = bench.c_abi_call_cost(channels)
    assert abs(r["ssim_of_zero_images"] - 1.0) < 1e-6
    assert 0 < r["enqueue_us"] < r["roundtrip_us"]
    assert r["device_us"] > 0
    print(json.dumps(r))
