"""The bounds-checked build (libfastssim_bounds.so, -DFSSIM_DEBUG_BOUNDS) on every kernel path.

There every global access checks its element index against the array first and
records a failure instead of making the access; compute-sanitizer is not
available, so this is the memory check.  A child process loads the library and
runs tiny, odd and batch shapes through each kernel (fused SSIM + gradient,
gradient with a per-image factor, forward tiles (plain and TMA loads) and streaming, converted and
Float64 inputs, the no-alloc entry point): no access may be out of range, and
the values must equal the regular build's.
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_DIR = os.path.join(ROOT, "fastcudassim.jl_b200", "lib")

CHILD = r"""
import json, sys
import numpy as np, torch
sys.path.insert(0, ROOT)
import __graft_entry__ as ge
pkg = ge.load_package()
nat = pkg._native
syn = __import__(pkg.__name__ + ".synthetic", fromlist=["x"])
if CHECKED:
    assert "bounds-checked" in nat.version(), nat.version()
    nat.debug_bounds_status(reset=True)
out = {}
cases = [((1, 1, 1, 2), "f32"), ((1, 37, 5, 1), "f32"), ((3, 1023, 767, 1), "f32"), ((2, 57, 33, 3), "u8"),
         ((4, 40, 129, 2), "f16"), ((3, 53, 41, 2), "f64"), ((3, 1100, 1400, 1), "f32"), ((5, 31, 20, 1), "f32"),
         ((1, 64, 70, 2), "f32")]   # one channel, height divisible by 4: the TMA tile loads
for shape, dt in cases:
    x, y = syn.host_pair(3, shape, 0.1, dtype=np.uint8 if dt == "u8" else np.float64)
    if dt != "u8":
        npdt = {"f32": np.float32, "f16": np.float16, "f64": np.float64}[dt]
        x, y = np.asfortranarray(x.astype(npdt)), np.asfortranarray(y.astype(npdt))
    xt, yt = pkg.jl_from_numpy(x), pkg.jl_from_numpy(y)
    vals, grad = pkg.dssim_with_gradient(xt, yt, True)
    fwd = pkg.ssim(xt, yt)
    gs = torch.linspace(-1, 1, shape[3], device="cuda")
    _, gsc = pkg.ssim_fwd_bwd(None, None, xt, yt, None, False, True, False, False, False, grad_scale=gs)
    s_na = torch.empty(shape[3], dtype=torch.float32, device="cuda")
    nat.fwd_bwd_noalloc(s_na.data_ptr(), nat.FLOAT32, shape[3], 0, nat.FLOAT32, xt.data_ptr(),
                        pkg.core.dtype_code(xt), yt.data_ptr(), pkg.core.dtype_code(yt),
                        *shape, nat.SKIP_BACKWARD | nat.SHOULD_ZERO, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    site, count = nat.debug_bounds_status(reset=True) if CHECKED else (0, 0)
    out[f"{shape}-{dt}"] = {
        "site": site, "count": count,
        "vals": torch.as_tensor(vals).double().cpu().reshape(-1).tolist(),
        "fwd": torch.as_tensor(fwd).double().cpu().reshape(-1).tolist(),
        "noalloc": s_na.double().cpu().tolist(),
        "grad": [float(grad.double().norm()), float(grad.double().sum())],
        "scaled": [float(gsc.double().norm()), float(gsc.double().sum())]}
print("RESULT " + json.dumps(out))
"""


def _run(lib, checked):
    env = dict(os.environ, FASTSSIM_LIB=lib)
    code = "ROOT = %r\nCHECKED = %r\n" % (ROOT, checked) + CHILD
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-3000:]
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("RESULT ")][-1]
    return json.loads(line[len("RESULT "):])


@pytest.fixture(scope="module")
def runs(pkg):
    lib = os.path.join(LIB_DIR, "libfastssim_bounds.so")
    if not os.path.exists(lib):
        pytest.fail("bounds-checked library not built (__graft_entry__.build())")
    return _run(lib, True), _run(os.path.join(LIB_DIR, "libfastssim.so"), False)


def test_no_out_of_range_access_on_any_kernel_path(runs):
    checked, _ = runs
    for case, r in checked.items():
        assert r["site"] == 0 and r["count"] == 0, (case, r["site"], r["count"])


def test_bounds_checked_build_computes_the_same_values(runs):
    checked, regular = runs
    assert checked.keys() == regular.keys()
    for case in checked:
        a, b = checked[case], regular[case]
        for key in ("vals", "fwd", "noalloc", "grad", "scaled"):
            np.testing.assert_allclose(a[key], b[key], rtol=1e-6, atol=1e-9, err_msg=f"{case} {key}")
        np.testing.assert_allclose(a["vals"], (1.0 - np.asarray(a["fwd"])) / 2, atol=1e-5, err_msg=case)
