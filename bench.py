"""Benchmark: SSIM + gradient throughput (Gpixel/s, % of HBM roofline) at 1/2/4/8 B200s,
plus the full-HD SSIM latency.

Workload (one step): 2048 images x 3 x 512 x 512 Float32 (x ~ U[0,1),
y = clamp(x + N(0, 0.1^2), 0, 1)), SSIM values and dSSIM/dx for every image;
the batch is split evenly over the N ranks (strong scaling, one process per
GPU) and the 2048 per-image SSIMs are all-gathered over NCCL.  Inputs are
12.9 GB, far larger than L2, so no flush is needed between steps.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

For N > 1 launch with torch.distributed.run (one rank per GPU).  Rank 0 prints
one JSON line.  ``--impl reference`` times the reference algorithm's CPU
restatement (the oracle; FastCUDASSIM.jl itself needs Julia, which is absent)
on the host cores, on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

N_IMAGES, C, H, W = 2048, 3, 512, 512
NOISE = 0.1
BYTES_PER_ELEM = 4 + 4 + 4      # x, y read; gradient written (Float32)
WORKLOAD = "ssim_with_gradient 2048x3x512x512 f32, batch-sharded, NCCL all-gather of per-image SSIM"


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def traffic_per_launch(n_local):
    """DRAM bytes per launch from the committed ncu summary (bytes per element x elements), or None."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            d = json.load(f)
        return float(d["dram_bytes_per_elem"]) * n_local * C * H * W
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sms, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            p = [s.strip() for s in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sms.append(float(p[1]))
                maxes.append(float(p[2]))
            except ValueError:
                continue
            for nm, v in zip(names, p[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sms) if sms else None, "sm_max_mhz": max(maxes) if maxes else None,
                "reasons": sorted(reasons), "samples": len(sms)}


# FP32 FMA-equivalents per element of the fused kernel, counted with ncu
# (sass__inst_executed_per_opcode: FFMA2/FADD2/FMUL2 count 2, FFMA/FADD/FMUL 1).
FMA_PER_ELEM = 221
# The forward pass alone: the 4-moment h- and w-passes (2 x 44), the products and the map.
FWD_FMA_PER_ELEM = 106


def fp32_frac(fma_per_elem, elems, ms, sms):
    """FP32-pipe fraction of a timed call: FMA-equivalents per second against 128 lanes per SM
    per clock at the maximum SM clock (the clock the side calls run at, not sampled for them)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            mhz = float(json.load(f)["sm_max_mhz"])
    except Exception:
        mhz = 1965.0
    return fma_per_elem * elems / (ms / 1e3) / (sms * 128 * mhz * 1e6)


def fp32_pipe(kern_s, n_local, clocks, sms):
    """The binding roof of the fused kernel: FP32 FMA pipe use against 128 lanes per SM
    per clock at the SM clock sampled during the timed region."""
    mhz = clocks.get("sm_mhz") or clocks.get("sm_max_mhz")
    if not mhz:
        return None
    achieved = FMA_PER_ELEM * n_local * C * H * W / kern_s / 1e12
    peak = sms * 128 * mhz * 1e6 / 1e12
    return {"fma_per_elem": FMA_PER_ELEM, "achieved_tfma_s": achieved, "peak_tfma_s": peak,
            "frac": achieved / peak, "clock_mhz": mhz}


def cpu_fullhd_ms(channels, reps=3):
    """The oracle's forward SSIM on one full-HD pair (ms, best of `reps`).  The oracle
    parallelises over (image, channel) planes, so it uses `channels` host threads."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    import __graft_entry__ as ge
    syn = __import__(ge.load_package().__name__ + ".synthetic", fromlist=["x"])
    x, y = syn.host_pair(7, (channels, 1080, 1920, 1), NOISE)
    best = None
    for _ in range(reps):
        t0 = time.perf_counter()
        oracle.ssim(x, y, flags=oracle.SKIP_BACKWARD, nthreads=channels)
        dt = (time.perf_counter() - t0) * 1e3
        best = dt if best is None else min(best, dt)
    return best


def cpu_batch32_dssim_grad_ms(nthreads, reps=2):
    """The oracle's DSSIM + gradient on the 32x3x256x256 batch (ms, best of `reps`) with
    `nthreads` host threads (it parallelises over the 96 channel planes)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    import __graft_entry__ as ge
    syn = __import__(ge.load_package().__name__ + ".synthetic", fromlist=["x"])
    x, y = syn.host_pair(11, (3, 256, 256, 32), None)
    best = None
    for _ in range(reps):
        t0 = time.perf_counter()
        oracle.ssim(x, y, flags=oracle.USE_DSSIM, nthreads=nthreads)
        dt = (time.perf_counter() - t0) * 1e3
        best = dt if best is None else min(best, dt)
    return best


def parity_sample(pkg, x, y, ssims, grad, first_image, seed):
    """Checks the benchmark batch itself, after the timed region: the first and last image
    of this rank's shard plus four seeded picks, each against the oracle in single and in
    double precision.  Returns the largest |delta (D)SSIM| and the largest relative-L2
    gradient error over the sampled images and both oracle modes."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    n = int(ssims.numel())
    rng = np.random.default_rng(seed)
    picks = sorted({0, n - 1} | {int(i) for i in rng.choice(n, size=min(4, n), replace=False)})
    max_ds, max_rel = 0.0, 0.0
    vals = ssims.double().cpu().numpy()
    for i in picks:
        xi, yi = pkg.jl_to_numpy(x[..., i:i + 1]), pkg.jl_to_numpy(y[..., i:i + 1])
        gi = pkg.jl_to_numpy(grad[..., i:i + 1]).astype(np.float64)
        for prec in ("f32", "f64"):
            rv, rg = oracle.ssim(xi, yi, precision=prec)
            max_ds = max(max_ds, abs(float(vals[i]) - float(rv[0])))
            max_rel = max(max_rel, float(np.linalg.norm(gi - rg) / max(np.linalg.norm(rg), 1e-30)))
    return {"images": [first_image + i for i in picks], "max_abs_ssim_err": max_ds,
            "max_rel_l2_grad_err": max_rel, "oracle": "f32 and f64 modes",
            "tolerance": {"ssim_abs": 1e-5, "grad_rel_l2": 1e-4}}


class CpuSample:
    """A sample of the workload on the host (seeded, same distributions) and the
    oracle (the reference algorithm in single precision, C with pthreads)."""

    def __init__(self, n_images, nthreads):
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle
        import __graft_entry__ as ge
        syn = __import__(ge.load_package().__name__ + ".synthetic", fromlist=["x"])
        self.oracle, self.n, self.threads = oracle, n_images, nthreads
        self.x, self.y = syn.host_pair(99, (C, H, W, n_images), NOISE)
        oracle.ssim(self.x[..., :1], self.y[..., :1], nthreads=nthreads)   # warm the library

    def one_pass(self):
        """Seconds for SSIM + gradient of the whole sample."""
        t0 = time.perf_counter()
        self.oracle.ssim(self.x, self.y, nthreads=self.threads)
        return time.perf_counter() - t0

    def rate(self, min_seconds):
        """Gpixel/s over as many passes as fill `min_seconds` of CPU time."""
        passes, spent = 0, 0.0
        while spent < min_seconds or passes == 0:
            spent += self.one_pass()
            passes += 1
        return passes * self.n * H * W / spent / 1e9, passes, spent


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    # about one second of work per step: 10 images per host thread (an image with its
    # gradient takes the oracle about 0.1 s on one core), at most 256 (2.4 GB of host memory)
    sample = max(4, min(256, 10 * threads))
    cs = CpuSample(sample, threads)
    for _ in range(args.warmup):
        cs.one_pass()
    times = [cs.one_pass() for _ in range(args.steps)]
    t = sum(times)
    value = args.steps * sample * H * W / t / 1e9
    line = {
        "impl": "reference", "metric": "SSIM+grad Gpixel/s", "value": value, "unit": "Gpixel/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * t / args.steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "sample_images_per_step": sample},
        "cpu_baseline": {"value": value, "unit": "Gpixel/s", "cores": threads, "kind": "port",
                         "sample": f"{sample} images of 3x512x512 with gradient per step (the oracle: "
                                   "FastCUDASSIM.jl's algorithm restated in C; Julia is not available)"},
        "e2e": {"value": value, "unit": "Gpixel/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def bind_to_gpu_numa_node(dev_index):
    """Restricts this process to the host CPUs of its GPU's NUMA node (read from sysfs), so
    that pinned host buffers allocated afterwards sit in that node's memory.  Returns the
    node, or None where the topology is not exposed (one node, or no sysfs entry)."""
    try:
        import torch
        pr = torch.cuda.get_device_properties(dev_index)
        bus = f"{pr.pci_domain_id:04x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
        with open(f"/sys/bus/pci/devices/{bus}/numa_node") as f:
            node = int(f.read().strip())
        if node < 0:
            return None
        with open(f"/sys/devices/system/node/node{node}/cpulist") as f:
            cpus = set()
            for part in f.read().strip().split(","):
                lo_, _, hi_ = part.partition("-")
                cpus.update(range(int(lo_), int(hi_ or lo_) + 1))
        os.sched_setaffinity(0, cpus)
        return node
    except Exception:
        return None


def run_ours(args):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import __graft_entry__ as ge
    pkg = ge.load_package()
    syn = __import__(pkg.__name__ + ".synthetic", fromlist=["x"])
    sharded = __import__(pkg.__name__ + ".sharded", fromlist=["x"])
    nat = pkg._native

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    lo, hi = sharded.shard_range(N_IMAGES, world, rank)
    n_local = hi - lo
    x, y = syn.device_pair((C, H, W, n_local), NOISE, seed=1000 + rank, device=dev)
    grad = pkg.jl_empty((C, H, W, n_local), torch.float32, dev)
    ssims = torch.empty(n_local, dtype=torch.float32, device=dev)
    all_scores = torch.empty(N_IMAGES, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    # Two score buffers in turn: the all-gather of step i runs on NCCL's stream while the
    # kernel of step i+1 writes the other buffer; before a buffer is written again the
    # stream waits for the gather that reads it.  Every gather ends inside the timed region.
    gather = sharded.ScoreGather(N_IMAGES, torch.float32, dev) if world > 1 else None
    score_bufs = [ssims, torch.empty_like(ssims)]
    pending = [None, None]

    def step(i):
        b = i % 2
        if pending[b] is not None:
            pending[b].wait()          # the current stream waits for the collective, not the host
            pending[b] = None
        pkg.ssim_with_gradient_(score_bufs[b], grad, x, y, None, True)
        if world > 1:
            pending[b] = gather.start(score_bufs[b])
        else:
            all_scores.copy_(score_bufs[b])

    def drain():
        for b in range(2):
            if pending[b] is not None:
                pending[b].wait()
                pending[b] = None

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    for i in range(args.warmup):
        step(i)
    drain()
    barrier()
    sampler = ClockSampler(local)
    sampler.start()
    k0 = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    k1 = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record(stream)
    for i in range(args.steps):
        b = i % 2
        if pending[b] is not None:
            pending[b].wait()
            pending[b] = None
        k0[i].record(stream)
        pkg.ssim_with_gradient_(score_bufs[b], grad, x, y, None, True)
        k1[i].record(stream)
        if world > 1:
            pending[b] = gather.start(score_bufs[b])
        else:
            all_scores.copy_(score_bufs[b])
    drain()
    e1.record(stream)
    barrier()
    clocks = sampler.stop()
    elapsed = e0.elapsed_time(e1) / 1e3
    kern = sum(a.elapsed_time(b) for a, b in zip(k0, k1)) / 1e3 / args.steps
    t = torch.tensor([elapsed, kern], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed, kern = float(t[0]), float(t[1])
    ssims = score_bufs[(args.steps - 1) % 2]          # the last timed step's values
    if world > 1:
        all_scores = gather.out                          # drained: the last step's full vector

    # ---- parity of the timed batch itself (outside the timed region), max over ranks
    parity = None
    if not args.no_parity:
        pr = parity_sample(pkg, x, y, ssims, grad, lo, seed=77 + rank)
        pt = torch.tensor([pr["max_abs_ssim_err"], pr["max_rel_l2_grad_err"]], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(pt, op=dist.ReduceOp.MAX)
        parity = {"max_abs_ssim_err": float(pt[0]), "max_rel_l2_grad_err": float(pt[1]),
                  "images_per_rank": len(pr["images"]), "rank0_images": pr["images"],
                  "oracle": pr["oracle"], "tolerance": pr["tolerance"],
                  "ok": bool(float(pt[0]) <= 1e-5 and float(pt[1]) <= 1e-4)}

    # ---- end to end: host buffers through the public API, copies inside the timed region
    e2e = None
    if not args.no_e2e:
        numa_node = bind_to_gpu_numa_node(local)
        hx = torch.empty(x.numel(), dtype=torch.float32, pin_memory=True)
        hy = torch.empty(y.numel(), dtype=torch.float32, pin_memory=True)
        hx.copy_(x.permute(3, 2, 1, 0).reshape(-1))
        hy.copy_(y.permute(3, 2, 1, 0).reshape(-1))
        hs = torch.empty(N_IMAGES, dtype=torch.float32, pin_memory=True)
        dx = pkg.jl_empty((C, H, W, n_local), torch.float32, dev)
        dy = pkg.jl_empty((C, H, W, n_local), torch.float32, dev)
        dxf = dx.permute(3, 2, 1, 0).reshape(-1)      # memory order: image n at [n*E, (n+1)*E)
        dyf = dy.permute(3, 2, 1, 0).reshape(-1)
        e2e_steps = max(1, min(args.steps, 3))
        # The host-to-device copies run on their own stream in chunks of images, and each
        # chunk's call starts once its copy has landed, so the copies overlap the kernels.
        copy_stream = torch.cuda.Stream(dev)
        n_chunks = min(16, n_local)
        bounds = [(n_local * j // n_chunks, n_local * (j + 1) // n_chunks) for j in range(n_chunks)]
        E = C * H * W
        landed = [torch.cuda.Event() for _ in bounds]

        def e2e_step():
            start = torch.cuda.Event()
            start.record(stream)                     # the previous step's calls are done with dx, dy
            copy_stream.wait_event(start)
            for (lo_i, hi_i), ev in zip(bounds, landed):
                with torch.cuda.stream(copy_stream):
                    dxf[lo_i * E:hi_i * E].copy_(hx[lo_i * E:hi_i * E], non_blocking=True)
                    dyf[lo_i * E:hi_i * E].copy_(hy[lo_i * E:hi_i * E], non_blocking=True)
                    ev.record(copy_stream)
                stream.wait_event(ev)
                pkg.ssim_with_gradient_(ssims[lo_i:hi_i], grad[..., lo_i:hi_i], dx[..., lo_i:hi_i],
                                        dy[..., lo_i:hi_i], None, True)
            scores = sharded.gather_scores(ssims, N_IMAGES) if world > 1 else ssims
            hs.copy_(scores, non_blocking=True)

        # host-to-device peak of this rank: one pinned 1 GiB copy (best of 3), all ranks at once
        barrier()
        nprobe = min(hx.numel(), 1 << 28)
        best = None
        for _ in range(3):
            pa, pb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            pa.record(copy_stream)
            with torch.cuda.stream(copy_stream):
                dxf[:nprobe].copy_(hx[:nprobe], non_blocking=True)
            pb.record(copy_stream)
            pb.synchronize()
            ms = pa.elapsed_time(pb)
            best = ms if best is None else min(best, ms)
        h2d_peak = nprobe * 4 / (best / 1e3) / 1e9

        e2e_step()
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        b.record(stream)
        barrier()
        t_local = a.elapsed_time(b) / 1e3
        h2d_bytes = 2 * n_local * C * H * W * 4
        te = torch.tensor([t_local], dtype=torch.float64, device=dev)
        rates = torch.tensor([h2d_bytes * e2e_steps / t_local / 1e9, h2d_peak], dtype=torch.float64, device=dev)
        rmin, rmax = rates.clone(), rates.clone()
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
            dist.all_reduce(rmin, op=dist.ReduceOp.MIN)
            dist.all_reduce(rmax, op=dist.ReduceOp.MAX)
        e2e = {"value": e2e_steps * N_IMAGES * H * W / float(te[0]) / 1e9, "unit": "Gpixel/s",
               "h2d_bytes_per_step": int(h2d_bytes), "d2h_bytes_per_step": int(N_IMAGES * 4),
               "steps": e2e_steps, "calls_per_step": n_chunks,
               "h2d_gbs_per_rank": {"min": float(rmin[0]), "max": float(rmax[0])},
               "h2d_peak_gbs_per_rank": {"min": float(rmin[1]), "max": float(rmax[1]),
                                         "how": "one pinned 1 GiB host-to-device copy, best of 3, all ranks at once"},
               "h2d_frac_of_peak": float(rmin[0]) / float(rmax[1]),
               "host_threads": os.cpu_count(),
               "rank0_numa_node": numa_node,
               "overlap": "pinned host buffers; H2D in image chunks on a copy stream, overlapped with the calls"}
        del hx, hy, dx, dy, dxf, dyf

    extras = {}
    if rank == 0 and not args.no_extras:
        extras = side_benchmarks(pkg, dev)
        if not args.no_cpu:   # the same full-HD SSIM on host cores (one thread per channel plane)
            extras["cpu_fullhd_1ch_ssim_ms"] = cpu_fullhd_ms(1)
            extras["cpu_fullhd_3ch_ssim_ms"] = cpu_fullhd_ms(3)
            extras["cpu_fullhd_cores"] = {"1ch": 1, "3ch": 3}
            ncores = os.cpu_count() or 1
            extras["cpu_batch32_3x256x256_dssim_grad_ms"] = {"1": cpu_batch32_dssim_grad_ms(1),
                                                             str(ncores): cpu_batch32_dssim_grad_ms(ncores)}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        n_cpu = 64
        rate, passes, spent = CpuSample(n_cpu, os.cpu_count() or 1).rate(min_seconds=10.0)
        cpu = {"value": rate, "unit": "Gpixel/s", "cores": os.cpu_count() or 1, "kind": "port",
               "sample": f"{n_cpu} images of 3x512x512 with gradient, {passes} passes ({spent:.1f} s), "
                         "oracle in C with pthreads"}

    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank != 0:
        return 0
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    peak, peak_kind = measured_peaks()
    pixels = N_IMAGES * H * W
    value = args.steps * pixels / elapsed / 1e9
    alg_bytes = n_local * C * H * W * BYTES_PER_ELEM
    achieved = alg_bytes / kern / 1e9
    line = {
        "metric": "SSIM+grad Gpixel/s", "value": value, "unit": "Gpixel/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * elapsed / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (device RNG, seeded)",
        "config": {"workload": WORKLOAD, "images": N_IMAGES, "images_per_gpu": n_local, "shape": [C, H, W],
                   "noise_sigma": NOISE, "l2": "inputs (12.9 GB) larger than L2, no flush",
                   "parallelism": f"batch-shard x{world}"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                     "traffic": traffic_per_launch(n_local),
                     "kernel": "fssim::pipe_kernel<96,true>", "kernel_ms": kern * 1e3,
                     "alg_bytes_per_launch": alg_bytes},
        "fp32_pipe": fp32_pipe(kern, n_local, clocks, sms),
        "cpu_baseline": cpu,
        "parity": parity,
        "e2e": e2e,
        "gpu_launches": args.steps,
        "clocks": clocks,
        "gelem_per_s": value * C,
    }
    line.update(extras)
    print(json.dumps(line), flush=True)
    return 0


def c_abi_call_cost(channels):
    """The library's own per-call cost from C, without Python (tests/c_client/fssim_call_cost.c,
    built here with gcc): host time of one full-HD forward call, its device time back to back,
    and one call plus the read of its value."""
    import tempfile
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    lib_dir = os.path.join(ROOT, "fastcudassim.jl_b200", "lib")
    exe = os.path.join(tempfile.mkdtemp(), "fssim_call_cost")
    subprocess.run(["gcc", "-O2", "-std=c11", "-o", exe, os.path.join(ROOT, "tests", "c_client", "fssim_call_cost.c"),
                    "-I", os.path.join(ROOT, "include"), "-I", os.path.join(cuda, "include"), "-L", lib_dir,
                    "-lfastssim", "-L", os.path.join(cuda, "lib64"), "-lcudart", "-Wl,-rpath," + lib_dir],
                   check=True, capture_output=True)
    r = subprocess.run([exe, str(channels), "200"], check=True, capture_output=True, text=True, timeout=120)
    return json.loads(r.stdout.strip().splitlines()[-1])


def side_benchmarks(pkg, dev):
    """Full-HD SSIM latency (3x1080x1920 forward) and the 32x3x256x256 DSSIM + gradient call,
    each timed with CUDA events after an L2 flush (their inputs fit in L2)."""
    import torch
    syn = __import__(pkg.__name__ + ".synthetic", fromlist=["x"])
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    out = {}

    def timed(fn, reps=30):
        ts = []
        for i in range(reps + 3):
            flush.zero_()
            # keep the device busy while the host enqueues the call, so the events
            # bracket device work only (the Python call itself takes tens of us)
            torch.cuda._sleep(2_000_000)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            b.synchronize()
            if i >= 3:
                ts.append(a.elapsed_time(b))
        return statistics.median(ts)

    # the floor of these latencies: a one-element kernel timed the same way (launch and events)
    one = torch.zeros(1, device=dev)
    out["event_floor_us"] = timed(lambda: one.add_(1.0)) * 1e3
    for name, shape, noise in (("fullhd_1ch", (1, 1080, 1920), 0.1), ("fullhd_3ch", (3, 1080, 1920), 0.05)):
        x, y = syn.device_pair(shape, noise, device=dev)
        s = torch.empty(1, dtype=torch.float32, device=dev)
        ms = timed(lambda: pkg.ssim_(s, x, y))
        walls = []
        for _ in range(20):
            flush.zero_()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            pkg.ssim(x, y)                      # returns a Python float: includes the D2H read
            walls.append((time.perf_counter() - t0) * 1e3)
        nbytes = x.numel() * 8
        out[f"{name}_ssim_ms"] = ms
        out[f"{name}_ssim_api_wall_ms"] = statistics.median(walls)
        out[f"{name}_ssim_hbm_frac"] = nbytes / (ms / 1e3) / 1e9 / measured_peaks()[0]
        out[f"{name}_ssim_fp32_frac"] = fp32_frac(FWD_FMA_PER_ELEM, x.numel(), ms, sms)
    for ch in (1, 3):   # the same calls from C: the library's own cost, without the Python layer
        try:
            out[f"fullhd_{ch}ch_c_abi"] = c_abi_call_cost(ch)
        except Exception as e:  # report, do not fail the benchmark line
            out[f"fullhd_{ch}ch_c_abi"] = {"error": str(e)[:200]}
    x, y = syn.device_pair((3, 256, 256, 32), None, device=dev)
    d = torch.empty(32, dtype=torch.float32, device=dev)
    g = pkg.jl_empty((3, 256, 256, 32), torch.float32, dev)
    ms = timed(lambda: pkg.dssim_with_gradient_(d, g, x, y, None, True))
    out["batch32_3x256x256_dssim_grad_ms"] = ms
    out["batch32_3x256x256_dssim_grad_hbm_frac"] = x.numel() * 12 / (ms / 1e3) / 1e9 / measured_peaks()[0]
    out["batch32_3x256x256_dssim_grad_fp32_frac"] = fp32_frac(FMA_PER_ELEM, x.numel(), ms, sms)
    # config 4: 64 x 3 x 512 x 512 in N0f8 and in Float16, Float32 gradient, converted in-kernel
    for tag, dt, nb in (("u8", torch.uint8, 1), ("f16", torch.float16, 2)):
        x, y = syn.device_pair((3, 512, 512, 64), 0.1, dtype=dt, device=dev)
        s = torch.empty(64, dtype=torch.float32, device=dev)
        g = pkg.jl_empty((3, 512, 512, 64), torch.float32, dev)
        ms = timed(lambda: pkg.ssim_with_gradient_(s, g, x, y, None, True), reps=10)
        out[f"batch64_3x512x512_{tag}_ssim_grad_ms"] = ms
        out[f"batch64_3x512x512_{tag}_ssim_grad_hbm_frac"] = x.numel() * (2 * nb + 4) / (ms / 1e3) / 1e9 / measured_peaks()[0]
        out[f"batch64_3x512x512_{tag}_ssim_grad_fp32_frac"] = fp32_frac(FMA_PER_ELEM, x.numel(), ms, sms)
        del x, y, g
    # Float64 inputs, values and gradient (the double-precision kernel): 16 x 3 x 512 x 512
    x, y = syn.device_pair((3, 512, 512, 16), 0.1, dtype=torch.float64, device=dev)
    s = torch.empty(16, dtype=torch.float64, device=dev)
    g = pkg.jl_empty((3, 512, 512, 16), torch.float64, dev)
    ms = timed(lambda: pkg.ssim_with_gradient_(s, g, x, y, None, True), reps=5)
    out["batch16_3x512x512_f64_ssim_grad_ms"] = ms
    out["batch16_3x512x512_f64_ssim_grad_gelem_s"] = x.numel() / (ms / 1e3) / 1e9
    del x, y, g
    # one autograd step (values, then the pullback of a per-image cotangent) on 64 x 3 x 512 x 512:
    # the reference's rrule (gradient with the values, broadcast in the pullback) against the
    # deferred rule (values only, then one gradient launch with the cotangent folded in)
    x, y = syn.device_pair((3, 512, 512, 64), 0.1, device=dev)
    x.requires_grad_(True)
    cot = torch.linspace(-1.0, 1.0, 64, device=dev)
    for tag, defer in (("eager", False), ("deferred", True)):
        def step():
            x.grad = None
            pkg.dssim_autograd(x, y, defer_gradient=defer).backward(cot)
        out[f"autograd_dssim_64x3x512x512_{tag}_ms"] = timed(step, reps=10)
    del x, y
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-extras", action="store_true")
    ap.add_argument("--no-parity", action="store_true")
    ap.add_argument("--profile-case", choices=["fused", "fwd", "fused_u8", "fused_f16", "fused_f64", "fhd1", "fhd3"],
                    default=None,
                    help="only run one kernel on a small case (a size for ncu captures): "
                         "warmup + steps launches and their mean time")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.profile_case:
        return profile_case(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


def profile_case(args):
    """warmup + steps launches of one kernel: on 64x3x512x512 (0.3 GB in Float32, larger than
    L2) for the batch cases, on one 1x1080x1920 or 3x1080x1920 image for the full-HD cases."""
    import torch
    import __graft_entry__ as ge
    pkg = ge.load_package()
    syn = __import__(pkg.__name__ + ".synthetic", fromlist=["x"])
    shape = {"fhd1": (1, 1080, 1920, 1), "fhd3": (3, 1080, 1920, 1)}.get(args.profile_case, (C, H, W, 64))
    dt = {"fused_u8": torch.uint8, "fused_f16": torch.float16,
          "fused_f64": torch.float64}.get(args.profile_case, torch.float32)
    if args.profile_case == "fused_f64":   # Float64 inputs, values and gradient (16 images)
        shape = (C, H, W, 16)
    odt = torch.float64 if dt == torch.float64 else torch.float32
    x, y = syn.device_pair(shape, NOISE, dtype=dt)
    s = torch.empty(shape[3], dtype=odt, device="cuda")
    g = pkg.jl_empty(shape, odt)
    def launch():
        if args.profile_case.startswith("fused"):
            pkg.ssim_with_gradient_(s, g, x, y, None, True)
        else:
            pkg.ssim_(s, x, y)
    for _ in range(args.warmup):
        launch()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        launch()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / max(args.steps, 1)
    print(json.dumps({"profile_case": args.profile_case, "launches": args.warmup + args.steps,
                      "ms_per_launch": ms, "gelem_per_s": x.numel() / ms / 1e6, "ssim0": float(s[0])}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
