#!/usr/bin/env python
"""G2V fwd+bwd benchmark (BASELINE.json metric: ms/step at 18k Gaussians x 1024-D on 200x200x16).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg3] [--impl ours|reference]

One step = forward of PyCudaGaussianVoxelizer + backward with randn upstream gradients for density
and grid_feats, i.e. the gradient of sum(density*gD) + sum(grid_feats*gF) w.r.t. means3D, opacity,
covariances and features.  Inputs are synthetic with the reference's distributions (seeded CPU
generation, test/test_reference.py:30-45).  Every input of a step is larger than L2 (grid_feats and its
gradient are 2.6 GB each at cfg3), so no L2 flush is needed between steps.

With N > 1 (torchrun, one rank per GPU) every rank runs its own scene (batched scenes, data-parallel,
no collective in the step); the reported time is the max over ranks ("scaling": "weak").
``--impl reference`` times the CPU restatement of the reference's algorithm (oracle/, float64, all host
threads) on a bounded x-slab sample of the same workload and, when the reference build exists in
oracle/_ref, also times that CUDA build on the GPU ("reference_cuda").
"""
from __future__ import annotations

import argparse
import glob
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(REPO, "shelfgaussian-cudagaussianvoxelizer_b200")
for _p in (REPO, PKG_DIR):
    if _p not in sys.path:
        sys.path.insert(0, _p)

RANGE = [-40.0, -40.0, -1.0, 40.0, 40.0, 5.4]
CONFIGS = {
    "cfg1": dict(n=512, c=32, size=0.4, range=[-8.0, -8.0, -1.0, 8.0, 8.0, 5.4], var_max=2.5, expand=0.0),
    "cfg2": dict(n=9000, c=768, size=0.4, range=RANGE, var_max=2.5, expand=0.0),
    "cfg3": dict(n=18000, c=1024, size=0.4, range=RANGE, var_max=2.5, expand=0.0),
    "cfg4": dict(n=18000, c=1024, size=0.4, range=RANGE, var_max=2.5, expand=0.05),
    "cfg5": dict(n=100000, c=256, size=0.2, range=RANGE, var_max=8.0, expand=0.0),
    # test_reference.py's forward shape; small enough for multi-pass ncu captures (grid_feats 328 MB > L2)
    "small128": dict(n=18000, c=128, size=0.4, range=RANGE, var_max=2.5, expand=0.0),
    # cfg3's Gaussian density and channels on a quarter of the area (100x100x16): same tile lists,
    # grid_feats 655 MB (> L2), small enough for multi-pass ncu captures
    "cfg3q": dict(n=4500, c=1024, size=0.4, range=[-20.0, -20.0, -1.0, 20.0, 20.0, 5.4], var_max=2.5, expand=0.0),
}
METRIC = "G2V fwd+bwd ms/step (18k Gaussians, 1024-D, 200×200×16) and % HBM roofline"


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def load_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as fh:
            d = json.load(fh)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ------------------------------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms around the timed region.

    The sampler is started and waited for (first sample written) before the timed region begins, so a
    short timed region still has samples; ``stop()`` keeps the samples whose timestamps fall inside the
    region (begin = end of the constructor, end = the call of ``stop()``) and, when the region was shorter
    than the sampling interval, the first sample after it began ("window": "nearest")."""
    FIELDS = ("timestamp,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    INTERVAL_MS = 50

    def __init__(self, gpu_id):
        self.proc = None
        self.gpu_id = str(gpu_id) if gpu_id is not None else None
        self.path = tempfile.mktemp(prefix="g2v_clocks_", suffix=".csv")
        for select in ((True, False) if self.gpu_id else (False,)):
            if self._start(select):
                break
        self.t_begin = time.time()

    def _start(self, select):
        try:
            self.fh = open(self.path, "w")
            cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms",
                   str(self.INTERVAL_MS)]
            if select:
                cmd += ["-i", self.gpu_id]
            self.proc = subprocess.Popen(cmd, stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
            return False
        t0 = time.time()
        while time.time() - t0 < 10.0:  # wait for the first sample (nvidia-smi start-up)
            if self.proc.poll() is not None:
                break
            if os.path.getsize(self.path) > 0:
                return True
            time.sleep(0.02)
        self._kill()
        return False

    def _kill(self):
        if self.proc is None:
            return
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        self.proc = None

    @staticmethod
    def _stamp(s):
        import datetime
        for fmt in ("%Y/%m/%d %H:%M:%S.%f", "%Y/%m/%d %H:%M:%S"):
            try:
                return datetime.datetime.strptime(s, fmt).timestamp()
            except ValueError:
                pass
        return None

    def stop(self):
        t_end = time.time()
        if self.proc is None:
            return None
        time.sleep(2.0 * self.INTERVAL_MS / 1000.0)  # the sample that follows the region's end
        self._kill()
        rows = []
        want = self.gpu_id.lower().replace("gpu-", "") if self.gpu_id else None
        with open(self.path) as fh:
            for line in fh:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 10:
                    continue
                if want and want.count("-") >= 4 and parts[1].lower().replace("gpu-", "") != want:
                    continue
                try:
                    rows.append((self._stamp(parts[0]), float(parts[2]), float(parts[3]), parts[6:10]))
                except ValueError:
                    continue
        os.unlink(self.path)
        if not rows:
            return None
        slack = self.INTERVAL_MS / 1000.0
        inside = [r for r in rows if r[0] is not None and self.t_begin - slack <= r[0] <= t_end + slack]
        window = "timed region"
        if not inside:
            after = [r for r in rows if r[0] is not None and r[0] >= self.t_begin]
            inside = after[:1] or rows[-1:]
            window = "nearest"
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({nm for r in inside for nm, v in zip(names, r[3]) if v.lower().startswith("active")})
        return {"sm_mhz": statistics.median([r[1] for r in inside]), "sm_max_mhz": inside[-1][2],
                "reasons": reasons, "samples": len(inside), "window": window,
                "interval_ms": self.INTERVAL_MS}


def gpu_id_for(dev_index):
    import torch
    try:
        u = str(torch.cuda.get_device_properties(dev_index).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        if vis:
            return vis.split(",")[dev_index]
        return dev_index


# ------------------------------------------------------------------------------------------------
def make_inputs(cfg, seed):
    from oracle import oracle
    size = [cfg["size"]] * 3
    m, o, c, f = oracle.generate_inputs(cfg["n"], cfg["c"], cfg["range"], seed=seed, var_max=cfg["var_max"],
                                        expand=cfg["expand"])
    return size, cfg["range"], m, o, c, f


def algorithmic_bytes(kernel, n, c, V, M, MB, ntiles):
    """Algorithmic HBM bytes of one launch over the whole grid: the bytes each kernel must move per unit of work
    (voxel rows of grid_feats / its gradient, feature rows, per-Gaussian records, CSR entries)."""
    per_gauss = n * (12 + 4 + 36 + 24)  # mean, opacity, cov_inv, lb/ub
    kernel = {"splat_tc_kernel": "splat_tile_kernel", "spass_tc_kernel": "spass_kernel",
              "fpass_tc_kernel": "fpass_kernel"}.get(kernel, kernel)
    if kernel == "splat_tile_kernel":
        return 4 * V * c + 4 * V + 4 * n * c + per_gauss + 4 * M + 4 * (ntiles + 1)
    if kernel == "spass_kernel":
        return 4 * V * c + 4 * n * c + 8 * V + 40 * M + per_gauss + 4 * M + 4 * (ntiles + 1)
    if kernel == "fpass_kernel":  # the gradient rows, D, the feature-gradient rows; partial rows are not algorithmic
        return 4 * V * c + 4 * V + 4 * n * c + per_gauss
    if kernel == "reduce_feats_kernel":
        return 4 * MB * c + 4 * n * c
    return None


def algorithmic_flops(kernel, c, M):
    """Contraction FLOPs of one launch (forward 2*64*M*C, backward 4*64*M*C, split here between
    the tile pass and the feature-gradient pass) and the tensor-core FLOPs that realise them with three
    bf16/f16 products (hi*hi + hi*lo + lo*hi) per fp32 product."""
    if kernel in ("splat_tc_kernel", "spass_tc_kernel", "fpass_tc_kernel"):
        alg = 2.0 * 64 * M * c
        return alg, 3.0 * alg
    return None, None


def load_bf16_peak():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as fh:
            d = json.load(fh)
        return float(d["bf16_tflops"]), "measured (MEASURED_PEAKS.json bf16_tflops, burst)"
    return 1590.0, "fallback"


def step_bytes(n, c, V, M):
    """Algorithmic bytes of one fwd+bwd step (8.11 GB at cfg3): forward = N*52 (mean, opacity, covariance)
    + 4NC (features) + 4V (density) + 4VC (grid_feats) + N*64 (cov_inv, boxes, voxel counts) + 4(N+1) + 4M;
    backward = 8V + 8VC (both gradients and density / grid_feats) + 4NC + N*76 + 4(N+1) + 4M + N*52 + 4NC."""
    fwd = n * 52 + 4 * n * c + 4 * V + 4 * V * c + n * 64 + 4 * (n + 1) + 4 * M
    bwd = 8 * V + 8 * V * c + 4 * n * c + n * 76 + 4 * (n + 1) + 4 * M + n * 52 + 4 * n * c
    return fwd + bwd


def run_ours(args, rank, world, dev):
    import numpy as np  # noqa: F401
    import torch
    import torch.distributed as dist
    from CudaGaussianVoxelizer import PyCudaGaussianVoxelizer, _C, _lib

    cfg = CONFIGS[args.config]
    if args.density_only:
        cfg = dict(cfg, c=0)
    size, rng, m_h, o_h, c_h, f_h = make_inputs(cfg, seed=args.seed + rank)
    (X, Y, Z), tiles = _C.grid_shape(size, rng)
    V = X * Y * Z
    n, c = cfg["n"], cfg["c"]
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    gD = torch.randn((X, Y, Z), device=dev, generator=g)
    gF = torch.randn((X, Y, Z, c), device=dev, generator=g)
    sr = args.cov_input == "sr"
    if sr:  # Gaussians given by scales and rotation quaternions (covariances formed in the kernels)
        from oracle import oracle
        s_h, q_h = oracle.generate_scale_rot(n, seed=args.seed + rank + 100, var_max=cfg["var_max"])
        host_in = (m_h, o_h, s_h, q_h, f_h)
    else:
        host_in = (m_h, o_h, c_h, f_h)
    if args.density_only:  # features=None: the density-only kernels
        host_in = host_in[:-1]
    leaves = [t.to(dev).requires_grad_() for t in host_in]
    if args.graph:  # whole step captured in one CUDA graph: capacity-capped module, no host synchronisation
        if sr:
            raise SystemExit("--graph takes covariance inputs")
        out0, mb0 = _C._forward_impl(*[t.detach() for t in leaves[:3]], size, rng,
                                     None if args.density_only else leaves[3].detach(), False, plan=True)
        caps = (int(out0[7].numel() * 1.25) + 1024, int(mb0 * 1.25) + 1024 if c > 0 else 0)
        del out0
        vox = PyCudaGaussianVoxelizer(voxel_size=size, voxel_range=rng, timing=False, max_pairs=caps[0],
                                      max_block_pairs=caps[1])
    else:
        vox = PyCudaGaussianVoxelizer(voxel_size=size, voxel_range=rng, timing=False)

    def call(v, ls):
        f = None if args.density_only else ls[-1]
        if sr:
            return v(ls[0], ls[1], features=f, scales=ls[2], rotations=ls[3])
        return v(ls[0], ls[1], ls[2], f)

    def grads(density, grid_feats, ls):
        if args.density_only:
            return torch.autograd.grad([density], ls, [gD])
        return torch.autograd.grad([density, grid_feats], ls, [gD, gF])

    def step():
        density, grid_feats, _ = call(vox, leaves)
        return grads(density, grid_feats, leaves)

    if args.graph:
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(3):
                step()
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, capture_error_mode="relaxed"):
            graph_out = step()  # noqa: F841  (static outputs of the captured step)
        eager_step = step

        def step():
            graph.replay()
    else:
        eager_step = step

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats(dev)
    resident = torch.cuda.memory_allocated(dev)
    sampler = ClockSampler(gpu_id_for(dev.index))
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    peak_mem = torch.cuda.max_memory_allocated(dev)
    barrier()
    ms = ev0.elapsed_time(ev1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())

    # per-kernel device time (CUDA events on the launch stream, inside the library) over K steps; graph
    # replays launch nothing from the host, so --graph profiles the same kernels through the eager module
    prof_step = eager_step
    _lib.profile_enable(True)
    for _ in range(args.steps):
        prof_step()
    torch.cuda.synchronize()
    prof = _lib.profile_read()
    _lib.profile_enable(False)
    launches_per_step = sum(v[1] for v in prof.values()) / args.steps

    # sizes for the roofline
    feat_d = None if args.density_only else leaves[-1].detach()
    if sr:
        out = _C._forward_impl(leaves[0].detach(), leaves[1].detach(), None, size, rng, feat_d, False,
                               scale_rot=(leaves[2].detach(), leaves[3].detach()))[0]
    else:
        out = _C.gaussian_voxelizer_forward(*[t.detach() for t in leaves[:3]], size, rng, feat_d, timing=False)
    M = int(out[7].numel())
    MB = _C.backward_plan(out[2], out[3], (X, Y, Z), c)
    del out
    ntiles = tiles[0] * tiles[1] * tiles[2]
    peak, peak_kind = load_peaks()
    top = max(prof.items(), key=lambda kv: kv[1][0])
    kname, (kms, kcount) = top
    kbytes = algorithmic_bytes(kname, n, c, V, M, MB, ntiles)
    avg_ms = kms / kcount
    achieved = kbytes / (avg_ms * 1e-3) / 1e9 if kbytes else None
    traffic = None
    tpath = os.path.join(REPO, "profiles", "ncu_traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as fh:
            traffic = json.load(fh).get(args.config, {}).get(kname)
    # the same launch against the tensor pipe (the contractions are tensor-bound at three split products)
    alg_flops, tc_flops = algorithmic_flops(kname, c, M)
    tpeak, tpeak_kind = load_bf16_peak()
    tensor = None
    if tc_flops:
        t_ach = tc_flops / (avg_ms * 1e-3) / 1e12
        tensor = {"achieved": t_ach, "peak": tpeak, "unit": "TFLOP/s", "frac": t_ach / tpeak,
                  "flops_per_launch": tc_flops, "algorithmic_flops_per_launch": alg_flops,
                  "peak_source": tpeak_kind,
                  "note": "contraction 2*64*M*C per launch executed as three bf16/f16 products"}
    roofline = {"bound": "hbm", "kernel": kname, "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": (achieved / peak) if achieved else None, "traffic": traffic,
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback",
                "algorithmic_bytes_per_launch": kbytes, "avg_launch_ms": avg_ms,
                "kernel_share": {k: round(v[0] / sum(x[0] for x in prof.values()), 4) for k, v in prof.items()},
                "kernel_ms_per_step": {k: round(v[0] / args.steps, 4) for k, v in prof.items()},
                "tensor": tensor}
    sb = step_bytes(n, c, V, M)

    # end-to-end through the public API with pinned host inputs (H2D inside the timed region)
    host = [t.pin_memory() for t in host_in]
    h2d = sum(t.numel() * t.element_size() for t in host)
    # stats timing off: the reference-style per-call timing synchronisations are optional
    vox_e2e = PyCudaGaussianVoxelizer(voxel_size=size, voxel_range=rng, timing=False)

    # Input pipeline of a training loop: step i + 1's inputs are copied host -> device on a copy stream
    # while step i computes (two device copies of the inputs), so the copies of K steps overlap the compute
    # of the previous ones; step i waits for its own copy only.  Every one of the K copies is issued and
    # completes inside the timed region (the first one before any compute, nothing is copied ahead of it).
    copy_stream = torch.cuda.Stream(device=dev)

    def e2e_fetch():
        with torch.cuda.stream(copy_stream):
            ls = [t.to(dev, non_blocking=True) for t in host]
            ev = torch.cuda.Event()
            ev.record(copy_stream)
        return ls, ev

    # the result of every step is copied device -> host into pinned memory (4 bytes) and read on the host
    # once the next step has been enqueued, as a training loop logs its losses: the host does not wait for
    # step i to finish before it enqueues step i + 1 (whose forward synchronises once, for the pair count)
    res_host = [torch.empty(1, dtype=torch.float32, pin_memory=True) for _ in range(2)]
    res_seen = []

    def e2e_result(t, slot):
        buf = res_host[slot]
        buf.copy_(t.reshape(-1)[:1], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(stream)
        return ev, buf

    def e2e_read(pending):
        ev, buf = pending
        ev.synchronize()
        res_seen.append(float(buf[0]))

    def e2e_step(fetched, prefetch, slot=0):
        # H2D of the inputs (fetched: this step's copies, already issued), forward, backward with the same
        # upstream gradients as the device-timed step, and a D2H copy of one element of the result (4 bytes);
        # prefetch issues the next step's copies before this step's compute is enqueued
        if args.graph:  # into the captured step's static inputs, then replay
            with torch.no_grad():
                for t, h in zip(leaves, host):
                    t.copy_(h, non_blocking=True)
            graph.replay()
            return e2e_result(graph_out[0], slot), None
        ls, ev = fetched
        stream.wait_event(ev)
        for t in ls:
            t.record_stream(stream)  # the caching allocator must not hand these to the copy stream early
        nxt = e2e_fetch() if prefetch else None
        ls = [t.requires_grad_() for t in ls]
        density, grid_feats, _ = call(vox_e2e, ls)
        gr = grads(density, grid_feats, ls)
        return e2e_result(gr[0], slot), nxt

    def e2e_run(k):
        fetched = None if args.graph else e2e_fetch()
        pending = None
        for i in range(k):
            out, fetched = e2e_step(fetched, prefetch=i + 1 < k, slot=i & 1)
            if pending is not None:
                e2e_read(pending)  # step i - 1's result, read after step i was enqueued
            pending = out
        e2e_read(pending)

    e2e_run(max(1, args.warmup))
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    copy_stream.wait_stream(stream)  # the first copy starts after e0
    e2e_run(args.steps)
    stream.wait_stream(copy_stream)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())

    cpu = cpu1 = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(cfg, args.seed, threads=os.cpu_count() or 1, steps=1)
        cpu1 = cpu_baseline_cfg1(args.seed)

    line = {
        "metric": METRIC, "value": round(ms, 4), "unit": "ms", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, reference distributions)",
        "config": {"workload": f"{args.config}: N={n} Gaussians, C={c} fp32 features, {X}x{Y}x{Z} voxels, "
                               f"fwd+bwd with randn upstream grads"
                               + (", Gaussians as scales + rotation quaternions (grads to both)" if sr else "")
                               + (", density only (features=None)" if args.density_only else "")
                               + (", the whole step replayed from one CUDA graph (capacity-capped module, no "
                                  "host sync)" if args.graph else ""),
                   "global_batch": world,
                   "scenes_per_rank": 1, "l2": "inputs larger than L2 (grid_feats 4*V*C bytes)",
                   "pairs_M": M, "block_pairs": MB, "parallelism": f"dp{world} (independent scenes)",
                   "e2e": "PyCudaGaussianVoxelizer(timing=False) + torch.autograd.grad with the upstream "
                          "gradients; pinned host inputs copied every step on a copy stream, step i + 1's copy "
                          "overlapping step i's compute (K copies inside the timed region); each step's result "
                          "copied to pinned host memory and read on the host after the next step is enqueued "
                          "(K reads inside the timed region)"},
        "roofline": roofline,
        "step_roofline": {"algorithmic_bytes": sb, "achieved_gbs": sb / (ms * 1e-3) / 1e9,
                          "frac": sb / (ms * 1e-3) / 1e9 / peak},
        "cpu_baseline": cpu,
        "cpu_baseline_cfg1": cpu1,
        "e2e": {"value": round(e2e_ms, 4), "unit": "ms", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4},
        "gpu_launches": int(round(launches_per_step * args.steps)),
        "clocks": clocks,
        "memory": {"peak_gb": round(peak_mem / 1e9, 3), "resident_before_steps_gb": round(resident / 1e9, 3),
                   "what": "torch.cuda.max_memory_allocated over the timed steps: inputs and the randn upstream "
                           "gradients (resident before the steps), outputs, gradients and the library's "
                           "workspaces"},
    }
    return line


def cpu_baseline(cfg, seed, threads, steps=1, slab_vox=16):
    """The oracle (float64 C restatement of the reference algorithm) on an x-slab of the grid: the
    forward and backward of the voxels in `slab_vox` x-columns at the centre of the grid; ms/step
    scaled to the full grid by X / slab_vox."""
    import numpy as np
    from oracle import oracle
    size, rng, m, o, c, f = make_inputs(cfg, seed)
    m, o, c, f = m.numpy(), o.numpy(), c.numpy(), f.numpy()
    bx = oracle.boxes(m, c, size, rng)
    X, Y, Z = bx.dims
    x0 = (X // 2 // 4) * 4 - slab_vox // 2
    x0 = max(0, x0 - x0 % 4)
    x1 = min(X, x0 + slab_vox)
    C = f.shape[1]
    rs = np.random.default_rng(7)
    gD = np.zeros((X, Y, Z), np.float32)
    gF = np.zeros((X, Y, Z, C), np.float32)
    gD[x0:x1] = rs.standard_normal((x1 - x0, Y, Z), dtype=np.float32)
    gF[x0:x1] = rs.standard_normal((x1 - x0, Y, Z, C), dtype=np.float32)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        D, F = oracle.forward(m, o, c, f, bx.lb, bx.ub, size, rng, (X, Y, Z), x_range=(x0, x1), nthreads=threads)
        oracle.backward(m, o, c, f, bx.lb, bx.ub, size, rng, (X, Y, Z), gD, gF, D, F, x_range=(x0, x1),
                        nthreads=threads)
        times.append(time.perf_counter() - t0)
        del D, F
    t = min(times)
    return {"value": round(t * 1e3 * X / (x1 - x0), 1), "unit": "ms", "cores": threads, "kind": "port",
            "sample_ms": round(t * 1e3, 1),
            "sample": f"x-slab of {x1 - x0} of {X} voxel columns (forward + backward of those voxels), "
                      f"float64, scaled x{X / (x1 - x0):.1f} to the full grid; {t:.2f} s per sample"}


def cpu_baseline_cfg1(seed, steps=3):
    """The reference's CPU brute force (its float64 restatement in oracle/, test/test_reference.py:57-79) at
    cfg1, the configuration the reference's own CPU test runs (N=512, C=32, 40x40x16): the whole grid,
    forward + backward with randn upstream gradients, timed on one thread and on every host thread."""
    import numpy as np
    import torch
    from oracle import oracle
    size, rng, m, o, c, f = make_inputs(CONFIGS["cfg1"], seed)
    m, o, c, f = m.numpy(), o.numpy(), c.numpy(), f.numpy()
    bx = oracle.boxes(m, c, size, rng)
    dims = bx.dims
    rs = np.random.default_rng(7)
    gD = rs.standard_normal(tuple(dims), dtype=np.float32)
    gF = rs.standard_normal(tuple(dims) + (f.shape[1],), dtype=np.float32)
    nproc = os.cpu_count() or 1
    out = {"unit": "ms", "kind": "port", "nproc": nproc, "torch_num_threads": torch.get_num_threads(),
           "steps": steps, "workload": "cfg1: N=512, C=32, 40x40x16 voxels, whole grid, fwd+bwd, float64"}
    for key, threads in (("threads_1", 1), ("threads_all", nproc)):
        ts = []
        for _ in range(steps + 1):  # the first run is a warm-up
            t0 = time.perf_counter()
            D, F = oracle.forward(m, o, c, f, bx.lb, bx.ub, size, rng, dims, nthreads=threads)
            oracle.backward(m, o, c, f, bx.lb, bx.ub, size, rng, dims, gD, gF, D, F, nthreads=threads)
            ts.append(time.perf_counter() - t0)
        out[key] = round(statistics.median(ts[1:]) * 1e3, 2)
    out["cores"] = {"threads_1": 1, "threads_all": nproc}
    return out


def reference_cuda(cfg, seed, dev, steps=5, warmup=2):
    """Time the reference's own CUDA build (oracle/_ref, compiled from its sources) on this GPU: `steps`
    forward + backward steps after `warmup`, CUDA events on the current stream, clocks sampled over the
    timed steps, and the allocator's peak memory over them (inputs and upstream gradients included)."""
    from oracle import build_ref
    ext = build_ref.load()
    if ext is None:
        return {"unavailable": "oracle/_ref has no reference build"}
    import torch
    size, rng, m, o, c, f = make_inputs(cfg, seed)
    m, o, c, f = [t.to(dev).contiguous() for t in (m, o, c, f)]
    vs = torch.tensor(size, dtype=torch.float32, device=dev)
    vr = torch.tensor(rng, dtype=torch.float32, device=dev)
    g = torch.Generator(device=dev).manual_seed(1000)
    out = ext.gaussian_voxelizer_forward(m, o, c, vs, vr, f)
    X, Y, Z = out[0].shape
    gD = torch.randn((X, Y, Z), device=dev, generator=g)
    gF = torch.randn((X, Y, Z, f.shape[1]), device=dev, generator=g)
    del out

    def step():
        d, ci, lb, ub, nv, gf, off, ids, fs = ext.gaussian_voxelizer_forward(m, o, c, vs, vr, f)
        r = ext.gaussian_voxelizer_backward(gD, gF, m, o, ci, vs, vr, lb, ub, nv, off, ids, d, gf, f)
        return fs, r[4]

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats(dev)
    sampler = ClockSampler(gpu_id_for(dev.index))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    st = [step() for _ in range(steps)]
    e1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1) / steps
    return {"value": round(ms, 3), "unit": "ms", "steps": steps, "warmup": warmup,
            "device": torch.cuda.get_device_name(dev),
            "fwd_sec": [round(a, 5) for a, _ in st], "bwd_sec": [round(b, 5) for _, b in st],
            "peak_mem_gb": round(torch.cuda.max_memory_allocated(dev) / 1e9, 3), "clocks": clocks,
            "source": "reference src/cuda_gaussian_voxelizer.cu built for sm_100a by oracle/build_ref.py"}


def run_forward_only(args, dev):
    """Profiling mode: only forward passes (for ncu captures of the splat kernels)."""
    import torch
    from CudaGaussianVoxelizer import _C
    cfg = CONFIGS[args.config]
    size, rng, m, o, c, f = make_inputs(cfg, seed=args.seed)
    m, o, c, f = [t.to(dev) for t in (m, o, c, f)]
    for _ in range(args.warmup):
        _C.gaussian_voxelizer_forward(m, o, c, size, rng, f, timing=False)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        _C.gaussian_voxelizer_forward(m, o, c, size, rng, f, timing=False)
    e1.record()
    torch.cuda.synchronize()
    return {"mode": "forward-only", "config": args.config, "ms_per_forward": e0.elapsed_time(e1) / args.steps}


def run_reference(args, rank, world, dev):
    cfg = CONFIGS[args.config]
    threads = os.cpu_count() or 1
    vals, samples = [], []
    t_region = time.perf_counter()
    for i in range(args.warmup + args.steps):
        if i == args.warmup:
            t_region = time.perf_counter()
        r = cpu_baseline(cfg, args.seed, threads=threads, steps=1)
        if i >= args.warmup:
            vals.append(r["value"])
            samples.append(r["sample_ms"])
    region_s = time.perf_counter() - t_region
    value = statistics.median(vals)
    cpu = dict(r)
    cpu["value"] = value
    # value: the metric for the whole workload (the sample's time scaled to the full grid); ms_per_step: what
    # one timed step actually took (one sample), so that steps x ms_per_step fits the timed region
    line = {"metric": METRIC, "value": value, "unit": "ms", "impl": "reference", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": statistics.median(samples),
            "higher_is_better": False,
            "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic (seeded, reference distributions)",
            "config": {"workload": f"{args.config}: N={cfg['n']}, C={cfg['c']}, CPU x-slab sample",
                       "global_batch": 1},
            "cpu_baseline": cpu, "e2e": {"value": value, "unit": "ms", "h2d_bytes_per_step": 0,
                                         "d2h_bytes_per_step": 0},
            "what_ran": {"samples_timed": args.steps, "samples_warmup": args.warmup,
                         "sample": cpu["sample"], "timed_region_s": round(region_s, 2),
                         "value_is": "median over the timed samples of the sample time scaled to the full grid",
                         "ms_per_step_is": "median time of one timed sample (one step of this arm)"},
            "cpu_baseline_cfg1": cpu_baseline_cfg1(args.seed)}
    if dev is not None and not args.no_reference_cuda:
        try:
            line["reference_cuda"] = reference_cuda(cfg, args.seed, dev)
        except Exception as exc:  # report, do not fail the CPU arm
            line["reference_cuda"] = {"unavailable": f"{type(exc).__name__}: {exc}"[:300]}
    return line


def run_single_scene(args, rank, world, dev):
    """One scene split into x-slabs over the ranks (CudaGaussianVoxelizer.distributed): every rank holds
    the same Gaussians, splats its slab, and one NCCL all-reduce sums the gradients.  Strong scaling:
    the total work is fixed as N grows; `value` is the max-over-ranks device time of a step."""
    import torch
    import torch.distributed as dist
    from CudaGaussianVoxelizer import _C, _lib
    from CudaGaussianVoxelizer.distributed import SlabGaussianVoxelizer, balanced_slab_bounds, tile_pairs_per_column

    cfg = CONFIGS[args.config]
    size, rng, m_h, o_h, c_h, f_h = make_inputs(cfg, seed=args.seed)  # the same scene on every rank
    (X, Y, Z), tiles = _C.grid_shape(size, rng)
    n, c = cfg["n"], cfg["c"]
    leaves = [t.to(dev).requires_grad_() for t in (m_h, o_h, c_h, f_h)]
    # slabs split by the (Gaussian, tile) pairs per tile column (the same counts on every rank)
    bounds = balanced_slab_bounds(tile_pairs_per_column(leaves[0].detach(), leaves[2].detach(), size, rng), world)
    vox = SlabGaussianVoxelizer(voxel_size=size, voxel_range=rng, rank=rank, world=world, tile_bounds=bounds)
    x0, x1 = vox.rows
    g = torch.Generator(device=dev).manual_seed(1000)
    gD = torch.randn((X, Y, Z), device=dev, generator=g)[x0:x1].contiguous()
    gF = torch.randn((X, Y, Z, c), device=dev, generator=g)[x0:x1].contiguous()

    def step():
        density, grid_feats, _ = vox(*leaves)
        return torch.autograd.grad([density, grid_feats], leaves, [gD, gF])

    def barrier():
        if world > 1:
            dist.barrier()

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        stream = torch.cuda.current_stream(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        t = e0.elapsed_time(e1) / args.steps
        if world > 1:
            tt = torch.tensor([t], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t = float(tt.item())
        return t

    sampler = ClockSampler(gpu_id_for(dev.index))
    ms = timed(step)
    clocks = sampler.stop()
    host = [t.pin_memory() for t in (m_h, o_h, c_h, f_h)]
    h2d = sum(t.numel() * t.element_size() for t in host)

    def e2e_step():
        ls = [t.to(dev, non_blocking=True).requires_grad_() for t in host]
        density, grid_feats, _ = vox(*ls)
        grads = torch.autograd.grad([density, grid_feats], ls, [gD, gF])
        return grads[0].reshape(-1)[:1].to("cpu").item()

    e2e_ms = timed(e2e_step)
    _lib.profile_enable(True)
    step()
    torch.cuda.synchronize()
    prof = _lib.profile_read()
    _lib.profile_enable(False)
    tot = sum(v[0] for v in prof.values()) or 1.0
    return {
        "metric": METRIC, "value": round(ms, 4), "unit": "ms", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": False, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, reference distributions)",
        "config": {"workload": f"{args.config}: one scene, N={n} Gaussians, C={c}, {X}x{Y}x{Z} voxels, split into "
                               f"{world} x-slabs of tiles balanced by (Gaussian, tile) pairs (tile column bounds "
                               f"{bounds}), one NCCL all-reduce of "
                               f"the packed gradients per step", "global_batch": 1,
                   "parallelism": f"x-slab split over {world} GPUs",
                   "l2": "inputs larger than L2 (grid_feats 4*V*C bytes)"},
        "rank0_kernel_share": {k: round(v[0] / tot, 4) for k, v in prof.items()},
        "e2e": {"value": round(e2e_ms, 4), "unit": "ms", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4},
        "gpu_launches": int(sum(v[1] for v in prof.values())),
        "clocks": clocks,
    }


def run_batched(args, rank, world, dev):
    """--scenes B: every step splats B scenes of the config (independent seeds) through ONE batched call
    (PyCudaGaussianVoxelizer with scene_sizes: one preparation + synchronisation, one splat, one
    backward for the batch), against the same B scenes as B single-scene calls (`loop_ms_per_step`).
    `value` is the batched step; per-rank work is fixed (weak scaling over ranks)."""
    import torch
    import torch.distributed as dist
    from CudaGaussianVoxelizer import PyCudaGaussianVoxelizer, _C, _lib

    cfg = CONFIGS[args.config]
    B = args.scenes
    scenes = [make_inputs(cfg, seed=args.seed + rank * B + b) for b in range(B)]
    size, rng = scenes[0][0], scenes[0][1]
    (X, Y, Z), tiles = _C.grid_shape(size, rng)
    V = X * Y * Z
    n, c = cfg["n"], cfg["c"]
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    gD = torch.randn((B, X, Y, Z), device=dev, generator=g)
    gF = torch.randn((B, X, Y, Z, c), device=dev, generator=g)
    host_in = [torch.cat([sc[2 + k] for sc in scenes]) for k in range(4)]
    leaves = [t.to(dev).requires_grad_() for t in host_in]
    sizes = [n] * B
    vox = PyCudaGaussianVoxelizer(voxel_size=size, voxel_range=rng, timing=False)

    def step():
        density, grid_feats, _ = vox(*leaves, scene_sizes=sizes)
        return torch.autograd.grad([density, grid_feats], leaves, [gD, gF])

    per_scene = [[t[b * n:(b + 1) * n].detach().clone().requires_grad_() for t in leaves] for b in range(B)]

    def loop_step():
        out = []
        for b in range(B):
            density, grid_feats, _ = vox(*per_scene[b])
            out.append(torch.autograd.grad([density, grid_feats], per_scene[b], [gD[b], gF[b]]))
        return out

    def barrier():
        if world > 1:
            dist.barrier()

    stream = torch.cuda.current_stream(dev)

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        t = e0.elapsed_time(e1) / args.steps
        if world > 1:
            tt = torch.tensor([t], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t = float(tt.item())
        return t

    sampler = ClockSampler(gpu_id_for(dev.index))
    ms = timed(step)
    clocks = sampler.stop()
    loop_ms = timed(loop_step)

    _lib.profile_enable(True)
    for _ in range(args.steps):
        step()
    torch.cuda.synchronize()
    prof = _lib.profile_read()
    _lib.profile_enable(False)
    launches = sum(v[1] for v in prof.values())
    off, nsc = _C._scene_offsets(sizes, n * B, dev)
    out, MB = _C._forward_impl(*[t.detach() for t in leaves[:3]], size, rng, leaves[3].detach(), False,
                               scenes=(off, nsc))
    M = int(out[7].numel())
    del out
    ntiles = tiles[0] * tiles[1] * tiles[2]
    peak, peak_kind = load_peaks()
    kname, (kms, kcount) = max(prof.items(), key=lambda kv: kv[1][0])
    kbytes = algorithmic_bytes(kname, n * B, c, V * B, M, MB, ntiles * B)
    avg_ms = kms / kcount
    achieved = kbytes / (avg_ms * 1e-3) / 1e9 if kbytes else None
    roofline = {"bound": "hbm", "kernel": kname, "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": (achieved / peak) if achieved else None, "traffic": None,
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback",
                "algorithmic_bytes_per_launch": kbytes, "avg_launch_ms": avg_ms,
                "kernel_share": {k: round(v[0] / sum(x[0] for x in prof.values()), 4) for k, v in prof.items()}}
    sb = step_bytes(n, c, V, M // B) * B

    host = [t.pin_memory() for t in host_in]
    h2d = sum(t.numel() * t.element_size() for t in host)

    def e2e_step():
        ls = [t.to(dev, non_blocking=True).requires_grad_() for t in host]
        density, grid_feats, _ = vox(*ls, scene_sizes=sizes)
        grads = torch.autograd.grad([density, grid_feats], ls, [gD, gF])
        return grads[0].reshape(-1)[:1].to("cpu").item()

    e2e_ms = timed(e2e_step)
    return {
        "metric": METRIC, "value": round(ms, 4), "unit": "ms", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, reference distributions)",
        "config": {"workload": f"{args.config} x {B} scenes per rank in one batched call: N={n} Gaussians, C={c}, "
                               f"{X}x{Y}x{Z} voxels per scene, fwd+bwd with randn upstream grads",
                   "global_batch": B * world, "scenes_per_rank": B, "pairs_M": M, "block_pairs": MB,
                   "l2": "inputs larger than L2", "parallelism": f"dp{world} x batched {B}"},
        "per_scene_ms": round(ms / B, 4), "loop_ms_per_step": round(loop_ms, 4),
        "batched_speedup_vs_loop": round(loop_ms / ms, 3),
        "roofline": roofline,
        "step_roofline": {"algorithmic_bytes": sb, "achieved_gbs": sb / (ms * 1e-3) / 1e9,
                          "frac": sb / (ms * 1e-3) / 1e9 / peak},
        "cpu_baseline": None,
        "e2e": {"value": round(e2e_ms, 4), "unit": "ms", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4},
        "gpu_launches": int(launches), "clocks": clocks,
    }


def _timed_steps(fn, args, world, dev):
    """W untimed steps, then K steps between CUDA events on the current stream; max over ranks (ms/step)."""
    import torch
    import torch.distributed as dist
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    t = e0.elapsed_time(e1) / args.steps
    if world > 1:
        tt = torch.tensor([t], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t = float(tt.item())
    return t


def extra_batch8_cfg4(args, rank, world, dev, total=8):
    """The batched-scenes config (cfg4: B=8 scenes of 18k x 1024-D over the range widened by 10%): the 8
    scenes are dealt to the ranks (scene b to rank b % N), each rank splats its scenes in one batched call
    and backpropagates; no collective inside the step.  ms per batch of 8 = max over ranks."""
    import torch
    from CudaGaussianVoxelizer import PyCudaGaussianVoxelizer, _C
    cfg = CONFIGS["cfg4"]
    mine = [b for b in range(total) if b % world == rank]
    B = len(mine)
    scenes = [make_inputs(cfg, seed=args.seed + 100 + b) for b in mine]
    size, rng = scenes[0][0], scenes[0][1]
    (X, Y, Z), _ = _C.grid_shape(size, rng)
    n, c = cfg["n"], cfg["c"]
    g = torch.Generator(device=dev).manual_seed(3000 + rank)
    shape = (B, X, Y, Z) if B > 1 else (X, Y, Z)
    gD = torch.randn(shape, device=dev, generator=g)
    gF = torch.randn(shape + (c,), device=dev, generator=g)
    leaves = [torch.cat([sc[2 + k] for sc in scenes]).to(dev).requires_grad_() for k in range(4)]
    vox = PyCudaGaussianVoxelizer(voxel_size=size, voxel_range=rng, timing=False)
    sizes = [n] * B

    def step():
        if B > 1:
            density, grid_feats, _ = vox(*leaves, scene_sizes=sizes)
        else:
            density, grid_feats, _ = vox(*leaves)
        return torch.autograd.grad([density, grid_feats], leaves, [gD, gF])

    ms = _timed_steps(step, args, world, dev)
    del leaves, gD, gF
    torch.cuda.empty_cache()
    return {"value": round(ms, 4), "unit": "ms per batch of 8 scenes", "scenes_per_rank": B, "n_gpus": world,
            "workload": f"cfg4: {total} scenes, N={n} Gaussians each over the range widened by 10%, C={c}, "
                        f"{X}x{Y}x{Z} voxels; scene b on rank b % N, one batched call per rank",
            "scaling": "strong (the batch of 8 is fixed)", "collective_in_step": False}


def extra_single_scene_cfg5(args, rank, world, dev):
    """The spatially sharded config (cfg5: one scene of 100k Gaussians x 256-D on 400x400x32): x-slabs of
    tiles over the ranks, replicated Gaussians, one NCCL all-reduce of the packed gradients per step
    (CudaGaussianVoxelizer.distributed).  ms per step = max over ranks; the all-reduce's own time
    (CUDA events around it on rank 0) is reported beside it."""
    import torch
    from CudaGaussianVoxelizer import _C
    from CudaGaussianVoxelizer import distributed as dmod
    cfg = CONFIGS["cfg5"]
    size, rng, m_h, o_h, c_h, f_h = make_inputs(cfg, seed=args.seed)
    (X, Y, Z), tiles = _C.grid_shape(size, rng)
    leaves = [t.to(dev).requires_grad_() for t in (m_h, o_h, c_h, f_h)]
    # slabs split by the (Gaussian, tile) pairs per tile column (the same counts on every rank)
    bounds = dmod.balanced_slab_bounds(dmod.tile_pairs_per_column(leaves[0].detach(), leaves[2].detach(), size, rng),
                                       world)
    vox = dmod.SlabGaussianVoxelizer(voxel_size=size, voxel_range=rng, rank=rank, world=world, tile_bounds=bounds)
    x0, x1 = vox.rows
    g = torch.Generator(device=dev).manual_seed(1000)
    gD = torch.randn((X, Y, Z), device=dev, generator=g)[x0:x1].contiguous()
    gF = torch.empty((x1 - x0, Y, Z, cfg["c"]), device=dev).normal_(generator=g)

    def step():
        density, grid_feats, _ = vox(*leaves)
        return torch.autograd.grad([density, grid_feats], leaves, [gD, gF])

    ms = _timed_steps(step, args, world, dev)
    ar_ms = None
    if world > 1:
        dmod.allreduce_events = []
        try:
            for _ in range(max(3, args.steps // 4)):
                step()
            torch.cuda.synchronize()
            ar_ms = statistics.median(a.elapsed_time(b) for a, b in dmod.allreduce_events)
        finally:
            dmod.allreduce_events = None
    packed_mb = cfg["n"] * (13 + cfg["c"]) * 4 / 1e6
    del leaves, gD, gF
    torch.cuda.empty_cache()
    return {"value": round(ms, 4), "unit": "ms", "n_gpus": world, "scaling": "strong (one fixed scene)",
            "workload": f"cfg5: N={cfg['n']} Gaussians, C={cfg['c']}, {X}x{Y}x{Z} voxels, var U(0.5,8); "
                        f"{world} x-slabs of tiles balanced by (Gaussian, tile) pairs (tile column bounds {bounds})",
            "allreduce_ms": None if ar_ms is None else round(ar_ms, 4),
            "allreduce_mb": round(packed_mb, 1) if world > 1 else 0.0,
            "collective_in_step": "one NCCL all-reduce (sum) of the packed [N x (13 + C)] gradients" if world > 1
            else "none (one rank)"}


LOSS_METRIC = "feature cosine loss fwd+bwd ms/step over the voxel grid and % HBM roofline"


def loss_bytes(kernel, V, C, nvalid):
    """Algorithmic HBM bytes of one cosine-loss launch: label + mask of every voxel (5 B), prediction and
    target rows of the valid voxels (8 C B), and for the backward the gradient of every voxel (4 C B)."""
    if kernel == "cosine_loss_fwd_kernel":
        return 5 * V + 8 * C * nvalid
    if kernel == "cosine_loss_bwd_kernel":
        return 5 * V + 8 * C * nvalid + 4 * C * V
    return None


def run_loss(args, rank, world, dev):
    """Feature cosine loss (PyCudaFeatsCosineLoss) forward + backward on a resident grid.

    Workload: the voxelizer's grid at --config (200x200x16 at cfg3) with --loss-channels channels (default
    the config's C), labels and masks drawn as in the reference's loss tests (25% labelled x 70% visible),
    target = prediction + 0.1 noise.  Every rank runs its own grid (weak scaling, no collective).  An L2
    flush (a 256 MB write) separates the timed steps; only the steps are inside the events."""
    import torch
    import torch.distributed as dist
    from CudaGaussianVoxelizer import PyCudaFeatsCosineLoss, _C, _lib

    cfg = CONFIGS[args.config]
    size = [cfg["size"]] * 3
    (X, Y, Z), _ = _C.grid_shape(size, cfg["range"])
    C = args.loss_channels or cfg["c"]
    V = X * Y * Z
    gen = torch.Generator(device=dev).manual_seed(2000 + rank)
    p = torch.randn((X, Y, Z, C), device=dev, generator=gen)
    g = p + 0.1 * torch.randn((X, Y, Z, C), device=dev, generator=gen)
    label = (torch.rand((X, Y, Z), device=dev, generator=gen) < 0.25).float()
    mask = torch.rand((X, Y, Z), device=dev, generator=gen) < 0.7
    nvalid = int((label.bool() & mask).sum().item())
    p.requires_grad_(True)
    crit = PyCudaFeatsCosineLoss(voxel_size=size, voxel_range=cfg["range"], timing=False)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        loss, _ = crit(label, mask, p, g)
        return torch.autograd.grad(loss, p)[0]

    def barrier():
        if world > 1:
            dist.barrier()

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        barrier()
        evs = []
        for _ in range(args.steps):
            flush.fill_(1)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            evs.append((e0, e1))
        torch.cuda.synchronize()
        barrier()
        t = sum(a.elapsed_time(b) for a, b in evs) / args.steps
        if world > 1:
            tt = torch.tensor([t], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t = float(tt.item())
        return t

    sampler = ClockSampler(gpu_id_for(dev.index))
    ms = timed(step)
    clocks = sampler.stop()

    _lib.profile_enable(True)
    for _ in range(args.steps):
        flush.fill_(1)
        step()
    torch.cuda.synchronize()
    prof = _lib.profile_read()
    _lib.profile_enable(False)
    peak, peak_kind = load_peaks()
    kern = {}
    for k, (kms, cnt) in prof.items():
        b = loss_bytes(k, V, C, nvalid)
        avg = kms / cnt
        kern[k] = {"avg_launch_ms": avg, "algorithmic_bytes_per_launch": b,
                   "achieved_gbs": b / (avg * 1e-3) / 1e9 if b else None,
                   "frac": b / (avg * 1e-3) / 1e9 / peak if b else None}
    top = "cosine_loss_bwd_kernel"
    traffic = None
    tpath = os.path.join(REPO, "profiles", "ncu_traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as fh:
            traffic = json.load(fh).get(f"loss_{args.config}_c{C}", {}).get(top)
    roofline = {"bound": "hbm", "kernel": top, "achieved": kern[top]["achieved_gbs"], "peak": peak, "unit": "GB/s",
                "frac": kern[top]["frac"], "traffic": traffic,
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback",
                "algorithmic_bytes_per_launch": kern[top]["algorithmic_bytes_per_launch"],
                "avg_launch_ms": kern[top]["avg_launch_ms"], "kernels": kern}

    # end to end: pinned host inputs copied every step, loss value read back
    host = [t.detach().cpu().pin_memory() for t in (label, mask, p, g)]
    h2d = sum(t.numel() * t.element_size() for t in host)
    crit_e2e = PyCudaFeatsCosineLoss(voxel_size=size, voxel_range=cfg["range"], timing=False)

    def e2e_step():
        lab, msk, pp, gg = [t.to(dev, non_blocking=True) for t in host]
        pp.requires_grad_(True)
        loss, _ = crit_e2e(lab, msk, pp, gg)
        grad = torch.autograd.grad(loss, pp)[0]
        return loss.item(), grad

    e2e_ms = timed(e2e_step)

    # the drop-in _C calls timed exactly like the reference build's (reference_loss_cuda): wall clock of
    # forward (count returned to the host, as the reference's signature requires) + backward, synchronised
    pd = p.detach()
    one = torch.ones((), device=dev)
    walls = []
    for i in range(args.warmup + args.steps):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        _, count, _ = _C.CudaFeatsCosinelossForward(label, mask, pd, g, timing=False)
        _C.CudaFeatsCosinelossBackward(one, label, mask, pd, g, count, timing=False)
        torch.cuda.synchronize()
        if i >= args.warmup:
            walls.append((time.perf_counter() - t0) * 1e3)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = loss_cpu_baseline(X, Y, Z, C)
    return {
        "metric": LOSS_METRIC, "value": round(ms, 4), "unit": "ms", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded; reference loss-test distributions)",
        "config": {"workload": f"loss on {args.config}'s grid: {X}x{Y}x{Z} voxels, C={C}, {nvalid} valid voxels "
                               f"(25% labelled x 70% visible), fwd+bwd via PyCudaFeatsCosineLoss + autograd",
                   "global_batch": world, "l2": "256 MB L2 flush between timed steps (outside the events)",
                   "parallelism": f"dp{world} (independent grids)"},
        "roofline": roofline, "cpu_baseline": cpu,
        "e2e": {"value": round(e2e_ms, 4), "unit": "ms", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4},
        "dropin_wall": {"value": round(statistics.median(walls), 4), "unit": "ms",
                        "what": "_C.CudaFeatsCosinelossForward + Backward, wall clock with host synchronisation, "
                                "timed like the reference build's arm"},
        "gpu_launches": int(sum(v[1] for v in prof.values())),
        "clocks": clocks,
    }


def loss_cpu_baseline(X, Y, Z, C, rows=None):
    """The float64 oracle of the loss (numpy) on an x-slab of the grid, scaled to the whole grid."""
    import numpy as np
    from oracle import oracle
    rows = rows or max(1, min(X, int(2e7 // max(1, Y * Z * max(C, 1)))))
    label, mask, p, g = oracle.generate_loss_inputs((rows, Y, Z), C, "noise", seed=0)
    label, mask, p, g = label.numpy(), mask.numpy(), p.numpy(), g.numpy()
    ts = []
    for _ in range(2):  # the first pass also pays the first touch of its float64 buffers
        t0 = time.perf_counter()
        _, count = oracle.cosine_loss_forward(label, mask, p, g)
        oracle.cosine_loss_backward(1.0, count, label, mask, p, g)
        ts.append(time.perf_counter() - t0)
    t = ts[-1]
    return {"value": round(t * 1e3 * X / rows, 1), "unit": "ms", "cores": 1, "kind": "port",
            "sample": f"x-slab of {rows} of {X} voxel rows ({rows * Y * Z} voxels, C={C}), numpy float64, scaled "
                      f"x{X / rows:.1f} to the full grid; {t:.2f} s per sample"}


def reference_loss_cuda(X, Y, Z, C, dev, steps=3):
    """The reference's own loss kernels (oracle/_ref build of src/cuda_feats_loss.cu) on the same grid."""
    from oracle import build_ref
    ext = build_ref.load()
    if ext is None:
        return {"unavailable": "oracle/_ref has no reference build"}
    import torch
    gen = torch.Generator(device=dev).manual_seed(2000)
    p = torch.randn((X, Y, Z, C), device=dev, generator=gen)
    g = p + 0.1 * torch.randn((X, Y, Z, C), device=dev, generator=gen)
    label = (torch.rand((X, Y, Z), device=dev, generator=gen) < 0.25).float()
    mask = torch.rand((X, Y, Z), device=dev, generator=gen) < 0.7
    one = torch.ones((), device=dev)
    ts = []
    for i in range(steps + 1):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        loss, count, _ = ext.CudaFeatsCosinelossForward(label, mask, p, g)
        ext.CudaFeatsCosinelossBackward(one, label, mask, p, g, count)
        torch.cuda.synchronize()
        if i:
            ts.append((time.perf_counter() - t0) * 1e3)
    return {"value": round(statistics.median(ts), 3), "unit": "ms",
            "what": "reference CUDA build of src/cuda_feats_loss.cu (oracle/_ref), forward + backward, wall clock "
                    "with its own host synchronisations"}


def run_loss_reference(args, rank, world, dev):
    cfg = CONFIGS[args.config]
    from CudaGaussianVoxelizer import _C
    (X, Y, Z), _ = _C.grid_shape([cfg["size"]] * 3, cfg["range"])
    C = args.loss_channels or cfg["c"]
    vals = []
    for i in range(args.warmup + args.steps):
        r = loss_cpu_baseline(X, Y, Z, C)
        if i >= args.warmup:
            vals.append(r["value"])
    value = statistics.median(vals)
    cpu = dict(r)
    cpu["value"] = value
    line = {"metric": LOSS_METRIC, "value": value, "unit": "ms", "impl": "reference", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": value, "higher_is_better": False,
            "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic (seeded)",
            "config": {"workload": f"loss on {args.config}'s grid {X}x{Y}x{Z}, C={C}, CPU x-slab sample",
                       "global_batch": 1},
            "cpu_baseline": cpu, "e2e": {"value": value, "unit": "ms", "h2d_bytes_per_step": 0,
                                         "d2h_bytes_per_step": 0}}
    if dev is not None and not args.no_reference_cuda:
        try:
            line["reference_cuda"] = reference_loss_cuda(X, Y, Z, C, dev)
        except Exception as exc:
            line["reference_cuda"] = {"unavailable": f"{type(exc).__name__}: {exc}"[:300]}
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="cfg3", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-reference-cuda", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the cfg4 batch-of-8 and cfg5 single-scene measurements of the default run")
    ap.add_argument("--forward-only", action="store_true", help="profiling mode: forward passes only")
    ap.add_argument("--path", default="voxelizer", choices=["voxelizer", "loss"],
                    help="voxelizer: the G2V fwd+bwd step (default); loss: the feature cosine loss fwd+bwd")
    ap.add_argument("--loss-channels", type=int, default=0, help="channels of the loss workload (default: config C)")
    ap.add_argument("--density-only", action="store_true", help="features=None (the density-only kernels)")
    ap.add_argument("--graph", action="store_true",
                    help="capture the whole step (capacity-capped module) in one CUDA graph and replay it")
    ap.add_argument("--scenes", type=int, default=1,
                    help="scenes per rank per step, splatted in one batched call (compared with a loop of calls)")
    ap.add_argument("--cov-input", default="cov", choices=["cov", "sr"],
                    help="voxelizer inputs: covariances (default) or scales + rotation quaternions")
    ap.add_argument("--single-scene", action="store_true",
                    help="one scene split into x-slabs over the ranks (strong scaling) instead of one scene per rank")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return
        import torch
        dev = torch.device("cuda", local) if torch.cuda.is_available() else None
        run = run_loss_reference if args.path == "loss" else run_reference
        print(json.dumps(run(args, rank, world, dev)), flush=True)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if args.forward_only:
        print(json.dumps(run_forward_only(args, dev)), flush=True)
        return
    if world > 1:
        # NCCL's initialisation log (communicator size, ranks, transports) goes to stderr, so the rank count
        # of the run is on record without touching the one JSON line on stdout
        os.environ.setdefault("NCCL_DEBUG", "INFO")
        os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    try:
        run = (run_loss if args.path == "loss" else run_single_scene if args.single_scene else
               run_batched if args.scenes > 1 else run_ours)
        line = run(args, rank, world, dev)
        default = run is run_ours and args.config == "cfg3" and not (args.density_only or args.graph or
                                                                      args.cov_input != "cov")
        if default and not args.no_extra:
            # the multi-GPU configs of the workload, measured in the same run at the same N
            line["batch8_cfg4"] = extra_batch8_cfg4(args, rank, world, dev)
            line["single_scene_cfg5"] = extra_single_scene_cfg5(args, rank, world, dev)
        if world > 1:
            line["comm"] = {"backend": dist.get_backend(), "world_size": dist.get_world_size(),
                            "nccl_version": ".".join(map(str, torch.cuda.nccl.version()))}
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
