#!/usr/bin/env python
"""Benchmark: 3DGS forward+backward views/sec at 1080p through gswarp_b200.

Workload (benchmark configuration 5, weak scaling): 6,000,000 Gaussians with the
config-2 distributions (SH degree 3), cameras on a radius-12 ring at random
elevations, 1920x1080.  Each GPU renders 8 views per step; each view does
forward, loss = L1 + 0.2 * (1 - SSIM) against a seeded target, backward; the
per-Gaussian gradients (59 floats per Gaussian in one flat buffer) are then
summed across ranks with one NCCL all-reduce.  A "step" is one such pass;
``value`` is views/sec of the whole job (8 * N views per step divided by the
max-over-ranks device time of a step).

``e2e`` runs the same step through the public API with each view's target
image copied from pinned host memory inside the timed region and the loss
read back to the host.  At N=1 the line also carries the single-view config-2
measurement (1M Gaussians, fwd+bwd raster + SSIM) and the CPU-oracle
baseline.  ``--impl reference`` times the CPU restatement of the reference's
kernels (the reference itself needs warp-lang, which this image lacks).

Launch: python bench.py [--gpus N --steps K --warmup W]; for N>1 under
torchrun (one rank per GPU, NCCL).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "3DGS fwd+bwd views/sec at 1080p, 1M–6M Gaussians, at 1/2/4/8 B200"
FLOATS_PER_GAUSSIAN = 59  # means 3, scales 3, rotations 4, opacity 1, SH 48


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--gaussians", type=int, default=6_000_000)
    p.add_argument("--views-per-gpu", type=int, default=8)
    p.add_argument("--width", type=int, default=1920)
    p.add_argument("--height", type=int, default=1080)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-cfg2", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-autograd", action="store_true", help="skip the drop-in autograd path comparison")
    p.add_argument("--no-optimizer", action="store_true", help="skip the fused Adam measurement")
    p.add_argument("--path", default="fused", choices=["fused", "autograd"],
                   help="the measured path: the fused training step, or the drop-in autograd path alone")
    p.add_argument("--backward-order", default="views", choices=["views", "ranges"],
                   help="fused step: per-view backward (default) or the range-ordered backward")
    p.add_argument("--deferred-views", type=int, default=None,
                   help="fused step: the last K views finish range by range (default: the library's)")
    return p.parse_args()


# ---------------------------------------------------------------------------
# clocks sampling during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        """``device_index`` is torch's ordinal; nvidia-smi is pointed at the same
        physical GPU by its UUID (torch's ordinals follow CUDA_VISIBLE_DEVICES,
        nvidia-smi's do not)."""
        import torch

        self.uuid = None
        try:
            u = str(torch.cuda.get_device_properties(device_index).uuid)
            self.uuid = u if u.startswith("GPU-") else f"GPU-{u}"
        except (AttributeError, RuntimeError):
            pass
        self.gpu = self.uuid or str(device_index)
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", self.gpu], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm), "gpu_uuid": self.uuid}


# ---------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------
def make_scene(args, device, rank):
    import torch

    from gswarp_b200 import workloads as wl

    scene = wl.config2_scene(seed=0, n=args.gaussians).to(device)
    views_all = wl.ring_views(64, seed=0, width=args.width, height=args.height)
    V = args.views_per_gpu
    views = [views_all[(rank * V + i) % 64].to(device) for i in range(V)]
    return scene, views


class Trainer:
    """Parameters, the flat gradient buffer and one data-parallel step over
    this rank's views, through one of two public paths:

    * ``fused``    -- gswarp_b200.training.FusedViewStep: the C ABI stage by
      stage with the photometric loss kernels and preprocess backward
      accumulating into the flat gradient buffer (no autograd);
    * ``autograd`` -- the drop-in path: gswarp_b200.GaussianRasterizer +
      fused_ssim under autograd (gswarp_b200.view_sharding.ViewShardedStep).
    """

    def __init__(self, scene, views, targets_dev, targets_host, world, device, path="fused"):
        import torch

        import gswarp_b200 as gs
        from gswarp_b200.training import FusedViewStep
        from gswarp_b200.view_sharding import ViewShardedStep

        self.gs = gs
        self.torch = torch
        self.path = path
        self.N = scene.n
        self.device = device
        self.world = world
        self.means = scene.means.contiguous().requires_grad_(True)
        self.scales = scene.scales.contiguous().requires_grad_(True)
        self.rots = scene.rotations.contiguous().requires_grad_(True)
        self.opac = scene.opacities.contiguous().requires_grad_(True)
        self.sh = scene.sh.contiguous().requires_grad_(True)
        self.params = [self.means, self.scales, self.rots, self.opac, self.sh]
        self.views = views
        self.targets_dev = targets_dev
        self.targets_host = targets_host
        self.bg = torch.zeros(3, device=device)
        self.settings = [
            gs.GaussianRasterizationSettings(
                image_height=v.height, image_width=v.width, tanfovx=v.tanfovx, tanfovy=v.tanfovy, bg=self.bg,
                scale_modifier=1.0, viewmatrix=v.viewmatrix, projmatrix=v.projmatrix, sh_degree=3,
                campos=v.campos, prefiltered=False)
            for v in views]
        self.loss_host = torch.zeros(len(views), dtype=torch.float32).pin_memory() if targets_host else None
        if path == "fused":
            self.fused = FusedViewStep(self.params, self.settings, l1_weight=1.0, ssim_weight=0.2)
            self.flat = self.fused.grads.flat
        else:
            self.means2d = torch.zeros_like(self.means, requires_grad=True)
            self.stage_tgt = [torch.empty_like(t) for t in targets_dev] if targets_host else None
            self.copy_stream = torch.cuda.Stream(device) if targets_host else None
            self.tgt_ready = [None] * len(views)
            self.e2e = False
            self.dp = ViewShardedStep(self.params, range(len(views)), self._view_loss)
            self.flat = self.dp.grads.flat

    def _view_loss(self, i):
        gs = self.gs
        if self.e2e:
            tgt = self.stage_tgt[i]
            self.torch.cuda.current_stream(self.device).wait_event(self.tgt_ready[i])
        else:
            tgt = self.targets_dev[i]
        self.means2d.grad = None
        color, radii, meta = gs.GaussianRasterizer(self.settings[i])(
            self.means, self.means2d, self.opac, shs=self.sh, scales=self.scales, rotations=self.rots)
        l1 = (color - tgt).abs().mean()
        ssim = gs.fused_ssim(color.unsqueeze(0), tgt.unsqueeze(0))
        return l1 + 0.2 * (1.0 - ssim)

    def step(self, e2e: bool = False):
        if self.path == "fused":
            losses = self.fused.step(self.targets_host if e2e else self.targets_dev)[:, 0]
        else:
            self.e2e = e2e
            if e2e:
                # every view's target is copied from pinned host memory on a copy stream at the start of
                # the step, each view waiting only for its own copy (the fused path does the same)
                torch = self.torch
                self.copy_stream.wait_stream(torch.cuda.current_stream(self.device))
                with torch.cuda.stream(self.copy_stream):
                    for i, t in enumerate(self.targets_host):
                        self.stage_tgt[i].copy_(t, non_blocking=True)
                        ev = torch.cuda.Event()
                        ev.record(self.copy_stream)
                        self.tgt_ready[i] = ev
            losses = self.torch.stack(self.dp.step().losses)
        if e2e:
            self.loss_host.copy_(losses, non_blocking=True)
        return losses


def timed(fn, steps, warmup, world):
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        fn()
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
        torch.distributed.barrier()
    return ms


def kernel_profile(trainer, steps=2):
    """CUDA-event timing of each native stage, launched on the current stream."""
    import torch

    from gswarp_b200 import _pipeline

    _pipeline.TIMERS.clear()
    _pipeline.TIMING_ENABLED = True
    fused = getattr(trainer, "fused", None)
    if fused is not None:
        fused.concurrent_views = False  # stage events measure one kernel at a time
    try:
        for _ in range(steps):
            trainer.step()
        torch.cuda.synchronize()
    finally:
        _pipeline.TIMING_ENABLED = False
        if fused is not None:
            fused.concurrent_views = True
    out = {}
    for name, evs in _pipeline.TIMERS.items():
        ts = [a.elapsed_time(b) for a, b, _ in evs]
        out[name] = {"launches": len(ts), "kernels": sum(x.get("kernels", 1) for _, _, x in evs),
                     "total_ms": sum(ts), "mean_ms": sum(ts) / max(len(ts), 1), "extra": [x for _, _, x in evs]}
    _pipeline.TIMERS.clear()
    return out


def measure_cfg2(device, steps, warmup):
    """Single view, benchmark configuration 2: 1M Gaussians SH3 1080p, fwd+bwd raster + L1 + SSIM."""
    import torch

    import gswarp_b200 as gs
    from gswarp_b200 import workloads as wl

    scene = wl.config2_scene(seed=0, n=1_000_000).to(device)
    view = wl.config2_view(seed=0).to(device)
    tgt = wl.target_image(0).to(device)
    out = {"gaussians": 1_000_000, "width": 1920, "height": 1080, "loss": "L1 + 0.2 (1 - SSIM)"}
    for path in ("fused", "autograd"):
        tr = Trainer(scene, [view], [tgt], None, 1, device, path=path)
        ms = timed(tr.step, steps, warmup, 1)
        out[path] = {"views_per_s": 1000.0 * steps / ms, "ms_per_view": ms / steps}
        del tr
    out["views_per_s"] = out["fused"]["views_per_s"]
    return out


def _event_ms(fn, reps, warmup):
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def measure_small_configs(device):
    """Benchmark configurations 1, 3 and 4 through the public API (device-resident
    inputs, CUDA events, mean over repetitions after warm-up)."""
    import torch

    import gswarp_b200 as gs
    from gswarp_b200 import workloads as wl

    out = {}
    # config 1: 10K Gaussians SH0 at 256x256, forward + backward with dL/dcolor ~ N(0,1)
    sc, view = wl.config1_scene(seed=0)
    sc = sc.to(device)
    v = view.to(device)
    rs = gs.GaussianRasterizationSettings(
        image_height=v.height, image_width=v.width, tanfovx=v.tanfovx, tanfovy=v.tanfovy,
        bg=torch.zeros(3, device=device), scale_modifier=1.0, viewmatrix=v.viewmatrix, projmatrix=v.projmatrix,
        sh_degree=0, campos=v.campos, prefiltered=False)
    ps = [t.clone().requires_grad_(True) for t in (sc.means, sc.opacities, sc.sh, sc.scales, sc.rotations)]
    m2d = torch.zeros_like(ps[0], requires_grad=True)
    gcol = torch.randn(3, v.height, v.width, generator=torch.Generator().manual_seed(0)).to(device)

    def cfg1():
        color, _, _ = gs.GaussianRasterizer(rs)(ps[0], m2d, ps[1], shs=ps[2], scales=ps[3], rotations=ps[4])
        color.backward(gcol)

    out["config1_ms"] = _event_ms(cfg1, 50, 5)
    # config 3: fused SSIM forward + backward on 4 x 3 x 1080 x 1920
    img, tgt = wl.config3_images(seed=0)
    img = img.to(device).requires_grad_(True)
    tgt = tgt.to(device)

    def cfg3():
        img.grad = None
        gs.fused_ssim(img, tgt).backward()

    out["config3_ssim_fwd_bwd_ms"] = _event_ms(cfg3, 20, 3)
    del img, tgt
    # config 4: KNN initialiser on 2M clustered points
    pts = wl.config4_points(seed=0).to(device)
    out["config4_knn_ms"] = _event_ms(lambda: gs.distCUDA2(pts), 10, 2)
    return out


def measure_flow(device, steps, warmup):
    """Config 2 through the flow rasterizer (top-K contributor outputs, K=20) against the standard one:
    forward + backward of an L1 loss on the colour, through the public autograd APIs."""
    import torch

    import gswarp_b200.rasterizer as std
    import gswarp_b200.rasterizer_flow as flow
    from gswarp_b200 import workloads as wl

    scene = wl.config2_scene(seed=0, n=1_000_000).to(device)
    v = wl.config2_view(seed=0).to(device)
    tgt = wl.target_image(0).to(device)
    ps = [t.clone().requires_grad_(True) for t in (scene.means, scene.opacities, scene.sh, scene.scales,
                                                    scene.rotations)]
    m2d = torch.zeros_like(ps[0], requires_grad=True)
    out = {"gaussians": 1_000_000, "top_k": flow.get_flow_topk()}
    for name, mod in (("standard", std), ("flow", flow)):
        rs = mod.GaussianRasterizationSettings(
            image_height=v.height, image_width=v.width, tanfovx=v.tanfovx, tanfovy=v.tanfovy,
            bg=torch.zeros(3, device=device), scale_modifier=1.0, viewmatrix=v.viewmatrix, projmatrix=v.projmatrix,
            sh_degree=3, campos=v.campos, prefiltered=False)
        r = mod.GaussianRasterizer(rs)

        def one():
            o = r(ps[0], m2d, ps[1], shs=ps[2], scales=ps[3], rotations=ps[4])
            (o[0] - tgt).abs().mean().backward()

        ms = _event_ms(one, steps, warmup)
        out[name] = {"views_per_s": 1000.0 / ms, "ms_per_view": ms}
    return out


def measure_compute_peaks(device) -> dict:
    """Measured FP32 and MUFU ex2 throughput of this GPU (the denominators of
    the render kernels' compute roofline): the library's gsb_peak_fp32 (packed
    f32x2 FMA chains) and gsb_peak_ex2 microkernels, 8 CTAs per SM, timed with
    CUDA events on the launching stream after warm-up (best of 5)."""
    import torch

    from gswarp_b200 import _lib

    L = _lib.load()
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    blocks = sms * 8
    out = torch.zeros(blocks, device=device)
    res = {"sms": sms}
    for name, fn, which, iters in (("fp32", L.gsb_peak_fp32, 0, 16384), ("ex2", L.gsb_peak_ex2, 1, 8192)):
        def launch():
            _lib.check(fn(blocks, iters, _lib.ptr(out), _lib.stream_handle(device)), name)
        best = min(_event_ms(launch, 1, 2) for _ in range(5))
        work = int(L.gsb_peak_work(which, blocks, iters))
        res[name] = work / (best * 1e-3)
        res[f"{name}_ms"] = best
    return {"fp32_tflops": res["fp32"] / 1e12, "ex2_tops": res["ex2"] / 1e12, "fp32_ms": res["fp32_ms"],
            "ex2_ms": res["ex2_ms"], "sms": sms,
            "how": "gsb_peak_fp32 / gsb_peak_ex2: 8 CTAs per SM of 256 threads, 8 independent chains each "
                   "(packed FFMA2 / MUFU.EX2), CUDA events, best of 5 after warm-up"}


def measure_adam(trainer, peaks):
    """The optimizer step that follows the all-reduce, on the bench's parameters and gradient buffer:
    gswarp_b200.optim.FusedAdam (one pass, 28 B per element) against torch.optim.Adam (foreach)."""
    import torch

    from gswarp_b200.optim import FusedAdam

    lrs = {"means": 1.6e-4, "scales": 5e-3, "rotations": 1e-3, "opacities": 2.5e-2, "sh_dc": 2.5e-3,
           "sh_rest": 1.25e-4}
    params = [p.detach() for p in trainer.params]
    flat = trainer.flat
    fa = FusedAdam(params, flat, lrs)
    ms_fused = _event_ms(fa.step, 10, 3)
    n = flat.numel()
    gbs = 28.0 * n / (ms_fused * 1e-3) / 1e9
    out = {"elements": n, "fused_ms": ms_fused, "fused_gbs": gbs,
           "fused_frac_of_hbm": gbs / peaks.get("hbm_gbs", 6650.0)}
    del fa
    ref = [p.clone().requires_grad_(True) for p in params]
    off = 0
    for t in ref:
        t.grad = flat[off:off + t.numel()].view_as(t)
        off += t.numel()
    opt = torch.optim.Adam([{"params": [t], "lr": 1e-3} for t in ref], lr=1e-3, eps=1e-15)
    out["torch_adam_ms"] = _event_ms(opt.step, 5, 2)
    del opt, ref
    torch.cuda.empty_cache()
    return out


def host_threads() -> int:
    """Host threads available to this process (its CPU affinity)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


class OracleView:
    """One full training view of the benchmark workload through the CPU
    oracle (the C++ restatement of the reference's kernels): preprocess + SH
    colour of every Gaussian, binning, render forward, L1 + 0.2 (1 - SSIM)
    against the view's target, render backward, preprocess + SH backward --
    the same stages as one view of the GPU step, at full 1920x1080."""

    def __init__(self, scene_cpu, views, targets):
        self.arrays = {k: getattr(scene_cpu, k).numpy() for k in ("means", "opacities", "scales", "rotations", "sh")}
        self.views = views
        self.targets = targets
        self.n = scene_cpu.n

    def run(self, i: int) -> None:
        import numpy as np

        import oracle

        v = self.views[i % len(self.views)]
        a = self.arrays
        W, H, P = v.width, v.height, self.n
        vm, pm, cp = v.viewmatrix.cpu().numpy(), v.projmatrix.cpu().numpy(), v.campos.cpu().numpy()
        pre = oracle.preprocess_fwd(a["means"], a["opacities"], vm, pm, v.tanfovx, v.tanfovy, W, H,
                                    scales=a["scales"], rotations=a["rotations"], sh=a["sh"], degree=3, campos=cp)
        pl_, ranges, _ = oracle.binning(pre, W, H)
        col, dep, alp, nc = oracle.render_fwd(W, H, ranges, pl_, pre["proj_2d"], pre["rgb"], pre["depths"],
                                              pre["conic_opacity"], np.zeros(3, np.float32))
        tgt = self.targets[i % len(self.targets)]
        _, _, dm = oracle.ssim_fwd(col[None], tgt[None])
        g_ssim = oracle.ssim_bwd(col[None], tgt[None], dm, -0.2)[0]
        gcol = (np.sign(col - tgt) / col.size + g_ssim).astype(np.float32)
        rb = oracle.render_bwd(W, H, P, ranges, pl_, pre["proj_2d"], pre["rgb"], pre["depths"], pre["conic_opacity"],
                               np.zeros(3, np.float32), alp, nc, gcol, np.zeros_like(dep), np.zeros_like(alp))
        oracle.preprocess_bwd(a["means"], pre["radii"], vm, pm, v.tanfovx, v.tanfovy, W, H, rb,
                              np.zeros((P, 2), np.float32), np.zeros((P, 3), np.float32),
                              np.zeros((P, 3), np.float32), scales=a["scales"], rotations=a["rotations"],
                              sh=a["sh"], degree=3, campos=cp, clamped=pre["clamped"])


def oracle_workload(args, n_views: int):
    from gswarp_b200 import workloads as wl

    scene = wl.config2_scene(seed=0, n=args.gaussians)
    views = wl.ring_views(64, seed=0, width=args.width, height=args.height)[:n_views]
    targets = [wl.target_image(i, args.height, args.width).numpy() for i in range(n_views)]
    return OracleView(scene, views, targets)


def cpu_baseline_sample(args, views_timed: int = 2) -> dict:
    """The oracle on all host threads over ``views_timed`` full views of the
    workload (after one untimed view), wall-clock."""
    import oracle

    cores = oracle.set_num_threads(host_threads())
    ov = oracle_workload(args, views_timed + 1)
    ov.run(views_timed)  # warm-up (first-touch of the oracle's buffers)
    t0 = time.perf_counter()
    for i in range(views_timed):
        ov.run(i)
    dt = time.perf_counter() - t0
    return {"value": views_timed / dt, "unit": "views/s", "cores": cores, "kind": "port",
            "sample": f"{views_timed} full {args.width}x{args.height} views of the workload ({args.gaussians} "
                      f"Gaussians, SH3; preprocess, binning, render, L1+SSIM, render and preprocess backward) "
                      f"through the oracle after one untimed view: {dt:.2f} s wall"}


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of each kernel at the default
# workload (6M Gaussians, 1920x1080, first view of the training step), from a 1-pass ncu capture of
# `python bench.py --steps 1 --warmup 1 --no-e2e --no-autograd --no-cfg2 --no-cpu-baseline --no-optimizer`.
MEASURED_TRAFFIC = {
    "render_bwd": 262.87e6 + 33.48e6,
    "render_fwd": 163.27e6 + 31.64e6,
    "preprocess_bwd": 1140.62e6 + 451.03e6,
    "preprocess_fwd": 380.36e6 + 331.54e6,
    "sh_colors": 1224.03e6 + 544.67e6,
}


# Algorithmic work per stage and view (fixed formulas; fp32/int32 = 4 B): N Gaussians, V of them binned (with
# tiles), R tile-Gaussian pairs, E pixel-Gaussian pairs up to each pixel's last contributor, T tiles, P_px
# pixels, M = 3 * P_px SSIM elements, `views` views per step.  Bytes are the minimum each stage must move
# through HBM; render FLOP per pair are the reference's per-pair arithmetic (28 forward, 70 backward) with one
# ex2 each; SSIM 336 FLOP per element.
# The fused multi-view step (fused=True): preprocess reads mean + opacity of every Gaussian and writes its
# radius, depth and tile count (28 B); a binned Gaussian also reads scale, rotation and its SH colour (40 B)
# and writes its render and binning records (80 B); the step's SH colour pass reads each SH row and mean once
# (204 B per step) and writes a colour per view (12 B).  Preprocess backward, per binned Gaussian: id, radius,
# mean, scale, rotation and clamp bits in (48 B), the render-gradient accumulator read and cleared (96 B), the
# 11 gradient floats of the flat buffer and the view's 3 colour-gradient floats read and written (112 B); the
# step's SH backward reads each SH row, mean and the views' colour gradients and writes the SH gradient and
# the means gradient (420 B per step over its views, plus 24 B per view for the colour gradients).
# The per-view autograd path (fused=False) evaluates SH and writes dense gradients for every Gaussian.
def stage_work(stage: str, N: int, R: int, E: int, T: int, P_px: int, V: int | None = None, views: int = 1,
               fused: bool = True) -> dict:
    M = 3 * P_px
    V = N if V is None else V
    if fused:
        pre_fwd = 28 * N + 120 * V + (204.0 / views + 12) * N
        pre_bwd = 260 * V + (420.0 / views + 24) * N
    else:
        pre_fwd, pre_bwd = 316 * N, 528 * N
    return {
        "preprocess_fwd": {"bytes": pre_fwd},
        # scan (8N) + emit (12R) + sort lower bound (24R) + point list (8R) + ranges (8T)
        "binning": {"bytes": 8 * N + 44 * R + 8 * T},
        "render_fwd": {"bytes": 44 * R + 24 * P_px, "flop": 28 * E, "ex2": E},
        "ssim_l1": {"bytes": 20 * M, "flop": 336 * M},
        "render_bwd": {"bytes": 44 * R + 28 * P_px + 40 * V, "flop": 70 * E, "ex2": E},
        "preprocess_bwd": {"bytes": pre_bwd},
    }[stage]


def bound_time(work: dict, peaks: dict, compute: dict) -> tuple[float, str]:
    """(seconds, bound) = the largest of bytes / HBM, FLOP / FP32, ex2 / MUFU."""
    t = {"hbm": work.get("bytes", 0) / (peaks.get("hbm_gbs", 6650.0) * 1e9)}
    if compute:
        t["fp32"] = work.get("flop", 0) / (compute["fp32_tflops"] * 1e12)
        t["mufu"] = work.get("ex2", 0) / (compute["ex2_tops"] * 1e12)
    b = max(t, key=t.get)
    return t[b], b


def roofline(prof, peaks, compute, pixels, N, tiles, workload_is_default=False):
    """Roofline of the dominant native kernel (by total time): its algorithmic
    work per launch (stage_work) against the measured peaks of the bound that
    work implies (HBM copy bandwidth, the FP32 / MUFU microkernels)."""
    if not prof:
        return None
    name, rec = max(prof.items(), key=lambda kv: kv[1]["total_ms"])
    mean_s = rec["mean_ms"] / 1000.0
    extra = rec["extra"][0] if rec["extra"] else {}
    R = extra.get("num_rendered", 0)
    E = extra.get("pairs", 0)
    V = extra.get("binned", extra.get("P", N))
    stage = {"bin_count": "binning", "bin_emit_sort": "binning", "loss_fwd": "ssim_l1",
             "loss_bwd": "ssim_l1"}.get(name, name)
    try:
        work = stage_work(stage, N, R, E, tiles, pixels, V=V)
    except KeyError:
        return {"kernel": name, "mean_launch_ms": rec["mean_ms"], "note": "no algorithmic model for this stage"}
    t_bound, bound = bound_time(work, peaks, compute)
    hbm_peak = peaks.get("hbm_gbs", 6650.0)
    traffic = MEASURED_TRAFFIC.get(name) if workload_is_default else None
    out = {"kernel": name, "bound": bound, "mean_launch_ms": round(rec["mean_ms"], 4),
           "roofline_ms": round(t_bound * 1e3, 4), "traffic": traffic,
           "algorithmic_bytes_per_launch": work.get("bytes"), "pairs": E or None}
    if bound == "fp32":
        out.update(achieved=round(work["flop"] / mean_s / 1e12, 3), peak=round(compute["fp32_tflops"], 2),
                   unit="TFLOP/s", peak_source="measured in this run (gsb_peak_fp32 microkernel)",
                   algorithmic_flop_per_launch=work["flop"])
    elif bound == "mufu":
        out.update(achieved=round(work["ex2"] / mean_s / 1e12, 3), peak=round(compute["ex2_tops"], 3),
                   unit="Tex2/s", peak_source="measured in this run (gsb_peak_ex2 microkernel)")
    else:
        out.update(achieved=round(work["bytes"] / mean_s / 1e9, 2), peak=hbm_peak, unit="GB/s",
                   peak_source=peaks.get("_source", "measured"))
    out["frac"] = round(out["achieved"] / out["peak"], 4) if out["peak"] else None
    # the same kernel against HBM too (its DRAM traffic per launch is `traffic`)
    out["hbm"] = {"achieved_gbs": round(work.get("bytes", 0) / mean_s / 1e9, 2), "peak_gbs": hbm_peak,
                  "frac": round(work.get("bytes", 0) / mean_s / 1e9 / hbm_peak, 4)}
    if compute and work.get("ex2"):
        out["mufu_frac"] = round(work["ex2"] / mean_s / 1e12 / compute["ex2_tops"], 4)
    return out


def step_roofline(prof, peaks, compute, N, pixels, tiles, views, ms_per_step, world, ar_gbs=770.0, fused=True):
    """Per-view roofline of the whole step: the sum over its stages of
    max(bytes / HBM, FLOP / FP32, ex2 / MUFU) (stage_work, with each view's
    measured R and E), plus at N > 1 the all-reduce's per-GPU ring traffic
    2(n-1)/n * 236 B * N over NVLink per step (770 GB/s per direction, the
    measured peer copy), against the measured time per view."""
    rb = prof.get("render_bwd", {}).get("extra", [])
    rf = prof.get("render_fwd", {}).get("extra", [])
    if not rb or not rf:
        return None
    stages = {}
    per_view = []
    for k in range(len(rb)):
        R = rb[k].get("num_rendered", 0)
        E = rf[k].get("pairs", 0) if k < len(rf) else 0
        V = rb[k].get("binned", N)
        t = 0.0
        for st in ("preprocess_fwd", "binning", "render_fwd", "ssim_l1", "render_bwd", "preprocess_bwd"):
            tt, b = bound_time(stage_work(st, N, R, E, tiles, pixels, V=V, views=views, fused=fused), peaks, compute)
            stages.setdefault(st, []).append((tt, b))
            t += tt
        per_view.append(t)
    t_view = sum(per_view) / len(per_view)
    ar = 0.0
    if world > 1:
        ar = 2.0 * (world - 1) / world * 4 * FLOATS_PER_GAUSSIAN * N / (ar_gbs * 1e9) / views
    measured = ms_per_step / 1e3 / views
    return {"roofline_ms_per_view": round((t_view + ar) * 1e3, 4), "measured_ms_per_view": round(measured * 1e3, 4),
            "frac": round((t_view + ar) / measured, 4),
            "stages_ms": {k: round(sum(x for x, _ in v) / len(v) * 1e3, 4) for k, v in stages.items()},
            "stage_bounds": {k: v[0][1] for k, v in stages.items()},
            "allreduce_ms": round(ar * 1e3, 4),
            "how": "sum over stages of max(bytes/HBM, FLOP/FP32, ex2/MUFU) per view (measured peaks) over the "
                   "measured device time per view"}


def measure_autograd(args, scene, views, targets_dev, targets_host, world, device, views_total):
    """The drop-in path (GaussianRasterizer + fused_ssim under autograd) on the same workload."""
    import torch

    tr_ag = Trainer(scene, views, targets_dev, targets_host, world, device, path="autograd")
    ms_ag = timed(tr_ag.step, args.steps, args.warmup, world)
    out = {"value": 1000.0 * views_total / ms_ag, "unit": "views/s",
           "path": "GaussianRasterizer + fused_ssim under autograd, ViewShardedStep"}
    if not args.no_e2e:
        ms_ag_e2e = timed(lambda: tr_ag.step(e2e=True), args.steps, 1, world)
        out["e2e"] = 1000.0 * views_total / ms_ag_e2e
    del tr_ag
    torch.cuda.empty_cache()
    return out


def run_reference(args):
    """The reference arm: gswarp needs warp-lang, which this image lacks, so
    the CPU restatement of its kernels (oracle/) runs the workload on all host
    threads.  A step is one full 1920x1080 view (the GPU arm's step is
    views_per_gpu of them); W untimed steps, then K timed ones, wall-clock.
    Under torchrun only rank 0 runs."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle

    cores = oracle.set_num_threads(host_threads())
    ov = oracle_workload(args, min(args.steps + args.warmup, 64))
    for i in range(args.warmup):
        ov.run(args.steps + i)
    times = []
    for i in range(args.steps):
        t0 = time.perf_counter()
        ov.run(i)
        times.append(time.perf_counter() - t0)
    ms = 1000.0 * sum(times) / len(times)
    v = 1000.0 / ms
    sample = (f"per step one full {args.width}x{args.height} view of the workload ({args.gaussians} Gaussians, SH3): "
              "preprocess, binning, render, L1+SSIM, render and preprocess backward through the oracle")
    line = {"metric": METRIC, "value": v, "unit": "views/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": f"config5: {args.gaussians} Gaussians SH3, {args.width}x{args.height}, "
                                   "L1+0.2(1-SSIM), fwd+bwd; one view per step",
                       "gaussians": args.gaussians},
            "cpu_baseline": {"value": v, "unit": "views/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": "views/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "step_ms": [round(1000.0 * t, 1) for t in times],
            "note": "gswarp needs warp-lang, absent from this image; the reference arm runs the C++ restatement "
                    "of its kernels (oracle/, pinned to the reference's own kernel code by golden vectors) on "
                    "all host threads"}
    print(json.dumps(line), flush=True)


def measure_allreduce(flat, world: int, reps: int = 5) -> dict:
    """The step's exchange alone: NCCL all-reduce (sum) of the flat gradient
    buffer, CUDA events on the current stream, max over ranks; bus bandwidth
    2(n-1)/n * bytes / time."""
    import torch

    nbytes = flat.numel() * flat.element_size()
    for _ in range(2):
        torch.distributed.all_reduce(flat)
    torch.cuda.synchronize()
    torch.distributed.barrier()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        torch.distributed.all_reduce(flat)
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / reps], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = float(t.item())
    bus = 2.0 * (world - 1) / world * nbytes / (ms * 1e-3) / 1e9
    env = {k: os.environ[k] for k in ("NCCL_ALGO", "NCCL_PROTO", "NCCL_NVLS_ENABLE") if k in os.environ}
    return {"bytes": nbytes, "ms": round(ms, 4), "busbw_gbs": round(bus, 1), "nccl_version": ".".join(
        str(x) for x in torch.cuda.nccl.version()), "env": env or "NCCL defaults"}


def nccl_algorithms(path) -> dict | str:
    """Algorithm, protocol and channels NCCL chose per all-reduce size, from
    its tuning log lines ("AllReduce: <bytes> Bytes -> Algo <a> proto <p>
    channel{Lo..Hi}={lo..hi}")."""
    import re

    if not path or not os.path.exists(path):
        return "not recorded (NCCL debug output configured by the caller)"
    pat = re.compile(r"AllReduce: (\d+) Bytes -> Algo (\w+) proto (\w+) channel\{Lo\.\.Hi\}=\{(\d+)\.\.(\d+)\}")
    seen = {}
    with open(path, errors="replace") as f:
        for line in f:
            m = pat.search(line)
            if m:
                seen[int(m.group(1))] = f"{m.group(2)}/{m.group(3)}/{int(m.group(5)) - int(m.group(4)) + 1}ch"
    big = sorted(seen, reverse=True)[:8]
    return {str(k): seen[k] for k in big} or "no tuning lines"


def dp_check(device, rank: int, world: int) -> dict:
    """Correctness of the data-parallel step on this job's ranks (outside the
    timed region): each rank renders its own 2 views of a 30K-Gaussian scene;
    the overlapped reduction (SH ranges all-reduced while the SH backward
    runs) must equal a rank-local step followed by one plain all-reduce of its
    flat buffer, block by block within 1e-4 relative (the render backward's
    atomics order the float sums differently run to run), and every rank must
    hold the same reduced buffer."""
    import torch
    import torch.distributed as dist

    import gswarp_b200 as gs
    from gswarp_b200 import workloads as wl
    from gswarp_b200.training import FusedViewStep

    singles = [dist.new_group(ranks=[r]) for r in range(world)]
    sc = wl.config2_scene(seed=5, n=30_000)
    cams = wl.ring_views(2 * world, seed=5, width=320, height=192)[2 * rank: 2 * rank + 2]
    params = [t.to(device).contiguous() for t in (sc.means, sc.scales, sc.rotations, sc.opacities, sc.sh)]
    bg = torch.zeros(3, device=device)
    settings = [gs.GaussianRasterizationSettings(
        image_height=v.height, image_width=v.width, tanfovx=v.tanfovx, tanfovy=v.tanfovy, bg=bg,
        scale_modifier=1.0, viewmatrix=v.viewmatrix.to(device), projmatrix=v.projmatrix.to(device), sh_degree=3,
        campos=v.campos.to(device), prefiltered=False) for v in cams]
    targets = [wl.target_image(100 + 2 * rank + i, 192, 320).to(device) for i in range(2)]
    overlapped = FusedViewStep([p.clone() for p in params], settings, batch_sh=True)
    overlapped.step(targets)
    local = FusedViewStep([p.clone() for p in params], settings, batch_sh=True, group=singles[rank])
    local.step(targets)
    summed = local.grads.flat.clone()
    dist.all_reduce(summed)
    got = overlapped.grads.flat
    first = got.clone()
    dist.broadcast(first, src=0)
    torch.cuda.synchronize()
    worst = 0.0
    off = 0
    for p in params:
        k = p.numel()
        x, y = got[off:off + k], summed[off:off + k]
        worst = max(worst, float((x - y).norm()) / (float(y.norm()) + 1e-30))
        off += k
    same = bool(torch.equal(first, got))
    other = float((got - local.grads.flat).norm()) / (float(got.norm()) + 1e-30)
    flags = torch.tensor([worst, 0.0 if same else 1.0, other], dtype=torch.float64, device=device)
    dist.all_reduce(flags, op=dist.ReduceOp.MAX)
    worst, differs, other = (float(v) for v in flags.tolist())
    ok = worst <= 1e-4 and differs == 0.0 and other > 1e-3
    return {"max_rel_block": worst, "ranks_identical": differs == 0.0, "other_ranks_contributed": other > 1e-3,
            "ok": ok, "how": "overlapped multi-view-SH reduction vs rank-local step + one all_reduce, "
                             "30K Gaussians, 2 views per rank at 320x192"}


def measure_reference_workloads(device) -> dict:
    """The reference's published microbenchmark workloads (docs/rasterizer.md:311-315, RTX 5090, Warp),
    with its input recipe (benchmarks/rasterizer_microbench.py:57-105: means U[-0.65,0.65]^2 x U[2,3],
    colours U[0,1], opacity U[0.1,0.9], scales U[0.025,0.06], identity rotation, identity view/proj,
    tanfov 1, background (0.05, 0.15, 0.25)) through gswarp_b200.GaussianRasterizer, CUDA events.
    Context only: another GPU, another process."""
    import torch

    import gswarp_b200 as gs

    def inputs(count, sh_degree):
        g = torch.Generator(device=device).manual_seed(count)
        m = torch.empty((count, 3), device=device)
        m[:, :2].uniform_(-0.65, 0.65, generator=g)
        m[:, 2].uniform_(2.0, 3.0, generator=g)
        col = torch.rand((count, 3), device=device, generator=g)
        op = torch.empty((count, 1), device=device).uniform_(0.1, 0.9, generator=g)
        sc = torch.empty((count, 3), device=device).uniform_(0.025, 0.06, generator=g)
        rot = torch.zeros((count, 4), device=device)
        rot[:, 0] = 1.0
        sh = None
        if sh_degree:
            sh = torch.randn((count, 16, 3), device=device, generator=g) * 0.1
            sh[:, 0, :] = col
        leaves = [m, col, op, sc, rot] + ([sh] if sh is not None else [])
        return [t.requires_grad_(True) for t in leaves]

    def settings(side, sh_degree):
        return gs.GaussianRasterizationSettings(
            image_height=side, image_width=side, tanfovx=1.0, tanfovy=1.0,
            bg=torch.tensor((0.05, 0.15, 0.25), device=device), scale_modifier=1.0,
            viewmatrix=torch.eye(4, device=device), projmatrix=torch.eye(4, device=device), sh_degree=sh_degree,
            campos=torch.zeros(3, device=device), prefiltered=False)

    out = {}
    for count, side, ref_ms in ((256 * 1024, 384, 2.215), (1024 * 1024, 640, 4.733)):
        m, col, op, sc, rot = inputs(count, 0)
        m2 = torch.zeros_like(m, requires_grad=True)
        r = gs.GaussianRasterizer(settings(side, 0))

        def step():
            color, radii, meta = r(m, m2, op, colors_precomp=col, scales=sc, rotations=rot)
            loss = (color.square().mean() + meta.alpha.mean() + 0.01 * meta.depth.mean()
                    + 1e-4 * (meta.proj_2D.square().mean() + meta.conic_2D.sum() + meta.conic_2D_inv.sum()))
            loss.backward()

        ms = _event_ms(step, 100, 20)
        out[f"{count // 1024}K_{side}x{side}_fwd_bwd_rgb"] = {"ms": round(ms, 4), "reference_warp_rtx5090_ms": ref_ms}
    m, col, op, sc, rot, sh = inputs(300_000, 3)
    m2 = torch.zeros_like(m, requires_grad=True)
    color, radii, meta = gs.GaussianRasterizer(settings(800, 3))(m, m2, op, shs=sh, scales=sc, rotations=rot)
    gout = torch.randn_like(color)
    ms = _event_ms(lambda: torch.autograd.grad(color, [m, op, sh, sc, rot], gout, retain_graph=True), 100, 20)
    out["300K_800x800_sh3_raster_backward"] = {"ms": round(ms, 4), "reference_warp_rtx5090_ms": 1.638,
                                               "visible": int((radii > 0).sum())}
    out["note"] = ("context only: the reference's published RTX 5090 figures for the same input recipe "
                   "(docs/rasterizer.md:311-315); not a comparison on the same GPU")
    return out


def run_ours(args):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    nccl_log = None
    if world > 1:
        if "NCCL_DEBUG_FILE" not in os.environ and os.environ.get("NCCL_DEBUG", "").upper() not in ("INFO", "TRACE"):
            # NCCL's tuning lines (to a file) name the algorithm and protocol of every collective
            nccl_log = f"/tmp/gsb_bench_nccl.{os.getpid()}.log"
            os.environ.update(NCCL_DEBUG="INFO", NCCL_DEBUG_SUBSYS="TUNING", NCCL_DEBUG_FILE=nccl_log)
        torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    from gswarp_b200 import workloads as wl
    from gswarp_b200 import _pipeline

    peaks = {}
    pk = ROOT / "MEASURED_PEAKS.json"
    if pk.exists():
        peaks = json.loads(pk.read_text())
        peaks["_source"] = "measured (MEASURED_PEAKS.json)"
    else:
        peaks = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "_source": "fallback"}

    scene, views = make_scene(args, device, rank)
    V = len(views)
    targets_dev = [wl.target_image(rank * V + i, args.height, args.width).to(device) for i in range(V)]
    targets_host = [t.cpu().pin_memory() for t in targets_dev] if not args.no_e2e else None
    tr = Trainer(scene, views, targets_dev, targets_host, world, device, path=args.path)
    if args.path == "fused":
        tr.fused.range_backward = args.backward_order == "ranges"
        if args.deferred_views is not None:
            tr.fused.deferred_views = args.deferred_views

    # device-resident timing with clock sampling
    sampler = ClockSampler(local)
    sampler.start()
    ms = timed(tr.step, args.steps, args.warmup, world)
    clocks = sampler.stop()
    views_total = V * world * args.steps
    value = 1000.0 * views_total / ms

    e2e = None
    if not args.no_e2e:
        ms_e2e = timed(lambda: tr.step(e2e=True), args.steps, 1, world)
        img_bytes = sum(t.numel() * 4 for t in targets_host)
        e2e = {"value": 1000.0 * views_total / ms_e2e, "unit": "views/s", "h2d_bytes_per_step": img_bytes,
               "d2h_bytes_per_step": V * 4}

    # the drop-in autograd path on the same workload, for comparison
    autograd_api = None
    if not args.no_autograd and args.path == "fused":
        autograd_api = measure_autograd(args, scene, views, targets_dev, targets_host, world, device, views_total)

    tr_ranged = args.path == "fused" and tr.fused.batch_sh and bool(tr.fused.range_backward)
    tr_deferred = (V if tr_ranged else min(V, int(tr.fused.deferred_views))) \
        if args.path == "fused" and tr.fused.batch_sh else 0
    prof = kernel_profile(tr, steps=1)
    launches = sum(v["kernels"] for v in prof.values())
    default = (args.gaussians, args.width, args.height) == (6_000_000, 1920, 1080)
    compute = measure_compute_peaks(device)
    pixels = args.width * args.height
    tiles = ((args.width + 15) // 16) * ((args.height + 15) // 16)
    rl = roofline(prof, peaks, compute, pixels, scene.n, tiles, workload_is_default=default)
    step_rl = step_roofline(prof, peaks, compute, scene.n, pixels, tiles, V, ms / args.steps, world,
                            fused=args.path == "fused")

    extra = {}
    if world > 1:
        extra["allreduce"] = measure_allreduce(tr.flat, world)
        extra["allreduce"]["nccl_algorithms"] = nccl_algorithms(nccl_log)
        extra["dp_check"] = dp_check(device, rank, world)
    if rank == 0 and world == 1:
        if not args.no_optimizer:
            extra["optimizer"] = measure_adam(tr, peaks)
        del tr
        torch.cuda.empty_cache()
        if not args.no_cfg2:
            extra["config2_single_view"] = measure_cfg2(device, max(3, args.steps), max(3, args.warmup))
            extra["other_configs"] = measure_small_configs(device)
            extra["flow_config2"] = measure_flow(device, max(3, args.steps), max(3, args.warmup))
            extra["reference_workloads"] = measure_reference_workloads(device)
        if not args.no_cpu_baseline:
            extra["cpu_baseline"] = cpu_baseline_sample(args)
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "views/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"config5: {args.gaussians} Gaussians SH3, {args.width}x{args.height}, "
                                   f"{args.views_per_gpu} views/GPU, L1+0.2(1-SSIM) fwd+bwd, NCCL all-reduce "
                                   f"of {FLOATS_PER_GAUSSIAN} floats/Gaussian",
                       "gaussians": args.gaussians, "views_per_gpu": args.views_per_gpu,
                       "parallelism": f"dp{world} (view-sharded)",
                       "l2": "inputs larger than L2 (6M-Gaussian scene, 1.4 GB of parameters)"},
            "clocks": clocks,
            "e2e": e2e,
            "path": ("gswarp_b200.training.FusedViewStep (C ABI stages, fused photometric loss, preprocess "
                     "backward accumulating into the flat gradient buffer)" if args.path == "fused" else
                     "GaussianRasterizer + fused_ssim under autograd, ViewShardedStep"),
            "backward_order": (("ranges" if tr_ranged else "views") if args.path == "fused" else None),
            "deferred_views": tr_deferred,
            "autograd_api": autograd_api,
            "gpu_launches": launches * args.steps,
            "roofline": rl,
            "step_roofline": step_rl,
            "compute_peaks": compute,
            "kernels": {k: {kk: vv for kk, vv in v.items() if kk != "extra"} for k, v in prof.items()},
        }
        line.update(extra)
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
