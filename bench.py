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
    return p.parse_args()


# ---------------------------------------------------------------------------
# clocks sampling during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
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
                "reasons": sorted(reasons), "samples": len(sm)}


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
            self.e2e = False
            self.dp = ViewShardedStep(self.params, range(len(views)), self._view_loss)
            self.flat = self.dp.grads.flat

    def _view_loss(self, i):
        gs = self.gs
        if self.e2e:
            tgt = self.stage_tgt[i]
            tgt.copy_(self.targets_host[i], non_blocking=True)
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


def cpu_baseline_sample(views, scene_cpu, band_rows=136):
    """Times the CPU oracle (all host threads) on one view of the workload:
    preprocess + binning of every Gaussian, then render, render backward, SSIM
    and preprocess backward on a centred band of `band_rows` image rows
    (1/8 of 1080); views/sec is extrapolated by the band's share of pixels."""
    import numpy as np

    import oracle

    v = views[0]
    W = v.width
    Hb = band_rows
    tanfovy_b = v.tanfovy * Hb / v.height
    from gswarp_b200 import workloads as wl

    vb = wl.look_at_view(v.campos.cpu().double().tolist(), [0.0, 0.0, 0.0], [0.0, 0.0, 1.0],
                         math.degrees(2 * math.atan(v.tanfovx)), W, Hb)
    # same camera, centred band: identical focal length, reduced height
    assert abs(vb.tanfovy - tanfovy_b) < 1e-9
    sc = scene_cpu
    t0 = time.perf_counter()
    pre = oracle.preprocess_fwd(sc.means.numpy(), sc.opacities.numpy(), vb.viewmatrix.numpy(), vb.projmatrix.numpy(),
                                vb.tanfovx, vb.tanfovy, W, Hb, scales=sc.scales.numpy(),
                                rotations=sc.rotations.numpy(), sh=sc.sh.numpy(), degree=3,
                                campos=vb.campos.numpy())
    pl_, ranges, _ = oracle.binning(pre, W, Hb)
    col, dep, alp, nc = oracle.render_fwd(W, Hb, ranges, pl_, pre["proj_2d"], pre["rgb"], pre["depths"],
                                          pre["conic_opacity"], np.zeros(3, np.float32))
    tgt = np.random.default_rng(0).uniform(0, 1, col.shape).astype(np.float32)
    ssim, _, dm = oracle.ssim_fwd(col[None], tgt[None])
    g_ssim = oracle.ssim_bwd(col[None], tgt[None], dm, -0.2)[0]
    gcol = (np.sign(col - tgt) / col.size + g_ssim).astype(np.float32)
    rb = oracle.render_bwd(W, Hb, sc.n, ranges, pl_, pre["proj_2d"], pre["rgb"], pre["depths"], pre["conic_opacity"],
                           np.zeros(3, np.float32), alp, nc, gcol, np.zeros_like(dep), np.zeros_like(alp))
    P = sc.n
    oracle.preprocess_bwd(sc.means.numpy(), pre["radii"], vb.viewmatrix.numpy(), vb.projmatrix.numpy(), vb.tanfovx,
                          vb.tanfovy, W, Hb, rb, np.zeros((P, 2), np.float32), np.zeros((P, 3), np.float32),
                          np.zeros((P, 3), np.float32), scales=sc.scales.numpy(), rotations=sc.rotations.numpy(),
                          sh=sc.sh.numpy(), degree=3, campos=vb.campos.numpy(), clamped=pre["clamped"])
    dt = time.perf_counter() - t0
    frac = Hb / v.height
    return {"value": frac / dt, "unit": "views/s", "cores": oracle.num_threads(), "kind": "port",
            "sample": f"one {sc.n}-Gaussian SH3 view: preprocess+binning of all Gaussians, render/backward/SSIM "
                      f"on a centred {W}x{Hb} band ({frac:.3f} of the pixels); views/s = pixel share / "
                      f"{dt:.2f} s wall"}


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of each kernel at the default
# workload (6M Gaussians, 1920x1080, first view of the training step), from a 1-pass ncu capture of
# `python bench.py --steps 1 --warmup 1 --no-e2e --no-autograd --no-cfg2 --no-cpu-baseline --no-optimizer`.
MEASURED_TRAFFIC = {
    "render_bwd": 262.64e6 + 31.48e6,
    "render_fwd": 163.58e6 + 31.18e6,
    "preprocess_bwd": 1136.76e6 + 450.03e6,
    "preprocess_fwd": 379.93e6 + 336.40e6,
    "sh_colors": 1224.03e6 + 544.70e6,
}


def roofline(prof, peaks, pixels, N, workload_is_default=False):
    """Roofline of the dominant native kernel (by total time)."""
    if not prof:
        return None
    name, rec = max(prof.items(), key=lambda kv: kv[1]["total_ms"])
    mean_s = rec["mean_ms"] / 1000.0
    extra = rec["extra"][0] if rec["extra"] else {}
    R = extra.get("num_rendered", 0)
    E = extra.get("pairs", 0)
    P = extra.get("P", N)
    # algorithmic bytes per launch: per-unit bytes the stage must move x units
    V = extra.get("binned", P)
    per_launch = {
        # pair id + 48-B record per pair; n_contrib, final alpha, colour grad per pixel; 48-B accumulator per
        # binned Gaussian, read and written
        "render_bwd": 52 * R + 20 * pixels + 96 * V,
        # pair id + record per pair; colour, alpha, depth, n_contrib per pixel
        "render_fwd": 52 * R + 24 * pixels,
        "preprocess_fwd": 316 * P,
        # accumulate mode: 288 B read + 236 B read-modify-written per visible Gaussian, 4 B (radius) otherwise
        "preprocess_bwd": 760 * extra.get("visible", P) + 4 * (P - extra.get("visible", P)),
        "binning": 8 * P + 12 * R + 24 * R + 8 * R,
        "loss_fwd": 60 * pixels,
        "loss_bwd": 72 * pixels,
    }.get(name, 0)
    peak = peaks.get("hbm_gbs", 6650.0)
    achieved = per_launch / mean_s / 1e9 if mean_s > 0 else 0.0
    traffic = MEASURED_TRAFFIC.get(name) if workload_is_default else None
    out = {"kernel": name, "bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
           "frac": round(achieved / peak, 4) if peak else None, "traffic": traffic,
           "mean_launch_ms": round(rec["mean_ms"], 4), "algorithmic_bytes_per_launch": per_launch,
           "peak_source": peaks.get("_source", "measured")}
    if name in ("render_bwd", "render_fwd") and E:
        flop = (70 if name == "render_bwd" else 28) * E
        fp32_peak = 148 * 128 * 2 * 1.965e9 / 1e12
        out["compute"] = {"bound": "fp32", "achieved_tflops": round(flop / mean_s / 1e12, 3),
                          "peak_tflops": round(fp32_peak, 1), "peak_source": "nominal (not measured)",
                          "frac": round(flop / mean_s / 1e12 / fp32_peak, 4), "pairs": E}
    return out


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
    """CPU restatement of the reference's kernels (warp-lang is absent)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch

    from gswarp_b200 import workloads as wl
    import oracle

    scene = wl.config2_scene(seed=0, n=args.gaussians)
    views = wl.ring_views(64, seed=0, width=args.width, height=args.height)[:1]
    for _ in range(max(0, min(args.warmup, 1))):
        pass  # CPU code has no JIT or cache warm-up to do
    vals = [cpu_baseline_sample(views, scene)["value"] for _ in range(max(1, args.steps))]
    v = statistics.median(vals)
    sample = cpu_baseline_sample.__doc__.split(":")[0]
    line = {"metric": METRIC, "value": v, "unit": "views/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 / v, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": "config5: 6M Gaussians SH3, 1920x1080, L1+0.2(1-SSIM), fwd+bwd",
                       "gaussians": args.gaussians},
            "cpu_baseline": {"value": v, "unit": "views/s", "cores": oracle.num_threads(), "kind": "port",
                             "sample": "per step one view of the workload: preprocess+binning of all Gaussians, "
                                       "render/backward/SSIM on a centred 1920x136 band, views/s by pixel share"},
            "e2e": {"value": v, "unit": "views/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "gswarp needs warp-lang, absent from this image; the reference arm runs the C++ restatement "
                    "of its kernels (oracle/) on all host cores"}
    print(json.dumps(line), flush=True)


def run_ours(args):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
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
    tr = Trainer(scene, views, targets_dev, targets_host, world, device)

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
    if not args.no_autograd:
        autograd_api = measure_autograd(args, scene, views, targets_dev, targets_host, world, device, views_total)

    prof = kernel_profile(tr, steps=1)
    launches = sum(v["kernels"] for v in prof.values())
    default = (args.gaussians, args.width, args.height) == (6_000_000, 1920, 1080)
    rl = roofline(prof, peaks, args.width * args.height, scene.n, workload_is_default=default)

    extra = {}
    if rank == 0 and world == 1:
        if not args.no_optimizer:
            extra["optimizer"] = measure_adam(tr, peaks)
        del tr
        torch.cuda.empty_cache()
        if not args.no_cfg2:
            extra["config2_single_view"] = measure_cfg2(device, max(3, args.steps), max(3, args.warmup))
            extra["other_configs"] = measure_small_configs(device)
            extra["flow_config2"] = measure_flow(device, max(3, args.steps), max(3, args.warmup))
        if not args.no_cpu_baseline:
            scene_cpu = wl.config2_scene(seed=0, n=args.gaussians)
            extra["cpu_baseline"] = cpu_baseline_sample([views[0]], scene_cpu)
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
            "path": "gswarp_b200.training.FusedViewStep (C ABI stages, fused photometric loss, preprocess "
                    "backward accumulating into the flat gradient buffer)",
            "autograd_api": autograd_api,
            "gpu_launches": launches * args.steps,
            "roofline": rl,
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
