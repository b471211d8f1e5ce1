"""Fused multi-view training step: the 3DGS hot path with no autograd glue.

The drop-in path (``GaussianRasterizer`` + ``fused_ssim`` under autograd)
runs every kernel of the hot path, but autograd adds work between them:
each view's per-Gaussian gradients come back as fresh tensors that
``AccumulateGrad`` then adds into the parameters' ``.grad`` (a full extra
read-read-write of 59 floats per Gaussian per view), unused outputs get
zero-filled gradients, and the L1 term is a chain of elementwise kernels.

``FusedViewStep`` runs the same stages through the C ABI directly, per view:

    preprocess -> binning -> render -> photometric loss fwd+bwd
               -> render backward -> preprocess backward

with the loss ``w_l1 * L1 + w_ssim * (1 - SSIM)`` (the loss the reference's
SSIM documentation pairs its fused SSIM with, gswarp docs/ssim.md:22, :91)
computed by one forward and one backward kernel pass, and with preprocess
backward ADDING each view's gradients straight into the flat gradient buffer
(``accumulate`` mode of ``gsb_preprocess_bwd``), whose SoA blocks are the
parameters' ``.grad``.  After the rank's views it takes part in one sum
all-reduce of that buffer, as ``view_sharding.ViewShardedStep`` does.

With more than one view (``batch_sh``, the default then), the SH work is
done once per step instead of once per view: every view renders the same
parameters, so one pass evaluates all the views' SH colours (reading each
SH row once), the views' preprocess reads 12-byte colours instead of
192-byte SH rows, their backward writes the clamped colour gradient, and
one pass after the last view turns those into the SH gradient and the
view-direction part of the means gradient.  Per view that removes one SH
read in the forward and an SH read plus an SH-gradient read-modify-write in
the backward for every visible Gaussian.

With a process group the multi-view step all-reduces the blocks that are
complete after the last view while the SH backward runs, and the SH rows
range by range as they are produced (``sh_reduce_chunks``).  A
range-ordered backward (``range_backward``) is also available: each view
stops after its render backward (into its own 48-byte-per-Gaussian
accumulator), and the views' preprocess backward then runs one Gaussian
range at a time -- per range, every view's accumulating preprocess backward
over its binned ids inside the range (the same kernel and the same
per-Gaussian order of additions as view by view, so the same bits), then
the SH backward of the range -- so that each finished range is all-reduced
while the next is computed.  It is off by default: it gives up the overlap
of each view's preprocess backward with the next view's forward, and on 2
GPUs that cost as much as the exchange it hid.

Gradients equal the autograd path's up to the float summation order of the
render backward's atomics (tests compare the two).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Sequence

import torch

from . import _lib, _pipeline as pl
from ._autograd import _camera
from ._runtime import resolve_execution_options
from .view_sharding import GradientBuffer

NUM_CHANNELS = 3
SSIM_C1 = 0.01 ** 2
SSIM_C2 = 0.03 ** 2


def photometric_loss_forward(img: torch.Tensor, target: torch.Tensor, l1_weight: float = 1.0,
                             ssim_weight: float = 0.2, out: torch.Tensor | None = None):
    """``(loss3, dm)``: loss3 = [w_l1*L1 + w_ssim*(1-SSIM), L1, SSIM] on the
    device, dm = the per-pixel maps backward needs.  Images are (C,H,W) or
    (B,C,H,W) fp32 on one CUDA device; 'same' padding."""
    x = pl._f32(img)
    y = pl._f32(target)
    if x.shape != y.shape or x.ndim not in (3, 4):
        raise ValueError("img and target must share a (C,H,W) or (B,C,H,W) shape")
    B, C, H, W = (1, *x.shape) if x.ndim == 3 else x.shape
    dev = x.device
    L = _lib.load()
    dm = torch.empty((3, B, C, H, W), dtype=torch.float32, device=dev)
    parts = torch.empty(2 * int(L.gsb_ssim_partials_count(B, C, H, W)), dtype=torch.float32, device=dev)
    loss3 = out if out is not None else torch.empty(3, dtype=torch.float32, device=dev)
    a = _lib.PhotoLossFwdArgs()
    a.B, a.C, a.H, a.W = B, C, H, W
    a.C1, a.C2 = SSIM_C1, SSIM_C2
    a.w_l1, a.w_ssim = float(l1_weight), float(ssim_weight)
    a.img, a.target, a.dm, a.partials, a.loss_out = (_lib.ptr(x), _lib.ptr(y), _lib.ptr(dm), _lib.ptr(parts),
                                                    _lib.ptr(loss3))
    with torch.cuda.device(dev), pl._stage_timer("loss_fwd", {"kernels": 2}):
        _lib.call("gsb_photo_loss_fwd", a, _lib.stream_handle(dev))
    return loss3, dm


def photometric_loss_backward(img: torch.Tensor, target: torch.Tensor, dm: torch.Tensor, l1_weight: float = 1.0,
                              ssim_weight: float = 0.2, upstream: float = 1.0) -> torch.Tensor:
    """upstream * d(w_l1*L1 + w_ssim*(1-SSIM))/d img, same shape as img."""
    x = pl._f32(img)
    y = pl._f32(target)
    B, C, H, W = (1, *x.shape) if x.ndim == 3 else x.shape
    if dm.shape != (3, B, C, H, W):
        raise ValueError("dm does not belong to these images")
    g = torch.empty_like(x)
    a = _lib.PhotoLossBwdArgs()
    a.B, a.C, a.H, a.W = B, C, H, W
    a.w_l1, a.w_ssim, a.upstream = float(l1_weight), float(ssim_weight), float(upstream)
    a.img, a.target, a.dm, a.grad_img = _lib.ptr(x), _lib.ptr(y), _lib.ptr(dm), _lib.ptr(g)
    with torch.cuda.device(x.device), pl._stage_timer("loss_bwd", {"kernels": 1}):
        _lib.call("gsb_photo_loss_bwd", a, _lib.stream_handle(x.device))
    return g


def backward_ranges(P: int, chunks: int) -> list[tuple[int, int]]:
    """The Gaussian ranges ``[b, e)`` the multi-view backward works through
    one after another: ``min(chunks, P)`` ranges of near-equal size, in
    order, covering ``[0, P)`` once (none for P = 0)."""
    n = max(1, min(int(chunks), P))
    return [(P * c // n, P * (c + 1) // n) for c in range(n)] if P > 0 else []


def range_slices(P: int, block_floats: Sequence[int], b: int, e: int) -> list[tuple[int, int]]:
    """Slices ``(lo, hi)`` of the flat gradient buffer that hold the
    Gaussians ``[b, e)``: the buffer is SoA blocks of ``block_floats[k]``
    floats per Gaussian (``(3, 3, 4, 1, 48)`` for means, scales, rotations,
    opacities and SH at degree 3), one slice per block."""
    out, off = [], 0
    for f in block_floats:
        out.append((off + f * b, off + f * e))
        off += f * P
    return out


def _distributed(group) -> bool:
    return (torch.distributed.is_available() and torch.distributed.is_initialized()
            and torch.distributed.get_world_size(group) > 1)


@dataclass(slots=True)
class _ViewState:
    """What the range-ordered preprocess backward reads of one view."""
    gaussians: pl.Gaussians
    cam: pl.Camera
    radii: torch.Tensor
    records: torch.Tensor
    ids: torch.Tensor
    grad_acc: torch.Tensor


class FusedViewStep:
    """One data-parallel training step over this rank's views, fused.

    ``params`` are (means (P,3), scales (P,3), rotations (P,4), opacities
    (P,1), sh (P,K,3)), the rasterizer's inputs; ``settings`` the
    ``GaussianRasterizationSettings`` of every view this rank renders.
    ``step(targets)`` takes one (3,H,W) target per view -- on the device, or
    in (pinned) host memory, in which case it is copied to the device inside
    the step -- and returns the per-view [loss, L1, SSIM] rows as a (V,3)
    device tensor.  Gradients are in ``self.grads`` (one flat buffer; its
    blocks are the parameters' ``.grad``) and are all-reduced across the
    process group when one is initialised.  The step ends with one host read
    of the device error word (a synchronisation), so an error flagged by any
    of its kernels raises ``RuntimeError`` from this call.
    """

    def __init__(self, params: Sequence[torch.Tensor], settings: Sequence, l1_weight: float = 1.0,
                 ssim_weight: float = 0.2, group=None, densify_stats: bool = False, batch_sh: bool | None = None):
        if len(params) != 5:
            raise ValueError("params must be (means, scales, rotations, opacities, sh)")
        means, scales, rots, opac, sh = params
        P = means.shape[0]
        for t, shape in ((means, (P, 3)), (scales, (P, 3)), (rots, (P, 4)), (opac, (P, 1))):
            if tuple(t.shape) != shape or t.dtype != torch.float32 or not t.is_contiguous():
                raise ValueError(f"parameter of shape {tuple(t.shape)} must be contiguous fp32 {shape}")
        if sh.ndim != 3 or sh.shape[0] != P or sh.shape[2] != NUM_CHANNELS or sh.dtype != torch.float32 \
                or not sh.is_contiguous():
            raise ValueError("sh must be contiguous fp32 (P, K, 3)")
        if not settings:
            raise ValueError("no views")
        self.params = list(params)
        self.settings = list(settings)
        self.cams = [_camera(rs) for rs in self.settings]
        self.modes = [pl.coverage_mode_id(resolve_execution_options(rs)) for rs in self.settings]
        self.bgs = [pl._f32(rs.bg).reshape(NUM_CHANNELS) for rs in self.settings]
        self.l1_weight = float(l1_weight)
        self.ssim_weight = float(ssim_weight)
        self.group = group
        self.grads = GradientBuffer(self.params)
        dev = means.device
        self.device = dev
        self.losses = torch.zeros((len(self.settings), 3), dtype=torch.float32, device=dev)
        self._staging: dict[int, torch.Tensor] = {}
        self._target_ready: dict[int, torch.cuda.Event] = {}
        self._copy_stream: torch.cuda.Stream | None = None
        self._grad_acc: list[torch.Tensor | None] = []
        self._side: list[torch.cuda.Stream] = []
        # consecutive views go to this many streams in turn (overlapping them); 1 = one stream
        self.num_streams = 2
        # multi-view SH: the views' preprocess and SH backward run after the last view's render
        # backward, one Gaussian range at a time, and each range is all-reduced (with a process group)
        # while the next one is computed
        self.backward_chunks = 8
        # range-ordered backward (multi-view SH only): off by default -- the per-view preprocess
        # backward overlaps the next view's forward on the other stream, which the range order gives up,
        # and on 2 GPUs the exchange it overlaps did not pay for that (25.5 ms per step either way)
        self.range_backward = False
        # a partial range order (multi-view SH only): the first V - deferred_views views run view by
        # view, the last deferred_views stop after their render backward and finish range by range as
        # above (range_backward set = every view deferred); the additions into the flat buffer keep
        # view order either way, so every setting gives the same bits
        self.deferred_views = 0
        # view-by-view order with a process group: 0 = SH backward, then one all-reduce of the buffer;
        # n > 0 = the blocks complete after the last view are all-reduced while the SH backward runs in
        # n Gaussian ranges, each range's SH rows while the next is computed, the means last
        self.sh_reduce_chunks = 4
        # 3DGS densification statistics, accumulated per view until reset_densify_stats():
        # xyz_gradient_accum += |d loss / d means2D (x, y)|, denom += 1 and max_radii2D = max(., radius)
        # for every Gaussian with a radius in the view
        self.densify_stats = densify_stats
        if densify_stats:
            self.xyz_gradient_accum = torch.zeros(P, dtype=torch.float32, device=dev)
            self.denom = torch.zeros(P, dtype=torch.float32, device=dev)
            self.max_radii2D = torch.zeros(P, dtype=torch.float32, device=dev)
        # SH colours and SH gradients once per step (all views share the parameters and the SH degree)
        degrees = {int(rs.sh_degree) for rs in self.settings}
        can_batch = len(degrees) == 1 and 1 <= sh.shape[1] <= 16 and \
            len({float(rs.scale_modifier) for rs in self.settings}) == 1
        if batch_sh is None:
            batch_sh = can_batch and len(self.settings) > 1
        elif batch_sh and not can_batch:
            raise ValueError("batch_sh needs one SH degree and scale modifier for all views and at most 16 "
                             "SH coefficients")
        self.batch_sh = bool(batch_sh)
        if self.batch_sh:
            V = len(self.settings)
            self._sh_degree = degrees.pop()
            self._campos = torch.stack([c.campos.reshape(3) for c in self.cams]).contiguous()
            self._colors = torch.empty((V, P, NUM_CHANNELS), dtype=torch.float32, device=dev)
            # the SH backward resets what it reads, so this stays zero between steps
            self._grad_colors = torch.zeros((V, P, NUM_CHANNELS), dtype=torch.float32, device=dev)
            self._scale_modifier = float(self.settings[0].scale_modifier)
        # one render-gradient accumulator per view for the range-ordered backward (the multi-view
        # preprocess backward zeroes what it reads, so they stay zero between steps)
        self._view_grad_acc: torch.Tensor | None = None

    @property
    def concurrent_views(self) -> bool:
        return self.num_streams > 1

    @concurrent_views.setter
    def concurrent_views(self, on: bool) -> None:
        self.num_streams = 2 if on else 1

    def _gaussians(self, rs) -> pl.Gaussians:
        means, scales, rots, opac, sh = self.params
        return pl.make_gaussians(means, opac, scales, rots, None, sh, None, rs.scale_modifier, rs.sh_degree)

    def _staging_buffer(self, i: int, t: torch.Tensor) -> torch.Tensor:
        buf = self._staging.get(i)
        if buf is None or buf.shape != t.shape:
            buf = torch.empty(t.shape, dtype=torch.float32, device=self.device)
            self._staging[i] = buf
        return buf

    def _upload_targets(self, targets: Sequence[torch.Tensor], main: torch.cuda.Stream) -> None:
        """Host targets are copied on a copy stream at the start of the step,
        each with an event that only its view's loss waits for, so the copies
        overlap the views' preprocess, binning and render."""
        if all(t.device == self.device for t in targets):
            return
        if self._copy_stream is None:
            self._copy_stream = torch.cuda.Stream(self.device)
        self._copy_stream.wait_stream(main)  # the previous step is done with the staging buffers
        with torch.cuda.stream(self._copy_stream):
            for i, t in enumerate(targets):
                if t.device == self.device:
                    continue
                self._staging_buffer(i, t).copy_(t, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(self._copy_stream)
                self._target_ready[i] = ev

    def _target(self, i: int, t: torch.Tensor) -> tuple[torch.Tensor, torch.cuda.Event | None]:
        if t.device == self.device:
            return pl._f32(t), None
        ready = self._target_ready.pop(i, None)
        buf = self._staging_buffer(i, t)
        if ready is None:  # not uploaded by step(): copy in stream order
            buf.copy_(t, non_blocking=True)
        return buf, ready

    def view(self, i: int, target: torch.Tensor, before_accumulate: torch.cuda.Event | None = None,
             lane: int = 0) -> None:
        """Forward + loss + backward of view ``i`` on the current stream;
        gradients are added into the flat buffer and the view's loss row
        into ``self.losses[i]``.  ``before_accumulate`` (if given) is waited
        for just before the accumulation into the flat buffer; ``lane``
        picks the render-gradient accumulator (one per concurrent stream)."""
        rs, cam, mode, bg = self.settings[i], self.cams[i], self.modes[i], self.bgs[i]
        g = self._gaussians(rs)
        P = g.P
        if target.shape != (NUM_CHANNELS, cam.H, cam.W):
            raise ValueError(f"target {i} must have shape (3, {cam.H}, {cam.W})")
        tgt, tgt_ready = self._target(i, target)
        if self.batch_sh:
            g.sh, g.colors = None, self._colors[i]
        pre = pl.preprocess(g, cam, mode, sparse=True, colors_clamp_signed=self.batch_sh)
        binned = pl.binning(pre, cam, mode, want_ids=True)
        ren = pl.render(pre, binned, cam, bg, False)
        if tgt_ready is not None:
            torch.cuda.current_stream(self.device).wait_event(tgt_ready)
        _, dm = photometric_loss_forward(ren.color, tgt, self.l1_weight, self.ssim_weight, out=self.losses[i])
        grad_img = photometric_loss_backward(ren.color, tgt, dm, self.l1_weight, self.ssim_weight)
        while len(self._grad_acc) <= lane:
            self._grad_acc.append(None)
        acc_buf = self._grad_acc[lane]
        if acc_buf is None or acc_buf.shape[0] != P:
            acc_buf = torch.zeros((P, _lib.GRAD_FLOATS), dtype=torch.float32, device=self.device)
            self._grad_acc[lane] = acc_buf
        grad_acc = pl.render_backward(pre.records, binned, cam, bg, ren.alpha, ren.n_contrib, grad_img, None, None,
                                      False, P, grad_acc=acc_buf)
        v_means, v_scales, v_rots, v_opac, v_sh = self.grads.views
        out = pl.PreprocessGrads(grad_means3D=v_means, grad_means2D=None, grad_opacity=v_opac,
                                 grad_scales=v_scales, grad_rotations=v_rots, grad_cov3D=None,
                                 grad_sh=None if self.batch_sh else v_sh,
                                 grad_colors=self._grad_colors[i] if self.batch_sh else None)
        if before_accumulate is not None:
            torch.cuda.current_stream(self.device).wait_event(before_accumulate)
        # reads each binned Gaussian's accumulator entry and zeroes it: the accumulator is all zero again
        # for the next view (render backward only touches binned Gaussians)
        pl.preprocess_backward(g, cam, pre.radii, pre.records, grad_acc, None, None, None, out=out, ids=binned.ids,
                               clear_grad_acc=True,
                               densify_grad_accum=self.xyz_gradient_accum if self.densify_stats else None,
                               grad_colors_clamped=self.batch_sh)
        if self.densify_stats:
            _lib.call("gsb_densify_stats", P, _lib.ptr(pre.radii), _lib.ptr(self.denom), _lib.ptr(self.max_radii2D),
                      _lib.stream_handle(self.device))

    def view_render_grads(self, i: int, target: torch.Tensor, grad_acc: torch.Tensor) -> _ViewState:
        """Multi-view SH, first half of view ``i`` on the current stream:
        forward, loss, loss backward and render backward into ``grad_acc``
        (the view's own zeroed (P, 12) accumulator).  Returns what the
        range-ordered preprocess backward of the step reads of this view."""
        rs, cam, mode, bg = self.settings[i], self.cams[i], self.modes[i], self.bgs[i]
        g = self._gaussians(rs)
        P = g.P
        if target.shape != (NUM_CHANNELS, cam.H, cam.W):
            raise ValueError(f"target {i} must have shape (3, {cam.H}, {cam.W})")
        tgt, tgt_ready = self._target(i, target)
        g.sh, g.colors = None, self._colors[i]
        pre = pl.preprocess(g, cam, mode, sparse=True, colors_clamp_signed=True)
        binned = pl.binning(pre, cam, mode, want_ids=True)
        ren = pl.render(pre, binned, cam, bg, False)
        if tgt_ready is not None:
            torch.cuda.current_stream(self.device).wait_event(tgt_ready)
        _, dm = photometric_loss_forward(ren.color, tgt, self.l1_weight, self.ssim_weight, out=self.losses[i])
        grad_img = photometric_loss_backward(ren.color, tgt, dm, self.l1_weight, self.ssim_weight)
        pl.render_backward(pre.records, binned, cam, bg, ren.alpha, ren.n_contrib, grad_img, None, None, False, P,
                           grad_acc=grad_acc)
        return _ViewState(gaussians=g, cam=cam, radii=pre.radii, records=pre.records, ids=binned.ids,
                          grad_acc=grad_acc)

    def reset_densify_stats(self) -> None:
        if self.densify_stats:
            self.xyz_gradient_accum.zero_()
            self.denom.zero_()
            self.max_radii2D.zero_()

    def step(self, targets: Sequence[torch.Tensor]) -> torch.Tensor:
        """Runs every view, then the all-reduce.  Consecutive views go to
        ``num_streams`` streams in turn, so one view's compute-bound render
        kernels overlap the next view's memory- and latency-bound preprocess
        and binning.  Each view finishes its own backward, the accumulations
        into the flat gradient buffer in view order (each waits for the
        previous one), then the multi-view SH backward and the all-reduce
        run; or, range-ordered (``range_backward``, or the last
        ``deferred_views`` views), those views stop after their render
        backward (each into its own accumulator) and their preprocess and the
        SH backward run afterwards on this stream, Gaussian range by Gaussian
        range, each range all-reduced while the next is computed."""
        if len(targets) != len(self.settings):
            raise ValueError(f"expected {len(self.settings)} targets, got {len(targets)}")
        n_streams = max(1, int(self.num_streams))
        with torch.cuda.device(self.device):
            main = torch.cuda.current_stream(self.device)
            while len(self._side) < n_streams - 1:
                self._side.append(torch.cuda.Stream(self.device))
            streams = [main] + self._side[: n_streams - 1]
            means, _, _, _, sh = self.params
            if self.batch_sh:
                # the SH block is stored whole by the SH backward; only the rest needs zeroing
                self.grads.flat[: self.grads.flat.numel() - sh.numel()].zero_()
                self.grads.attach()
                pl.sh_colors_views(means, sh, self._sh_degree, self._campos, out=self._colors)
            else:
                self.grads.zero_()
            P, V = means.shape[0], len(targets)
            deferred = 0
            if self.batch_sh:
                deferred = V if self.range_backward else max(0, min(V, int(self.deferred_views)))
            ranged = deferred > 0
            if ranged and (self._view_grad_acc is None or self._view_grad_acc.shape[:2] != (deferred, P)):
                self._view_grad_acc = torch.zeros((deferred, P, _lib.GRAD_FLOATS), dtype=torch.float32,
                                                  device=self.device)
            self._upload_targets(targets, main)
            ready = torch.cuda.Event()
            ready.record(main)
            for side in streams[1:]:
                side.wait_event(ready)  # zeroed buffers, targets and parameters visible to every stream
            if ranged:
                first = V - deferred
                prev = None
                for i in range(first):
                    s = streams[i % n_streams]
                    with torch.cuda.stream(s):
                        self.view(i, targets[i], before_accumulate=prev, lane=i % n_streams)
                        prev = torch.cuda.Event()
                        prev.record(s)
                states = []
                for i in range(first, V):
                    s = streams[i % n_streams]
                    with torch.cuda.stream(s):
                        st = self.view_render_grads(i, targets[i], self._view_grad_acc[i - first])
                        if s is not main:
                            for buf in (st.radii, st.records, st.ids):
                                buf.record_stream(main)
                        states.append((i, st))
                for side in streams[1:]:
                    done = torch.cuda.Event()
                    done.record(side)
                    main.wait_event(done)
                self._ranged_backward(states)
            else:
                prev = None
                for i, t in enumerate(targets):
                    s = streams[i % n_streams]
                    with torch.cuda.stream(s):
                        self.view(i, t, before_accumulate=prev, lane=i % n_streams)
                        prev = torch.cuda.Event()
                        prev.record(s)
                # the last view's event follows every earlier one (each view's accumulation waits for the
                # previous)
                main.wait_event(prev)
                if self.batch_sh and _distributed(self.group) and self.sh_reduce_chunks > 0:
                    self._sh_backward_and_reduce()
                else:
                    if self.batch_sh:
                        pl.sh_backward_views(means, sh, self._sh_degree, self._campos, self._grad_colors,
                                             self.grads.views[4], self.grads.views[0])
                    self.grads.all_reduce(self.group)
            # errors flagged by the last view's emit and sort (earlier views' are read by the next
            # view's binning): raised by this call, before anyone uses its gradients
            pl.raise_device_errors(self.device)
        return self.losses

    def _sh_backward_and_reduce(self) -> None:
        """All-reduces (on NCCL's stream) while the SH backward runs: first the
        scales, rotations and opacities (complete after the last view), then
        the SH rows range by range, each while the next range is computed,
        and the means last (the SH backward adds their view-direction term).
        The sums are elementwise, so the result equals one all-reduce of the
        whole buffer."""
        means, _, _, _, sh = self.params
        P = means.shape[0]
        flat = self.grads.flat
        blocks = [v.numel() // P if P else 0 for v in self.grads.views]
        whole = range_slices(P, blocks, 0, P)
        works = [torch.distributed.all_reduce(flat[whole[1][0]:whole[3][1]], group=self.group, async_op=True)]
        for b, e in backward_ranges(P, self.sh_reduce_chunks):
            pl.sh_backward_views(means, sh, self._sh_degree, self._campos, self._grad_colors, self.grads.views[4],
                                 self.grads.views[0], begin=b, end=e)
            lo, hi = range_slices(P, blocks, b, e)[4]
            works.append(torch.distributed.all_reduce(flat[lo:hi], group=self.group, async_op=True))
        works.append(torch.distributed.all_reduce(flat[whole[0][0]:whole[0][1]], group=self.group, async_op=True))
        for w in works:
            w.wait()

    def _ranged_backward(self, states: list) -> None:
        """The second half of a multi-view step, on the current stream, one
        Gaussian range after another: every deferred view's (``states``:
        (view index, state) pairs, in view order, after the views that ran
        view by view) preprocess backward over its binned ids inside the range
        (accumulated into the flat buffer in view order, as view by view),
        then the SH backward of the range
        (stores the SH rows, adds the view-direction term to the means).
        With a process group each finished range is all-reduced on NCCL's
        stream while the next range is computed; the sums are elementwise,
        so the result equals one all-reduce of the whole buffer.  Finding
        the ranges' bounds in the views' id lists costs one host read."""
        means, _, _, _, sh = self.params
        P = means.shape[0]
        flat = self.grads.flat
        v_means, v_scales, v_rots, v_opac, v_sh = self.grads.views
        blocks = [v.numel() // P if P else 0 for v in self.grads.views]
        ranges = backward_ranges(P, self.backward_chunks)
        if not ranges:
            return
        bounds = torch.tensor([b for b, _ in ranges] + [P], dtype=torch.int32, device=self.device)
        splits = torch.stack([torch.searchsorted(st.ids, bounds) for _, st in states]).tolist()
        if self.densify_stats:
            for _, st in states:
                _lib.call("gsb_densify_stats", P, _lib.ptr(st.radii), _lib.ptr(self.denom),
                          _lib.ptr(self.max_radii2D), _lib.stream_handle(self.device))
        # one argument block per view; per range only the id slice changes
        args = []
        for v, st in states:
            out = pl.PreprocessGrads(grad_means3D=v_means, grad_means2D=None, grad_opacity=v_opac,
                                     grad_scales=v_scales, grad_rotations=v_rots, grad_cov3D=None, grad_sh=None,
                                     grad_colors=self._grad_colors[v])
            args.append(pl.preprocess_backward_args(
                st.gaussians, st.cam, st.radii, st.records, st.grad_acc, None, None, None, out, True, ids=st.ids,
                clear_grad_acc=True, densify_grad_accum=self.xyz_gradient_accum if self.densify_stats else None,
                grad_colors_clamped=True))
        L = _lib.load()
        stream = _lib.stream_handle(self.device)
        dist = _distributed(self.group)
        works = []
        for r, (b, e) in enumerate(ranges):
            for k, (_, st) in enumerate(states):
                lo, hi = splits[k][r], splits[k][r + 1]
                if hi <= lo:
                    continue
                a = args[k]
                a.ids = st.ids.data_ptr() + 4 * lo
                a.num_ids = hi - lo
                with pl._stage_timer("preprocess_bwd", {"P": P, "kernels": 1, "accumulate": True,
                                                        "visible": hi - lo}):
                    _lib.check(L.gsb_preprocess_bwd(ctypes.byref(a), stream), "gsb_preprocess_bwd")
            pl.sh_backward_views(means, sh, self._sh_degree, self._campos, self._grad_colors, v_sh, v_means,
                                 begin=b, end=e)
            if dist:
                for lo, hi in range_slices(P, blocks, b, e):
                    if hi > lo:
                        works.append(torch.distributed.all_reduce(flat[lo:hi], group=self.group, async_op=True))
        for w in works:
            w.wait()
