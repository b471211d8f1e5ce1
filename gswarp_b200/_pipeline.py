"""Host side of the rasterizer: stage order, buffer allocation, C-ABI calls.

Mirrors the stage pipeline of gswarp (methods/pipeline.py:11-45 ->
preprocess_ops.py:289-581, binning_ops.py:84-431, render_ops.py:16-93,
backward_ops.py:376-746).  Every buffer, workspaces included, comes from the
torch caching allocator on the caller's current stream; the native library
owns no memory.  The forward performs exactly one host synchronization: the
pair count read after the depth-ordered scan, as the reference does
(binning_ops.py:243-252).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from . import _coverage
from ._runtime import BLOCK_X, BLOCK_Y, ExecutionOptions

NUM_CHANNELS = 3
MAX_BINNING_PAIRS = (1 << 31) - 1

_STICKY: dict[int, torch.Tensor] = {}

# Optional CUDA-event timing of the native stages (used by bench.py): when
# enabled, every stage call records (start, end, info) on the current stream.
TIMING_ENABLED = False
TIMERS: dict[str, list] = {}


class _stage_timer:
    def __init__(self, name: str, info: dict | None = None):
        self.name = name
        self.info = info or {}

    def __enter__(self):
        if TIMING_ENABLED:
            self.a = torch.cuda.Event(enable_timing=True)
            self.b = torch.cuda.Event(enable_timing=True)
            self.a.record()
        return self

    def __exit__(self, *exc):
        if TIMING_ENABLED and exc[0] is None:
            self.b.record()
            TIMERS.setdefault(self.name, []).append((self.a, self.b, self.info))
        return False


def sticky_error_word(device: torch.device) -> torch.Tensor:
    """Per-device int64 word that kernels OR error bits into (checked at the
    next host synchronization)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _STICKY.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int64, device=device)
        _STICKY[idx] = t
    return t


def _device_error(bits: int) -> RuntimeError:
    return RuntimeError(f"gswarp_b200 device error word {int(bits):#x} "
                        "(bounded wait timed out or binning mismatch)")


def raise_device_errors(device: torch.device) -> None:
    """Reads the sticky error word of ``device`` (a synchronisation of the
    current stream) and raises if a kernel flagged an error since the last
    check; the word is cleared before raising.  Binning checks it at its own
    host read of the pair count, which covers every earlier call; this
    covers the calls after it (the emit and sort of the last binning)."""
    sticky = sticky_error_word(device)
    bits = int(sticky.item())
    if bits:
        sticky.zero_()
        raise _device_error(bits)


def _f32(t: torch.Tensor) -> torch.Tensor:
    t = t.detach()
    if t.dtype != torch.float32:
        t = t.float()
    if not t.is_contiguous():
        t = t.contiguous()
    return t


def _aligned16(t: torch.Tensor) -> torch.Tensor:
    return t if t.data_ptr() % 16 == 0 else t.clone()


def _workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


@dataclass(slots=True)
class Camera:
    W: int
    H: int
    tanfovx: float
    tanfovy: float
    viewmatrix: torch.Tensor
    projmatrix: torch.Tensor
    campos: torch.Tensor

    @property
    def focal_x(self) -> float:
        return self.W / (2.0 * float(self.tanfovx))

    @property
    def focal_y(self) -> float:
        return self.H / (2.0 * float(self.tanfovy))

    @property
    def grid(self) -> tuple[int, int]:
        return (self.W + BLOCK_X - 1) // BLOCK_X, (self.H + BLOCK_Y - 1) // BLOCK_Y


@dataclass(slots=True)
class Gaussians:
    means3D: torch.Tensor
    opacities: torch.Tensor
    scales: torch.Tensor | None
    rotations: torch.Tensor | None
    cov3D: torch.Tensor | None
    sh: torch.Tensor | None          # (P, K, 3) view of the caller's tensor
    colors: torch.Tensor | None
    scale_modifier: float
    degree: int

    @property
    def P(self) -> int:
        return self.means3D.shape[0]


@dataclass(slots=True)
class Preprocessed:
    radii: torch.Tensor
    proj_2d: torch.Tensor | None
    conic_2d: torch.Tensor | None
    conic_2d_inv: torch.Tensor | None
    depths: torch.Tensor
    tiles_touched: torch.Tensor
    records: torch.Tensor
    cov3d: torch.Tensor | None = None
    bin_records: torch.Tensor | None = None


@dataclass(slots=True)
class Binned:
    num_rendered: int
    point_list: torch.Tensor
    ranges: torch.Tensor
    ids: torch.Tensor | None = None   # ascending ids of the Gaussians with tiles (if requested)


@dataclass(slots=True)
class Rendered:
    color: torch.Tensor
    depth: torch.Tensor
    alpha: torch.Tensor
    n_contrib: torch.Tensor
    # flow render auxiliary outputs (top_k > 0)
    gs_per_pixel: torch.Tensor | None = None
    weight_per_gs_pixel: torch.Tensor | None = None
    x_mu: torch.Tensor | None = None


def make_gaussians(means3D, opacities, scales, rotations, cov3D, sh, colors, scale_modifier, degree) -> Gaussians:
    P = means3D.shape[0]

    def opt(t, shape):
        if t is None or t.numel() == 0:
            return None
        return _f32(t).reshape(shape)

    sh_t = None
    if sh is not None and sh.numel() != 0:
        sh_t = _f32(sh).reshape(P, -1, NUM_CHANNELS)
    rot = opt(rotations, (P, 4))
    return Gaussians(
        means3D=_f32(means3D),
        opacities=_f32(opacities).reshape(P),
        scales=opt(scales, (P, 3)),
        rotations=_aligned16(rot) if rot is not None else None,
        cov3D=opt(cov3D, (P, 6)),
        sh=sh_t,
        colors=opt(colors, (P, NUM_CHANNELS)),
        scale_modifier=float(scale_modifier),
        degree=int(degree),
    )


def coverage_mode_id(options: ExecutionOptions | None) -> int:
    return _coverage.kernel_mode("auto" if options is None else options.tile_coverage_mode)


BIN_RECORD_FLOATS = 8
MAX_TILE_GRID = 65535


def preprocess(g: Gaussians, cam: Camera, coverage_mode: int, want_cov3d: bool = False,
               bin_records: bool = True, sparse: bool = False, colors_clamp_signed: bool = False) -> Preprocessed:
    """Runs the fused preprocess.  With ``bin_records`` (the default) it also
    writes the 32-byte per-Gaussian records the binning emit reads instead of
    gathering radii, render records, conic_2D_inv and tiles_touched.
    ``sparse`` (internal training step) skips what only the autograd outputs
    need: proj_2D / conic_2D / conic_2D_inv are not produced and render
    records are written only for Gaussians with a radius.
    ``colors_clamp_signed``: ``g.colors`` comes from ``sh_colors_views``
    (clamped channels stored as -0.0), so the records carry the SH path's
    clamp bits."""
    P = g.P
    dev = g.means3D.device
    cov3d = None
    if want_cov3d:
        cov3d = g.cov3D if g.cov3D is not None else torch.empty((P, 6), dtype=torch.float32, device=dev)
    out = Preprocessed(
        cov3d=cov3d,
        radii=torch.empty(P, dtype=torch.int32, device=dev),
        proj_2d=None if sparse else torch.empty((P, 2), dtype=torch.float32, device=dev),
        conic_2d=None if sparse else torch.empty((P, 3), dtype=torch.float32, device=dev),
        conic_2d_inv=None if sparse else torch.empty((P, 3), dtype=torch.float32, device=dev),
        depths=torch.empty(P, dtype=torch.float32, device=dev),
        tiles_touched=torch.empty(P, dtype=torch.int32, device=dev),
        records=torch.empty((P, _lib.RECORD_FLOATS), dtype=torch.float32, device=dev),
    )
    gx, gy = cam.grid
    if bin_records and P > 0 and gx <= MAX_TILE_GRID and gy <= MAX_TILE_GRID:
        out.bin_records = torch.empty((P, BIN_RECORD_FLOATS), dtype=torch.float32, device=dev)
    elif sparse:
        out.conic_2d_inv = torch.empty((P, 3), dtype=torch.float32, device=dev)  # the gathering emit needs it
    if P == 0:
        return out
    a = _lib.PreprocessArgs()
    a.P, a.W, a.H = P, cam.W, cam.H
    a.means = _lib.ptr(g.means3D)
    a.scales = _lib.ptr(g.scales)
    a.rotations = _lib.ptr(g.rotations)
    a.cov3d_precomp = _lib.ptr(g.cov3D)
    a.scale_modifier = g.scale_modifier
    a.opacities = _lib.ptr(g.opacities)
    a.viewmatrix = _lib.ptr(cam.viewmatrix)
    a.projmatrix = _lib.ptr(cam.projmatrix)
    a.campos = _lib.ptr(cam.campos)
    a.tanfovx, a.tanfovy = float(cam.tanfovx), float(cam.tanfovy)
    a.focal_x, a.focal_y = cam.focal_x, cam.focal_y
    a.sh = _lib.ptr(g.sh)
    a.sh_degree = g.degree
    a.sh_coeffs = g.sh.shape[1] if g.sh is not None else 0
    a.colors_precomp = _lib.ptr(g.colors)
    a.coverage_mode = coverage_mode
    a.radii = _lib.ptr(out.radii)
    a.proj_2d = _lib.ptr(out.proj_2d)
    a.conic_2d = _lib.ptr(out.conic_2d)
    a.conic_2d_inv = _lib.ptr(out.conic_2d_inv)
    a.depths = _lib.ptr(out.depths)
    a.tiles_touched = _lib.ptr(out.tiles_touched)
    a.records = _lib.ptr(out.records)
    a.cov3d_out = _lib.ptr(cov3d) if (cov3d is not None and g.cov3D is None) else None
    a.bin_records = _lib.ptr(out.bin_records)
    a.sparse_records = int(sparse)
    a.colors_clamp_signed = int(colors_clamp_signed)
    with _stage_timer("preprocess_fwd", {"P": P, "kernels": 1}):
        _lib.call("gsb_preprocess_fwd", a, _lib.stream_handle(dev))
    return out


def binning(pre: Preprocessed, cam: Camera, coverage_mode: int, want_ids: bool = False) -> Binned:
    """Binning.  With ``want_ids`` the result also lists, in ascending order,
    the Gaussians that touch at least one tile (the only ones the render
    backward gives a gradient)."""
    P = pre.radii.shape[0]
    dev = pre.radii.device
    gx, gy = cam.grid
    tiles = gx * gy
    L = _lib.load()
    stream = _lib.stream_handle(dev)
    ranges = torch.empty((tiles, 2), dtype=torch.int32, device=dev)
    if P == 0:
        ranges.zero_()
        empty = torch.empty(0, dtype=torch.int32, device=dev)
        return Binned(0, empty, ranges, empty if want_ids else None)
    depth_order = torch.empty(P, dtype=torch.int32, device=dev)
    offsets = torch.empty(P, dtype=torch.int32, device=dev)
    status = torch.empty(3, dtype=torch.int64, device=dev)
    ws_bytes = int(L.gsb_bin_count_workspace_bytes(P))
    ws = _workspace(ws_bytes, dev)
    a = _lib.BinCountArgs()
    a.P = P
    a.depths = _lib.ptr(pre.depths)
    a.radii = _lib.ptr(pre.radii)
    a.tiles_touched = _lib.ptr(pre.tiles_touched)
    a.depth_order = _lib.ptr(depth_order)
    a.point_offsets = _lib.ptr(offsets)
    ids = torch.empty(P, dtype=torch.int32, device=dev) if want_ids else None
    a.binned_ids = _lib.ptr(ids)
    a.status_out = _lib.ptr(status)
    a.workspace = _lib.ptr(ws)
    a.workspace_bytes = ws_bytes
    # compaction, depth-key histogram + bin bases, 4 depth passes, depth-ordered scan
    with _stage_timer("bin_count", {"P": P, "kernels": 8}):
        _lib.call("gsb_bin_count", a, stream)
    sticky = sticky_error_word(dev)
    total, err, num_binned, sticky_bits = torch.cat([status, sticky]).tolist()
    if err or sticky_bits:
        sticky.zero_()
        raise _device_error(int(err) | int(sticky_bits))
    if total < 0 or total > MAX_BINNING_PAIRS:
        raise OverflowError(
            "binning tile-reference count exceeds signed int32; reduce Gaussian footprint or image size"
        )
    R = int(total)
    point_list = torch.empty(max(R, 1), dtype=torch.int32, device=dev)
    ws2_bytes = int(L.gsb_bin_sort_workspace_bytes(R, cam.W, cam.H))
    ws2 = _workspace(ws2_bytes, dev) if R > 0 else _workspace(256, dev)
    b = _lib.BinSortArgs()
    b.P, b.W, b.H = P, cam.W, cam.H
    b.num_rendered = R
    b.coverage_mode = coverage_mode
    b.depth_order = _lib.ptr(depth_order)
    b.point_offsets = _lib.ptr(offsets)
    b.radii = _lib.ptr(pre.radii)
    b.records = _lib.ptr(pre.records)
    b.conic_2d_inv = _lib.ptr(pre.conic_2d_inv)
    b.tiles_touched = _lib.ptr(pre.tiles_touched)
    b.point_list = _lib.ptr(point_list)
    b.ranges = _lib.ptr(ranges)
    b.error_word = _lib.ptr(sticky)
    b.workspace = _lib.ptr(ws2)
    b.workspace_bytes = ws2.numel()
    b.bin_records = _lib.ptr(pre.bin_records)
    b.bin_status = _lib.ptr(status)
    # emit, then either the tile sort (histogram + bin bases, one pass per 8 bits of the tile
    # id, ranges fix-up) or, with one tile or one pair, the single-range kernel
    passes = ((gx * gy - 1).bit_length() + 7) // 8 if gx * gy > 1 else 0
    kernels = 0 if R == 0 else (2 if passes == 0 or R <= 1 else 4 + passes)
    with _stage_timer("bin_emit_sort", {"P": P, "num_rendered": R, "kernels": kernels}):
        _lib.call("gsb_bin_emit_sort", b, stream)
    return Binned(R, point_list[:R], ranges, ids[:int(num_binned)] if ids is not None else None)


def render(pre: Preprocessed, binned: Binned, cam: Camera, background: torch.Tensor, compute_depth: bool,
           top_k: int = 0, split_aux: bool = True) -> Rendered:
    """Render forward; ``top_k > 0`` also fills the flow auxiliary outputs
    (first ``top_k`` contributors per pixel: ids, weights, centre offsets),
    through a 16-byte-record scratch and a split kernel (``split_aux``) or
    written directly by the render."""
    dev = pre.records.device
    H, W = cam.H, cam.W
    out = Rendered(
        color=torch.empty((NUM_CHANNELS, H, W), dtype=torch.float32, device=dev),
        depth=torch.empty((1, H, W), dtype=torch.float32, device=dev),
        alpha=torch.empty((1, H, W), dtype=torch.float32, device=dev),
        n_contrib=torch.empty(H * W, dtype=torch.int32, device=dev),
    )
    aux_scratch = None
    if top_k > 0:
        out.gs_per_pixel = torch.empty((top_k, H, W), dtype=torch.int32, device=dev)
        out.weight_per_gs_pixel = torch.empty((top_k, H, W), dtype=torch.float32, device=dev)
        out.x_mu = torch.empty((2, top_k, H, W), dtype=torch.float32, device=dev)
        if split_aux:  # one 16-byte record per slot, split into the three outputs by a second kernel
            aux_scratch = torch.empty((top_k, H, W, 4), dtype=torch.float32, device=dev)
    a = _lib.RenderFwdArgs()
    a.W, a.H = W, H
    a.compute_depth = int(bool(compute_depth))
    a.ranges = _lib.ptr(binned.ranges)
    a.point_list = _lib.ptr(binned.point_list) if binned.num_rendered > 0 else None
    a.records = _lib.ptr(pre.records) if pre.records.numel() else _lib.ptr(torch.zeros(16, device=dev))
    a.background = _lib.ptr(background)
    a.out_color = _lib.ptr(out.color)
    a.out_depth = _lib.ptr(out.depth)
    a.out_alpha = _lib.ptr(out.alpha)
    a.n_contrib = _lib.ptr(out.n_contrib)
    a.top_k = int(top_k) if top_k > 0 else 0
    a.gs_per_pixel = _lib.ptr(out.gs_per_pixel)
    a.weight_per_gs_pixel = _lib.ptr(out.weight_per_gs_pixel)
    a.x_mu = _lib.ptr(out.x_mu)
    a.aux_scratch = _lib.ptr(aux_scratch)
    info = {"num_rendered": binned.num_rendered, "P": pre.records.shape[0],
            "kernels": 2 if aux_scratch is not None else 1}
    with _stage_timer("render_fwd", info):
        _lib.call("gsb_render_fwd", a, _lib.stream_handle(dev))
    if TIMING_ENABLED:
        info["pairs"] = int(out.n_contrib.sum(dtype=torch.int64))
    return out


def render_backward(pre_records, binned: Binned, cam: Camera, background, out_alpha, n_contrib,
                    grad_color, grad_depth, grad_alpha, compute_depth: bool, P: int,
                    grad_acc: torch.Tensor | None = None) -> torch.Tensor:
    """Render backward into ``grad_acc`` (P,12) -- a fresh zero-filled tensor,
    or the caller's, which must be zero (e.g. kept zero by preprocess
    backward's clear_grad_acc)."""
    dev = pre_records.device
    if grad_acc is None:
        grad_acc = torch.zeros((P, _lib.GRAD_FLOATS), dtype=torch.float32, device=dev)
    if binned.num_rendered == 0 or P == 0:
        return grad_acc
    a = _lib.RenderBwdArgs()
    a.W, a.H, a.P = cam.W, cam.H, P
    a.compute_depth = int(bool(compute_depth))
    a.ranges = _lib.ptr(binned.ranges)
    a.point_list = _lib.ptr(binned.point_list)
    a.records = _lib.ptr(pre_records)
    a.background = _lib.ptr(background)
    a.out_alpha = _lib.ptr(out_alpha)
    a.n_contrib = _lib.ptr(n_contrib)
    a.grad_color = _lib.ptr(grad_color)
    a.grad_depth = _lib.ptr(grad_depth)
    a.grad_alpha = _lib.ptr(grad_alpha)
    a.grad_acc = _lib.ptr(grad_acc)
    info = {"num_rendered": binned.num_rendered, "P": P, "kernels": 1}
    with _stage_timer("render_bwd", info):
        _lib.call("gsb_render_bwd", a, _lib.stream_handle(dev))
    if TIMING_ENABLED:
        info["pairs"] = int(n_contrib.sum(dtype=torch.int64))
        info["binned"] = int(binned.ids.numel()) if binned.ids is not None else \
            int(torch.unique(binned.point_list).numel())
    return grad_acc


@dataclass(slots=True)
class PreprocessGrads:
    grad_means3D: torch.Tensor
    grad_means2D: torch.Tensor
    grad_opacity: torch.Tensor
    grad_scales: torch.Tensor | None
    grad_rotations: torch.Tensor | None
    grad_cov3D: torch.Tensor | None
    grad_sh: torch.Tensor | None
    grad_colors: torch.Tensor | None


def preprocess_backward_args(g: Gaussians, cam: Camera, radii, records, grad_acc, grad_proj_2d, grad_conic_2d,
                             grad_conic_2d_inv, out: "PreprocessGrads", accumulate: bool,
                             ids: torch.Tensor | None = None, clear_grad_acc: bool = False,
                             densify_grad_accum: torch.Tensor | None = None,
                             grad_colors_clamped: bool = False) -> "_lib.PreprocessBwdArgs":
    """The argument block of one ``gsb_preprocess_bwd`` call (see
    ``preprocess_backward``); a caller that runs the same view over several
    id slices changes only ``ids`` / ``num_ids`` between calls."""
    a = _lib.PreprocessBwdArgs()
    a.P, a.W, a.H = g.P, cam.W, cam.H
    a.means = _lib.ptr(g.means3D)
    a.radii = _lib.ptr(radii)
    a.scales = _lib.ptr(g.scales)
    a.rotations = _lib.ptr(g.rotations)
    a.cov3d_precomp = _lib.ptr(g.cov3D)
    a.scale_modifier = g.scale_modifier
    a.viewmatrix = _lib.ptr(cam.viewmatrix)
    a.projmatrix = _lib.ptr(cam.projmatrix)
    a.campos = _lib.ptr(cam.campos)
    a.tanfovx, a.tanfovy = float(cam.tanfovx), float(cam.tanfovy)
    a.focal_x, a.focal_y = cam.focal_x, cam.focal_y
    a.sh = _lib.ptr(g.sh)
    a.sh_degree = g.degree
    a.sh_coeffs = g.sh.shape[1] if g.sh is not None else 0
    a.records = _lib.ptr(records)
    a.grad_acc = _lib.ptr(grad_acc)
    a.grad_proj_2d = _lib.ptr(grad_proj_2d)
    a.grad_conic_2d = _lib.ptr(grad_conic_2d)
    a.grad_conic_2d_inv = _lib.ptr(grad_conic_2d_inv)
    a.accumulate = int(accumulate)
    a.ids = _lib.ptr(ids) if ids is not None and ids.numel() else None
    a.num_ids = int(ids.numel()) if ids is not None else 0
    a.clear_grad_acc = int(clear_grad_acc)
    a.densify_grad_accum = _lib.ptr(densify_grad_accum)
    a.grad_colors_clamped = int(grad_colors_clamped)
    a.grad_means3d = _lib.ptr(out.grad_means3D)
    a.grad_means2d = _lib.ptr(out.grad_means2D)
    a.grad_scales = _lib.ptr(out.grad_scales)
    a.grad_rotations = _lib.ptr(out.grad_rotations)
    a.grad_opacity = _lib.ptr(out.grad_opacity)
    a.grad_sh = _lib.ptr(out.grad_sh)
    a.grad_colors = _lib.ptr(out.grad_colors)
    a.grad_cov3d = _lib.ptr(out.grad_cov3D)
    return a


def preprocess_backward(g: Gaussians, cam: Camera, radii, records, grad_acc, grad_proj_2d, grad_conic_2d,
                        grad_conic_2d_inv, out: PreprocessGrads | None = None,
                        ids: torch.Tensor | None = None, clear_grad_acc: bool = False,
                        densify_grad_accum: torch.Tensor | None = None,
                        grad_colors_clamped: bool = False) -> PreprocessGrads:
    """Per-Gaussian backward.  With ``out`` given, gradients are added into
    its buffers (multi-view accumulation); otherwise fresh tensors are made.
    ``ids`` (accumulate mode only) restricts the work to those Gaussians --
    the binned ids, when the only gradients are the render's.
    ``grad_colors_clamped``: the colour gradient goes through the forward's
    clamp flags (the input of ``sh_backward_views``)."""
    if ids is not None and out is None:
        raise ValueError("an id list needs accumulation buffers (out=...)")
    P = g.P
    dev = g.means3D.device
    acc = out is not None
    if out is None:
        out = PreprocessGrads(
            grad_means3D=torch.empty((P, 3), dtype=torch.float32, device=dev),
            grad_means2D=torch.empty((P, 3), dtype=torch.float32, device=dev),
            grad_opacity=torch.empty(P, dtype=torch.float32, device=dev),
            grad_scales=torch.empty((P, 3), dtype=torch.float32, device=dev) if g.cov3D is None else None,
            grad_rotations=torch.empty((P, 4), dtype=torch.float32, device=dev) if g.cov3D is None else None,
            grad_cov3D=torch.empty((P, 6), dtype=torch.float32, device=dev) if g.cov3D is not None else None,
            grad_sh=torch.empty(g.sh.shape, dtype=torch.float32, device=dev) if g.sh is not None else None,
            grad_colors=torch.empty((P, 3), dtype=torch.float32, device=dev) if g.sh is None else None,
        )
    if P == 0:
        return out
    a = preprocess_backward_args(g, cam, radii, records, grad_acc, grad_proj_2d, grad_conic_2d, grad_conic_2d_inv,
                                 out, acc, ids, clear_grad_acc, densify_grad_accum, grad_colors_clamped)
    if ids is not None and ids.numel() == 0:
        return out
    info = {"P": P, "kernels": 1, "accumulate": acc}
    with _stage_timer("preprocess_bwd", info):
        _lib.call("gsb_preprocess_bwd", a, _lib.stream_handle(dev))
    if TIMING_ENABLED:
        info["visible"] = int(ids.numel()) if ids is not None else int((radii > 0).sum())
    return out


def _sh_views_args(means: torch.Tensor, sh: torch.Tensor, degree: int, campos: torch.Tensor):
    P = means.shape[0]
    if sh.ndim != 3 or sh.shape[0] != P or sh.shape[2] != NUM_CHANNELS or not 1 <= sh.shape[1] <= 16:
        raise ValueError("sh must be (P, K, 3) with 1 <= K <= 16")
    if campos.ndim != 2 or campos.shape[1] != 3:
        raise ValueError("campos must be (num_views, 3)")
    a = _lib.SHViewsArgs()
    a.P, a.num_views = P, campos.shape[0]
    a.sh_degree, a.sh_coeffs = int(degree), sh.shape[1]
    a.means, a.sh, a.campos = _lib.ptr(means), _lib.ptr(sh), _lib.ptr(campos)
    return a


def sh_colors_views(means: torch.Tensor, sh: torch.Tensor, degree: int, campos: torch.Tensor,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """(V,P,3) clamped SH colours of every Gaussian from each of the V
    cameras in ``campos`` (V,3); clamped channels are -0.0."""
    means, sh, campos = _f32(means), _f32(sh), _f32(campos)
    a = _sh_views_args(means, sh, degree, campos)
    shape = (campos.shape[0], means.shape[0], NUM_CHANNELS)
    if out is None:
        out = torch.empty(shape, dtype=torch.float32, device=means.device)
    elif tuple(out.shape) != shape or out.dtype != torch.float32 or not out.is_contiguous():
        raise ValueError(f"out must be contiguous fp32 {shape}")
    a.colors = _lib.ptr(out)
    with torch.cuda.device(means.device), _stage_timer("sh_colors", {"kernels": 1}):
        _lib.call("gsb_sh_colors_views", a, _lib.stream_handle(means.device))
    return out


def sh_backward_views(means: torch.Tensor, sh: torch.Tensor, degree: int, campos: torch.Tensor,
                      grad_colors: torch.Tensor, grad_sh: torch.Tensor, grad_means3D: torch.Tensor,
                      accumulate: bool = False, clear_grad_colors: bool = True, begin: int = 0,
                      end: int | None = None) -> None:
    """SH gradient (stored into ``grad_sh``, or added with ``accumulate``) and
    the view-direction term of the means gradient (added into
    ``grad_means3D``) from the views' clamped colour gradients (V,P,3), for
    the Gaussians [begin, end) (all by default)."""
    means, sh, campos = _f32(means), _f32(sh), _f32(campos)
    a = _sh_views_args(means, sh, degree, campos)
    P = means.shape[0]
    for t, shape in ((grad_colors, (campos.shape[0], P, NUM_CHANNELS)), (grad_sh, tuple(sh.shape)),
                     (grad_means3D, (P, 3))):
        if tuple(t.shape) != shape or t.dtype != torch.float32 or not t.is_contiguous():
            raise ValueError(f"gradient buffer must be contiguous fp32 {shape}")
    a.grad_colors, a.grad_sh, a.grad_means3d = _lib.ptr(grad_colors), _lib.ptr(grad_sh), _lib.ptr(grad_means3D)
    a.clear_grad_colors, a.accumulate = int(clear_grad_colors), int(accumulate)
    end = P if end is None else int(end)
    if not 0 <= begin <= end <= P:
        raise ValueError(f"need 0 <= begin <= end <= {P}")
    if begin == end:
        return
    a.begin, a.end = int(begin), end
    with torch.cuda.device(means.device), _stage_timer("sh_backward", {"kernels": 1}):
        _lib.call("gsb_sh_backward_views", a, _lib.stream_handle(means.device))


def mark_visible(means3D: torch.Tensor, viewmatrix: torch.Tensor) -> torch.Tensor:
    pts = _f32(means3D)
    if pts.ndim != 2 or pts.shape[1] != 3:
        raise ValueError("means3D must have dimensions (num_points, 3)")
    out = torch.empty(pts.shape[0], dtype=torch.uint8, device=pts.device)
    if pts.shape[0] == 0:
        return out.to(torch.bool)
    with torch.cuda.device(pts.device):
        _lib.call("gsb_mark_visible", pts.shape[0], _lib.ptr(pts), _lib.ptr(_f32(viewmatrix)), _lib.ptr(out),
                  _lib.stream_handle(pts.device))
    return out.view(torch.bool)
