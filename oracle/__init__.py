"""CPU parity oracle for gswarp_b200 (test infrastructure only).

ctypes bindings over ``oracle/_build/liboracle.so`` (built from
``oracle/gsb_oracle.cpp`` by ``oracle/Makefile``).  The C++ file restates the
arithmetic of gswarp v1.1.0's Warp kernels for the 3DGS training path; every
function there cites the reference file:line it follows.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this package.  The product (``gswarp_b200``) never does.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "liboracle.so"
_lib = None

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")


def build(force: bool = False) -> Path:
    """Compile the oracle library with its Makefile (no-op when up to date)."""
    if force or not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < (_HERE / "gsb_oracle.cpp").stat().st_mtime:
        subprocess.run(["make", "-C", str(_HERE), "CXX=g++"], check=True, capture_output=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = ctypes.CDLL(str(_LIB_PATH))
        _declare(_lib)
    return _lib


def _opt(arr):
    """numpy array or None -> pointer (None passes NULL)."""
    if arr is None:
        return None
    return arr.ctypes.data_as(ctypes.c_void_p)


def _declare(L):
    c_int, c_float, c_ll, vp = ctypes.c_int, ctypes.c_float, ctypes.c_longlong, ctypes.c_void_p
    L.or_count_tiles.restype = c_int
    L.or_count_tiles.argtypes = [c_float] * 8 + [c_int] * 4
    L.or_emit_tiles.restype = c_int
    L.or_emit_tiles.argtypes = [c_float] * 8 + [c_int] * 4 + [_i32p, c_int]
    L.or_threshold_log.restype = c_float
    L.or_threshold_log.argtypes = [c_float]
    L.or_threshold_log_batch.restype = None
    L.or_threshold_log_batch.argtypes = [_f32p, _f32p, c_ll]
    L.or_preprocess_fwd.restype = None
    L.or_preprocess_fwd.argtypes = (
        [c_int, _f32p, vp, vp, c_float, vp, _f32p, _f32p, _f32p]
        + [c_float] * 4 + [c_int] * 3 + [vp, c_int, c_int, vp]
        + [_f32p, _i32p, _f32p, _i32p, _f32p, _f32p, _f32p, _i32p, _f32p, vp, vp]
    )
    L.or_mark_visible.restype = None
    L.or_mark_visible.argtypes = [c_int, _f32p, _f32p, _u8p]
    L.or_binning.restype = c_ll
    L.or_binning.argtypes = [c_int, _f32p, _i32p, _f32p, _f32p, _f32p, _i32p, c_int, c_int, c_int,
                             vp, c_ll, _i32p, vp]
    L.or_render_fwd.restype = None
    L.or_render_fwd.argtypes = [c_int, c_int, _i32p, _i32p, _f32p, _f32p, _f32p, _f32p, _f32p, c_int,
                                _f32p, _f32p, _f32p, _i32p, vp, vp]
    L.or_render_flow_aux.restype = None
    L.or_render_flow_aux.argtypes = [c_int, c_int, _i32p, _i32p, _f32p, _f32p, c_int, _i32p, _f32p, _f32p]
    L.or_render_bwd.restype = None
    L.or_render_bwd.argtypes = [c_int, c_int, c_int, _i32p, _i32p, _f32p, _f32p, _f32p, _f32p, _f32p,
                                _f32p, _i32p, _f32p, _f32p, _f32p, c_int,
                                _f32p, _f32p, _f32p, _f32p, vp, vp, c_float, vp, vp]
    L.or_preprocess_bwd.restype = None
    L.or_preprocess_bwd.argtypes = (
        [c_int, _f32p, _i32p, vp, vp, c_float, vp, _f32p, _f32p] + [c_float] * 4
        + [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, vp, c_int, c_int, vp, vp]
        + [_f32p, _f32p, vp, vp, _f32p, vp, vp, vp]
    )
    L.or_ssim_fwd.restype = None
    L.or_ssim_fwd.argtypes = [c_int] * 4 + [_f32p, _f32p, c_float, c_float, c_int,
                                            ctypes.POINTER(ctypes.c_double), vp, vp, vp, vp]
    L.or_ssim_bwd.restype = None
    L.or_ssim_bwd.argtypes = [c_int] * 4 + [_f32p, _f32p, _f32p, _f32p, _f32p, c_float, c_float,
                                            c_int, _f32p]
    L.or_knn_bounds.restype = None
    L.or_knn_bounds.argtypes = [c_int, _f32p, _f32p, _f32p]
    L.or_knn_codes.restype = None
    L.or_knn_codes.argtypes = [c_int, _f32p, _f32p, _f32p, _u32p]
    L.or_knn.restype = c_ll
    L.or_knn.argtypes = [c_int, _f32p, _f32p]
    L.or_knn_bruteforce.restype = None
    L.or_knn_bruteforce.argtypes = [c_int, _f32p, _f32p]
    L.or_num_threads.restype = c_int
    L.or_num_threads.argtypes = []
    L.or_set_num_threads.restype = None
    L.or_set_num_threads.argtypes = [c_int]


def _c(a, dtype=np.float32):
    return np.ascontiguousarray(np.asarray(a, dtype=dtype))


def num_threads() -> int:
    return int(lib().or_num_threads())


def set_num_threads(n: int) -> int:
    """Sets the oracle's OpenMP thread count (overriding OMP_NUM_THREADS) and
    returns the count now in effect."""
    lib().or_set_num_threads(int(n))
    return num_threads()


def count_tiles(px, py, cov_aa, cov_cc, ca, cb, cc, opacity, radius, grid_x, grid_y, mode=1) -> int:
    return int(lib().or_count_tiles(px, py, cov_aa, cov_cc, ca, cb, cc, opacity, radius, grid_x, grid_y, mode))


def emit_tiles(px, py, cov_aa, cov_cc, ca, cb, cc, opacity, radius, grid_x, grid_y, mode=1):
    cap = max(1, grid_x * grid_y)
    out = np.zeros(cap, dtype=np.int32)
    n = lib().or_emit_tiles(px, py, cov_aa, cov_cc, ca, cb, cc, opacity, radius, grid_x, grid_y, mode, out, cap)
    return out[:n].copy()


def threshold_log(x):
    x = _c(x)
    out = np.empty_like(x)
    lib().or_threshold_log_batch(x, out, x.size)
    return out


def preprocess_fwd(means, opacities, view, proj, tanfovx, tanfovy, W, H, *, scales=None,
                   rotations=None, cov3d_precomp=None, scale_modifier=1.0, sh=None, degree=0,
                   campos=None, mode=1):
    """Returns a dict of numpy outputs (same names as the CUDA path)."""
    means = _c(means).reshape(-1, 3)
    P = means.shape[0]
    opac = _c(opacities).reshape(-1)
    view = _c(view).reshape(-1)
    proj = _c(proj).reshape(-1)
    focal_x = np.float32(W / (2.0 * float(tanfovx)))
    focal_y = np.float32(H / (2.0 * float(tanfovy)))
    sc = _c(scales).reshape(-1, 3) if scales is not None else None
    ro = _c(rotations).reshape(-1, 4) if rotations is not None else None
    cp = _c(cov3d_precomp).reshape(-1, 6) if cov3d_precomp is not None else None
    K = 0
    shf = None
    if sh is not None:
        shf = _c(sh).reshape(P, -1, 3)
        K = shf.shape[1]
    cam = _c(campos).reshape(-1) if campos is not None else np.zeros(3, np.float32)
    out = dict(
        cov3d=np.zeros((P, 6), np.float32), visible=np.zeros(P, np.int32),
        depths=np.zeros(P, np.float32), radii=np.zeros(P, np.int32),
        proj_2d=np.zeros((P, 2), np.float32), conic_2d=np.zeros((P, 3), np.float32),
        conic_2d_inv=np.zeros((P, 3), np.float32), tiles_touched=np.zeros(P, np.int32),
        conic_opacity=np.zeros((P, 4), np.float32), rgb=np.zeros((P, 3), np.float32),
        clamped=np.zeros((P, 3), np.int32),
    )
    lib().or_preprocess_fwd(
        P, means, _opt(sc), _opt(ro), float(scale_modifier), _opt(cp), opac, view, proj,
        float(np.float32(tanfovx)), float(np.float32(tanfovy)), float(focal_x), float(focal_y), int(W), int(H), int(mode),
        _opt(shf), int(degree), int(K), _opt(cam),
        out["cov3d"], out["visible"], out["depths"], out["radii"], out["proj_2d"], out["conic_2d"],
        out["conic_2d_inv"], out["tiles_touched"], out["conic_opacity"],
        _opt(out["rgb"]) if shf is not None else None, _opt(out["clamped"]) if shf is not None else None,
    )
    return out


def mark_visible(means, view):
    means = _c(means).reshape(-1, 3)
    out = np.zeros(means.shape[0], np.uint8)
    lib().or_mark_visible(means.shape[0], means, _c(view).reshape(-1), out)
    return out.astype(bool)


def binning(pre, W, H, mode=1):
    """Canonical sorted pair list: (point_list, ranges (T,2), tile_keys)."""
    P = pre["radii"].shape[0]
    args = [P, _c(pre["proj_2d"]), _c(pre["radii"], np.int32), _c(pre["conic_opacity"]),
            _c(pre["conic_2d_inv"]), _c(pre["depths"]), _c(pre["tiles_touched"], np.int32),
            int(W), int(H), int(mode)]
    gx, gy = (W + 15) // 16, (H + 15) // 16
    ranges = np.zeros((gx * gy, 2), np.int32)
    total = int(lib().or_binning(*args, None, 0, ranges, None))
    point_list = np.zeros(max(total, 1), np.int32)
    keys = np.zeros(max(total, 1), np.int32)
    got = int(lib().or_binning(*args, _opt(point_list), total, ranges, _opt(keys)))
    if got != total:
        raise RuntimeError("oracle binning: count and emit disagree")
    return point_list[:total], ranges, keys[:total]


def render_fwd(W, H, ranges, point_list, xy, features, depths, conic_opacity, bg, compute_depth=True,
               with_margin=False):
    """(color, depth, alpha, n_contrib), plus with ``with_margin`` two (H, W)
    arrays: the per-pixel smallest relative margin of the pixel's thresholded
    decisions (exponent sign, alpha >= 1/255, T*(1-alpha) < 1e-4) and the
    largest absolute size of the exponent's terms among the pairs it blends."""
    npix = W * H
    color = np.zeros((3, H, W), np.float32)
    depth = np.zeros((1, H, W), np.float32)
    alpha = np.zeros((1, H, W), np.float32)
    n_contrib = np.zeros(npix, np.int32)
    margin = np.ones((H, W), np.float32) if with_margin else None
    cond = np.zeros((H, W), np.float32) if with_margin else None
    pl = _c(point_list, np.int32) if len(point_list) else np.zeros(1, np.int32)
    lib().or_render_fwd(W, H, _c(ranges, np.int32).reshape(-1), pl, _c(xy), _c(features), _c(depths),
                        _c(conic_opacity), _c(bg), int(bool(compute_depth)), color, depth, alpha, n_contrib,
                        _opt(margin), _opt(cond))
    if with_margin:
        return color, depth, alpha, n_contrib, margin, cond
    return color, depth, alpha, n_contrib


def render_flow_aux(W, H, ranges, point_list, xy, conic_opacity, top_k):
    """Top-K contributor outputs of the flow render: (gs_per_pixel (K,H,W) i32,
    weight_per_gs_pixel (K,H,W), x_mu (2,K,H,W))."""
    gs = np.zeros((top_k, H, W), np.int32)
    wt = np.zeros((top_k, H, W), np.float32)
    xm = np.zeros((2, top_k, H, W), np.float32)
    pl = _c(point_list, np.int32) if len(point_list) else np.zeros(1, np.int32)
    lib().or_render_flow_aux(W, H, _c(ranges, np.int32).reshape(-1), pl, _c(xy), _c(conic_opacity), int(top_k),
                             gs, wt, xm)
    return gs, wt, xm


def render_bwd(W, H, P, ranges, point_list, xy, features, depths, conic_opacity, bg, out_alpha,
               n_contrib, grad_color, grad_depth, grad_alpha, compute_depth=True, with_abs=False,
               with_margin=False, flag_eps=None):
    """Per-Gaussian render gradients; ``with_abs`` adds "abs" (P, 10), the
    sum of |term| per gradient component (xy 2, depth, conic 4, rgb 3), and
    "cond_abs" (P, 10), the sum of |term| times the absolute size of the
    term's exponent terms (its sensitivity to rounding in the exponent);
    ``with_margin`` adds "margin" (H, W), the smallest relative margin of the
    decisions the backward re-evaluates (exponent sign, alpha >= 1/255) over
    each pixel's contributors; ``flag_eps`` adds "flagged_abs" (P, 10), the
    part of "abs" that comes from pixels whose margin is below flag_eps."""
    g_xy = np.zeros((P, 2), np.float32)
    g_d = np.zeros(P, np.float32)
    g_co = np.zeros((P, 4), np.float32)
    g_rgb = np.zeros((P, 3), np.float32)
    g_abs = np.zeros((P, 10), np.float64) if with_abs else None
    margin = np.ones((H, W), np.float32) if with_margin else None
    flagged = np.zeros((P, 10), np.float64) if flag_eps is not None else None
    cond = np.zeros((P, 10), np.float64) if with_abs else None
    pl = _c(point_list, np.int32) if len(point_list) else np.zeros(1, np.int32)
    lib().or_render_bwd(W, H, P, _c(ranges, np.int32).reshape(-1), pl, _c(xy), _c(features), _c(depths),
                        _c(conic_opacity), _c(bg), _c(out_alpha).reshape(-1), _c(n_contrib, np.int32),
                        _c(grad_color).reshape(-1), _c(grad_depth).reshape(-1), _c(grad_alpha).reshape(-1),
                        int(bool(compute_depth)), g_xy, g_d, g_co, g_rgb, _opt(g_abs), _opt(margin),
                        float(flag_eps or 0.0), _opt(flagged), _opt(cond))
    out = dict(grad_xy=g_xy, grad_depth=g_d, grad_conic_opacity=g_co, grad_rgb=g_rgb)
    if with_abs:
        out["abs"] = g_abs
        out["cond_abs"] = cond
    if with_margin:
        out["margin"] = margin
    if flag_eps is not None:
        out["flagged_abs"] = flagged
    return out


def preprocess_bwd(means, radii, view, proj, tanfovx, tanfovy, W, H, render_grads, grad_proj_2d,
                   grad_conic_2d, grad_conic_2d_inv, *, scales=None, rotations=None, cov3d_precomp=None,
                   scale_modifier=1.0, sh=None, degree=0, campos=None, clamped=None):
    means = _c(means).reshape(-1, 3)
    P = means.shape[0]
    focal_x = np.float32(W / (2.0 * float(tanfovx)))
    focal_y = np.float32(H / (2.0 * float(tanfovy)))
    K = 0
    shf = None
    if sh is not None:
        shf = _c(sh).reshape(P, -1, 3)
        K = shf.shape[1]
    out = dict(
        grad_means3d=np.zeros((P, 3), np.float32), grad_means2d=np.zeros((P, 3), np.float32),
        grad_opacity=np.zeros(P, np.float32),
    )
    gs = np.zeros((P, 3), np.float32) if cov3d_precomp is None else None
    gr = np.zeros((P, 4), np.float32) if cov3d_precomp is None else None
    gc3 = np.zeros((P, 6), np.float32) if cov3d_precomp is not None else None
    gsh = np.zeros((P, max(K, 1), 3), np.float32) if shf is not None else None
    gcol = np.zeros((P, 3), np.float32) if shf is None else None
    cam = _c(campos).reshape(-1) if campos is not None else np.zeros(3, np.float32)
    cl = _c(clamped, np.int32).reshape(-1, 3) if clamped is not None else np.zeros((P, 3), np.int32)
    lib().or_preprocess_bwd(
        P, means, _c(radii, np.int32), _opt(_c(scales).reshape(-1, 3) if scales is not None else None),
        _opt(_c(rotations).reshape(-1, 4) if rotations is not None else None), float(scale_modifier),
        _opt(_c(cov3d_precomp).reshape(-1, 6) if cov3d_precomp is not None else None),
        _c(view).reshape(-1), _c(proj).reshape(-1), float(np.float32(tanfovx)), float(np.float32(tanfovy)),
        float(focal_x), float(focal_y),
        _c(render_grads["grad_xy"]), _c(render_grads["grad_depth"]), _c(render_grads["grad_conic_opacity"]),
        _c(render_grads["grad_rgb"]), _c(grad_proj_2d), _c(grad_conic_2d), _c(grad_conic_2d_inv),
        _opt(shf), int(degree), int(K), _opt(cam), _opt(cl),
        out["grad_means3d"], out["grad_means2d"], _opt(gs), _opt(gr), out["grad_opacity"],
        _opt(gsh), _opt(gcol), _opt(gc3),
    )
    if gs is not None:
        out["grad_scales"] = gs
        out["grad_rotations"] = gr
    if gc3 is not None:
        out["grad_cov3d"] = gc3
    if gsh is not None:
        out["grad_sh"] = gsh
    if gcol is not None:
        out["grad_colors"] = gcol
    return out


C1 = 0.01 ** 2
C2 = 0.03 ** 2


def ssim_fwd(img1, img2, valid=False):
    img1 = _c(img1)
    img2 = _c(img2)
    B, CH, H, W = img1.shape
    s = ctypes.c_double(0.0)
    if valid:
        smap = np.zeros((B, CH, H - 10, W - 10), np.float32)
    else:
        smap = np.zeros_like(img1)
    dm = [np.zeros_like(img1) for _ in range(3)]
    lib().or_ssim_fwd(B, CH, H, W, img1, img2, float(np.float32(C1)), float(np.float32(C2)), int(valid),
                      ctypes.byref(s), _opt(smap), _opt(dm[0]), _opt(dm[1]), _opt(dm[2]))
    n = smap.size
    return s.value / n, smap, dm


def ssim_bwd(img1, img2, dm, upstream=1.0, valid=False):
    img1 = _c(img1)
    img2 = _c(img2)
    B, CH, H, W = img1.shape
    n = B * CH * (H - 10) * (W - 10) if valid else B * CH * H * W
    inv_n = float(np.float32(1.0 / float(n)))
    grad = np.zeros_like(img1)
    lib().or_ssim_bwd(B, CH, H, W, img1, img2, _c(dm[0]), _c(dm[1]), _c(dm[2]), inv_n,
                      float(np.float32(upstream)), int(valid), grad)
    return grad


def knn(points):
    pts = _c(points).reshape(-1, 3)
    out = np.zeros(pts.shape[0], np.float32)
    evals = lib().or_knn(pts.shape[0], pts, out)
    return out, int(evals)


def knn_bruteforce(points):
    pts = _c(points).reshape(-1, 3)
    out = np.zeros(pts.shape[0], np.float32)
    lib().or_knn_bruteforce(pts.shape[0], pts, out)
    return out


def knn_codes(points):
    pts = _c(points).reshape(-1, 3)
    mn = np.zeros(3, np.float32)
    mx = np.zeros(3, np.float32)
    lib().or_knn_bounds(pts.shape[0], pts, mn, mx)
    codes = np.zeros(pts.shape[0], np.uint32)
    lib().or_knn_codes(pts.shape[0], pts, mn, mx, codes)
    return codes, mn, mx
