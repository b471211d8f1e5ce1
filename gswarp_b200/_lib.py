"""ctypes bindings of libgsb200.so (the C ABI declared in include/gsb200.h).

The shared library is built in-tree by ``gswarp_b200/csrc/build.py`` into
``gswarp_b200/_lib/libgsb200.so``.  There is no fallback: if the library is
missing or fails to load, every operation raises.  The structures below
mirror the C structs field for field.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "_lib" / "libgsb200.so"

GSB_OK = 0
GSB_ERR_INVALID = -1
GSB_ERR_OVERFLOW = -2
GSB_ERR_CUDA = -3
GSB_ERR_TIMEOUT = -4

ABI_VERSION = 16
RECORD_FLOATS = 12
GRAD_FLOATS = 12

c_int = ctypes.c_int
c_float = ctypes.c_float
c_ll = ctypes.c_longlong
vp = ctypes.c_void_p


class PreprocessArgs(ctypes.Structure):
    _fields_ = [
        ("P", c_int), ("W", c_int), ("H", c_int),
        ("means", vp), ("scales", vp), ("rotations", vp), ("cov3d_precomp", vp),
        ("scale_modifier", c_float),
        ("opacities", vp), ("viewmatrix", vp), ("projmatrix", vp), ("campos", vp),
        ("tanfovx", c_float), ("tanfovy", c_float), ("focal_x", c_float), ("focal_y", c_float),
        ("sh", vp), ("sh_degree", c_int), ("sh_coeffs", c_int),
        ("colors_precomp", vp),
        ("coverage_mode", c_int),
        ("radii", vp), ("proj_2d", vp), ("conic_2d", vp), ("conic_2d_inv", vp), ("depths", vp),
        ("tiles_touched", vp), ("records", vp), ("cov3d_out", vp), ("bin_records", vp),
        ("sparse_records", c_int), ("colors_clamp_signed", c_int),
    ]


class BinCountArgs(ctypes.Structure):
    _fields_ = [
        ("P", c_int),
        ("depths", vp), ("radii", vp), ("tiles_touched", vp),
        ("depth_order", vp), ("point_offsets", vp), ("binned_ids", vp), ("status_out", vp),
        ("workspace", vp), ("workspace_bytes", ctypes.c_size_t),
    ]


class BinSortArgs(ctypes.Structure):
    _fields_ = [
        ("P", c_int), ("W", c_int), ("H", c_int),
        ("num_rendered", c_ll),
        ("coverage_mode", c_int),
        ("depth_order", vp), ("point_offsets", vp), ("radii", vp), ("records", vp),
        ("conic_2d_inv", vp), ("tiles_touched", vp),
        ("point_list", vp), ("ranges", vp), ("error_word", vp),
        ("workspace", vp), ("workspace_bytes", ctypes.c_size_t), ("bin_records", vp),
        ("bin_status", vp),
    ]


class RenderFwdArgs(ctypes.Structure):
    _fields_ = [
        ("W", c_int), ("H", c_int), ("compute_depth", c_int),
        ("ranges", vp), ("point_list", vp), ("records", vp), ("background", vp),
        ("out_color", vp), ("out_depth", vp), ("out_alpha", vp), ("n_contrib", vp),
        ("top_k", c_int), ("gs_per_pixel", vp), ("weight_per_gs_pixel", vp), ("x_mu", vp),
        ("aux_scratch", vp),
    ]


class RenderBwdArgs(ctypes.Structure):
    _fields_ = [
        ("W", c_int), ("H", c_int), ("P", c_int), ("compute_depth", c_int),
        ("ranges", vp), ("point_list", vp), ("records", vp), ("background", vp),
        ("out_alpha", vp), ("n_contrib", vp),
        ("grad_color", vp), ("grad_depth", vp), ("grad_alpha", vp),
        ("grad_acc", vp),
    ]


class PreprocessBwdArgs(ctypes.Structure):
    _fields_ = [
        ("P", c_int), ("W", c_int), ("H", c_int),
        ("means", vp), ("radii", vp), ("scales", vp), ("rotations", vp), ("cov3d_precomp", vp),
        ("scale_modifier", c_float),
        ("viewmatrix", vp), ("projmatrix", vp), ("campos", vp),
        ("tanfovx", c_float), ("tanfovy", c_float), ("focal_x", c_float), ("focal_y", c_float),
        ("sh", vp), ("sh_degree", c_int), ("sh_coeffs", c_int),
        ("records", vp), ("grad_acc", vp),
        ("grad_proj_2d", vp), ("grad_conic_2d", vp), ("grad_conic_2d_inv", vp),
        ("accumulate", c_int),
        ("grad_means3d", vp), ("grad_means2d", vp), ("grad_scales", vp), ("grad_rotations", vp),
        ("grad_opacity", vp), ("grad_sh", vp), ("grad_colors", vp), ("grad_cov3d", vp),
        ("ids", vp), ("num_ids", c_int), ("clear_grad_acc", c_int), ("densify_grad_accum", vp),
        ("grad_colors_clamped", c_int),
    ]


class SHViewsArgs(ctypes.Structure):
    _fields_ = [
        ("P", c_int), ("num_views", c_int), ("sh_degree", c_int), ("sh_coeffs", c_int),
        ("means", vp), ("sh", vp), ("campos", vp), ("colors", vp),
        ("grad_colors", vp), ("clear_grad_colors", c_int), ("grad_sh", vp), ("grad_means3d", vp),
        ("accumulate", c_int), ("begin", c_int), ("end", c_int),
    ]


class SSIMFwdArgs(ctypes.Structure):
    _fields_ = [
        ("B", c_int), ("C", c_int), ("H", c_int), ("W", c_int),
        ("valid", c_int), ("C1", c_float), ("C2", c_float),
        ("img1", vp), ("img2", vp), ("dm", vp), ("partials", vp), ("loss", vp),
    ]


class SSIMBwdArgs(ctypes.Structure):
    _fields_ = [
        ("B", c_int), ("C", c_int), ("H", c_int), ("W", c_int),
        ("valid", c_int),
        ("img1", vp), ("img2", vp), ("dm", vp), ("upstream", vp), ("grad_img1", vp),
    ]


class PhotoLossFwdArgs(ctypes.Structure):
    _fields_ = [
        ("B", c_int), ("C", c_int), ("H", c_int), ("W", c_int),
        ("C1", c_float), ("C2", c_float), ("w_l1", c_float), ("w_ssim", c_float),
        ("img", vp), ("target", vp), ("dm", vp), ("partials", vp), ("loss_out", vp),
    ]


class PhotoLossBwdArgs(ctypes.Structure):
    _fields_ = [
        ("B", c_int), ("C", c_int), ("H", c_int), ("W", c_int),
        ("w_l1", c_float), ("w_ssim", c_float), ("upstream", c_float),
        ("img", vp), ("target", vp), ("dm", vp), ("grad_img", vp),
    ]


class AdamArgs(ctypes.Structure):
    _fields_ = [
        ("P", c_int), ("sh_coeffs", c_int), ("params", vp * 5),
        ("grad", vp), ("exp_avg", vp), ("exp_avg_sq", vp),
        ("lr", ctypes.c_double * 6), ("beta1", ctypes.c_double), ("beta2", ctypes.c_double),
        ("eps", ctypes.c_double), ("step", c_int),
    ]


class KNNArgs(ctypes.Structure):
    _fields_ = [
        ("P", c_int), ("points", vp), ("out", vp), ("error_word", vp),
        ("workspace", vp), ("workspace_bytes", ctypes.c_size_t),
    ]


_lib = None
_lib_lock = threading.Lock()

EXPORTED = (
    "gsb_abi_version", "gsb_last_error", "gsb_preprocess_fwd", "gsb_mark_visible",
    "gsb_bin_count_workspace_bytes", "gsb_bin_count", "gsb_bin_sort_workspace_bytes",
    "gsb_bin_emit_sort", "gsb_render_fwd", "gsb_render_bwd", "gsb_preprocess_bwd",
    "gsb_ssim_partials_count", "gsb_ssim_fwd", "gsb_ssim_bwd", "gsb_knn_workspace_bytes",
    "gsb_knn", "gsb_selftest_threshold_log", "gsb_ssim_fwd_noalloc", "gsb_photo_loss_fwd",
    "gsb_photo_loss_bwd", "gsb_adam_step", "gsb_densify_stats", "gsb_sh_colors_views",
    "gsb_sh_backward_views", "gsb_block_dim", "gsb_peak_fp32", "gsb_peak_ex2", "gsb_peak_work",
)


def _declare(L) -> None:
    def fn(name, res, args):
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args

    P = ctypes.POINTER
    fn("gsb_abi_version", c_int, [])
    fn("gsb_last_error", ctypes.c_char_p, [])
    fn("gsb_block_dim", c_int, [ctypes.c_char_p])
    fn("gsb_peak_fp32", c_int, [c_int, c_int, vp, vp])
    fn("gsb_peak_ex2", c_int, [c_int, c_int, vp, vp])
    fn("gsb_peak_work", c_ll, [c_int, c_int, c_int])
    fn("gsb_preprocess_fwd", c_int, [P(PreprocessArgs), vp])
    fn("gsb_mark_visible", c_int, [c_int, vp, vp, vp, vp])
    fn("gsb_bin_count_workspace_bytes", ctypes.c_size_t, [c_int])
    fn("gsb_bin_count", c_int, [P(BinCountArgs), vp])
    fn("gsb_bin_sort_workspace_bytes", ctypes.c_size_t, [c_ll, c_int, c_int])
    fn("gsb_bin_emit_sort", c_int, [P(BinSortArgs), vp])
    fn("gsb_render_fwd", c_int, [P(RenderFwdArgs), vp])
    fn("gsb_render_bwd", c_int, [P(RenderBwdArgs), vp])
    fn("gsb_preprocess_bwd", c_int, [P(PreprocessBwdArgs), vp])
    fn("gsb_ssim_partials_count", c_int, [c_int, c_int, c_int, c_int])
    fn("gsb_ssim_fwd", c_int, [P(SSIMFwdArgs), vp])
    fn("gsb_ssim_bwd", c_int, [P(SSIMBwdArgs), vp])
    fn("gsb_photo_loss_fwd", c_int, [P(PhotoLossFwdArgs), vp])
    fn("gsb_photo_loss_bwd", c_int, [P(PhotoLossBwdArgs), vp])
    fn("gsb_adam_step", c_int, [P(AdamArgs), vp])
    fn("gsb_densify_stats", c_int, [c_int, vp, vp, vp, vp])
    fn("gsb_sh_colors_views", c_int, [P(SHViewsArgs), vp])
    fn("gsb_sh_backward_views", c_int, [P(SHViewsArgs), vp])
    fn("gsb_knn_workspace_bytes", ctypes.c_size_t, [c_int])
    fn("gsb_knn", c_int, [P(KNNArgs), vp])
    fn("gsb_selftest_threshold_log", c_int, [vp, vp, c_ll, vp])


def load():
    """Load (once) and return the native library; raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lib_lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise ImportError(
                    f"gswarp_b200 native library not found at {LIB_PATH}; "
                    "build it with `python -c 'import __graft_entry__ as g; g.build()'` "
                    "or `python gswarp_b200/csrc/build.py`"
                )
            L = ctypes.CDLL(str(LIB_PATH), mode=os.RTLD_LOCAL)
            _declare(L)
            if L.gsb_abi_version() != ABI_VERSION:
                raise ImportError("libgsb200.so ABI version mismatch; rebuild the library")
            _lib = L
    return _lib


def ptr(t: torch.Tensor | None):
    """Raw device pointer of a tensor (None -> NULL)."""
    if t is None:
        return None
    return ctypes.c_void_p(t.data_ptr())


def stream_handle(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def check(status: int, what: str) -> None:
    if status == GSB_OK:
        return
    msg = load().gsb_last_error()
    msg = msg.decode() if msg else what
    if status == GSB_ERR_INVALID:
        raise ValueError(msg)
    if status == GSB_ERR_OVERFLOW:
        raise OverflowError(msg)
    raise RuntimeError(f"{what} failed ({status}): {msg}")


def call(name: str, *args) -> None:
    L = load()
    check(getattr(L, name)(*args), name)
