"""Runtime controls and the per-call option snapshot.

Mirrors gswarp/_internal/backends/warp/runtime.py:33-516 (flags, setters,
``ExecutionOptions``) and gswarp/_tuning.py's public helpers.  Only
``compute_depth`` and the tile-coverage mode change what the kernels do.
The binning sort modes of the reference ("warp_radix", "torch",
"warp_depth_stable_tile") all produce the same canonical pair order, so every
mode name is accepted and served by the one native radix sort.  Auto-tuning
switches are accepted for compatibility; launch shapes here are fixed per
kernel for sm_100a.
"""

from __future__ import annotations

import os
from contextlib import contextmanager
from contextvars import ContextVar
from dataclasses import dataclass
from typing import Any

import torch

from . import _coverage

BLOCK_X = 16
BLOCK_Y = 16
BINNING_SORT_MODES = ("warp_radix", "torch", "warp_depth_stable_tile")
DEFAULT_BACKWARD_MODE = "manual"
DEFAULT_BINNING_SORT_MODE = "warp_depth_stable_tile"
DEFAULT_TILE_COVERAGE_MODE = "auto"

_BACKWARD_MODE = DEFAULT_BACKWARD_MODE
_BINNING_SORT_MODE = DEFAULT_BINNING_SORT_MODE
_TILE_COVERAGE_MODE = DEFAULT_TILE_COVERAGE_MODE
_COMPUTE_DEPTH = os.environ.get("GSWARP_COMPUTE_DEPTH", "1") != "0"
_AUTO_TUNE_ENABLED = True
_AUTO_TUNE_VERBOSE = True

# Kernel classes whose launch shapes the native library reports
# (gsb_block_dim): the sm_100a shapes are fixed at compile time.
KERNEL_CLASSES = (
    "preprocess", "preprocess_sh16", "sh_colors_views", "binning_scan", "binning_emit", "radix_sort",
    "render_forward", "render_backward", "render_backward_small_grid", "backward_preprocess", "backward_preprocess_sh16", "sh_backward_views",
    "ssim_fwd", "ssim_bwd", "ssim_fwd_h", "ssim_fwd_v", "ssim_bwd_h", "ssim_bwd_v", "knn_morton", "knn_gather",
    "knn_box_minmax", "knn_box_dist", "knn_search", "adam",
)
_REGISTERED_KERNEL_CLASSES: dict[str, tuple[int, str]] = {}


@dataclass(frozen=True, slots=True)
class ExecutionOptions:
    """Immutable runtime choices owned by one frontend invocation."""

    backward_mode: str
    binning_sort_mode: str
    tile_coverage_mode: str
    compute_depth: bool
    auto_tune: bool
    auto_tune_verbose: bool


_ACTIVE: ContextVar[ExecutionOptions | None] = ContextVar("gswarp_b200_execution_options", default=None)


@contextmanager
def execution_options(options: ExecutionOptions):
    token = _ACTIVE.set(options)
    try:
        yield options
    finally:
        _ACTIVE.reset(token)


def get_active_options() -> ExecutionOptions | None:
    return _ACTIVE.get()


def get_active_compute_depth() -> bool:
    o = _ACTIVE.get()
    return _COMPUTE_DEPTH if o is None else o.compute_depth


def get_active_tile_coverage_mode() -> str:
    o = _ACTIVE.get()
    return _TILE_COVERAGE_MODE if o is None else o.tile_coverage_mode


def get_backward_mode() -> str:
    return _BACKWARD_MODE


def set_backward_mode(mode: str) -> None:
    global _BACKWARD_MODE
    if mode != "manual":
        raise ValueError("mode must be 'manual'")
    _BACKWARD_MODE = mode


def get_binning_sort_mode() -> str:
    return _BINNING_SORT_MODE


def set_binning_sort_mode(mode: str) -> None:
    global _BINNING_SORT_MODE
    if mode not in BINNING_SORT_MODES:
        raise ValueError("mode must be one of 'torch', 'warp_radix', or 'warp_depth_stable_tile'")
    _BINNING_SORT_MODE = mode


def get_tile_coverage_mode() -> str:
    return _TILE_COVERAGE_MODE


def set_tile_coverage_mode(mode: str) -> None:
    global _TILE_COVERAGE_MODE
    _TILE_COVERAGE_MODE = _coverage.check_policy(mode)


def get_compute_depth() -> bool:
    return _COMPUTE_DEPTH


def set_compute_depth(enabled: bool) -> None:
    global _COMPUTE_DEPTH
    _COMPUTE_DEPTH = bool(enabled)


def get_runtime_auto_tuning_config() -> tuple[bool, bool]:
    return _AUTO_TUNE_ENABLED, _AUTO_TUNE_VERBOSE


def set_runtime_auto_tuning(enabled: bool = True, verbose: bool = True) -> None:
    global _AUTO_TUNE_ENABLED, _AUTO_TUNE_VERBOSE
    _AUTO_TUNE_ENABLED = bool(enabled)
    _AUTO_TUNE_VERBOSE = bool(verbose)


def resolve_execution_options(raster_settings) -> ExecutionOptions:
    """Merge global defaults and per-call settings (runtime_context.py:12-36)."""
    backward_mode = getattr(raster_settings, "backward_mode", None)
    sort_mode = getattr(raster_settings, "binning_sort_mode", None)
    if backward_mode is not None and backward_mode != "manual":
        raise ValueError("mode must be 'manual'")
    if sort_mode is not None and sort_mode not in BINNING_SORT_MODES:
        raise ValueError("sort_mode must be one of 'torch', 'warp_radix', or 'warp_depth_stable_tile'")
    return ExecutionOptions(
        backward_mode=_BACKWARD_MODE if backward_mode is None else backward_mode,
        binning_sort_mode=_BINNING_SORT_MODE if sort_mode is None else sort_mode,
        tile_coverage_mode=_coverage.concrete(_TILE_COVERAGE_MODE),
        compute_depth=_COMPUTE_DEPTH,
        auto_tune=bool(getattr(raster_settings, "auto_tune", True)),
        auto_tune_verbose=bool(getattr(raster_settings, "auto_tune_verbose", True)),
    )


def normalize_device(device=None) -> torch.device:
    if device is None:
        return torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")
    d = torch.device(device)
    if d.type == "cuda" and d.index is None and torch.cuda.is_available():
        d = torch.device("cuda", torch.cuda.current_device())
    return d


def get_canonical_device(device=None) -> str:
    return str(normalize_device(device))


def register_kernel_class(name: str, registers_per_thread: int, family: str = "compute") -> None:
    """Accepted for API compatibility (gswarp/_tuning.py); launch shapes are fixed."""
    _REGISTERED_KERNEL_CLASSES[str(name)] = (int(registers_per_thread), str(family))


def get_tuned_block_dim(kernel_class: str, device=None) -> int:
    """Threads per CTA the native library launches for ``kernel_class``
    (the reference returns its tuned block_dim, or 256 when it has none,
    gswarp/_tuning.py:342-375); a class the library does not launch gets
    the reference's default of 256."""
    from . import _lib

    n = int(_lib.load().gsb_block_dim(str(kernel_class).encode()))
    return n if n > 0 else 256


def get_default_parameter_info() -> dict[str, dict[str, Any]]:
    return {
        "BLOCK_X": {"value": BLOCK_X, "category": "kernel_tile", "auto_tunable": False,
                    "description": "Tile width of the render kernels (compile-time)."},
        "BLOCK_Y": {"value": BLOCK_Y, "category": "kernel_tile", "auto_tunable": False,
                    "description": "Tile height of the render kernels (compile-time)."},
        "DEFAULT_BACKWARD_MODE": {"value": DEFAULT_BACKWARD_MODE, "category": "runtime",
                                  "auto_tunable": False, "description": "Only 'manual' exists."},
        "DEFAULT_BINNING_SORT_MODE": {"value": DEFAULT_BINNING_SORT_MODE, "category": "runtime",
                                      "auto_tunable": False,
                                      "description": "All modes map to the native stable radix sort."},
        "DEFAULT_TILE_COVERAGE_MODE": {"value": DEFAULT_TILE_COVERAGE_MODE, "category": "runtime",
                                       "auto_tunable": False,
                                       "description": "'auto' resolves to AccuTile for baseline 3DGS."},
    }


_TUNING_REPORTS: dict[str, dict[str, Any]] = {}


def initialize_runtime_tuning(device=None, verbose: bool = True) -> dict[str, Any]:
    d = normalize_device(device)
    key = str(d)
    rep = _TUNING_REPORTS.get(key)
    if rep is None:
        rep = {"device": key, "kernel_block_dims": {k: get_tuned_block_dim(k) for k in KERNEL_CLASSES}, "backend": "gswarp_b200 sm_100a"}
        if d.type == "cuda" and torch.cuda.is_available():
            p = torch.cuda.get_device_properties(d)
            rep.update(name=p.name, sm_count=p.multi_processor_count,
                       total_memory_bytes=p.total_memory, capability=f"{p.major}.{p.minor}")
        _TUNING_REPORTS[key] = rep
        if verbose:
            print(f"[gswarp_b200] {rep}")
    return dict(rep)


def get_runtime_tuning_report(device=None) -> dict[str, Any]:
    return initialize_runtime_tuning(device, verbose=False)
