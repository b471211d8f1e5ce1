"""gswarp_b200 -- B200-native (sm_100a) 3DGS training hot path behind
gswarp's drop-in API: GaussianRasterizationSettings / GaussianRasterizer,
fused_ssim and distCUDA2."""

__version__ = "0.1.0"

from .rasterizer import (  # noqa: F401
    GaussianRasterizationSettings,
    GaussianRasterizer,
    RasterizerMeta,
    rasterize_gaussians,
    initialize_runtime_tuning,
    get_runtime_tuning_report,
    clear_warp_caches,
    get_warp_cache_report,
    get_backward_mode,
    set_backward_mode,
    get_compute_depth,
    set_compute_depth,
    get_binning_sort_mode,
    set_binning_sort_mode,
    get_tile_coverage_mode,
    set_tile_coverage_mode,
)
from ._runtime import get_tuned_block_dim, register_kernel_class, get_canonical_device  # noqa: F401
from .fused_ssim import fused_ssim  # noqa: F401
from .knn import distCUDA2  # noqa: F401
