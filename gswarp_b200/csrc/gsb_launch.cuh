// gsb_launch.cuh -- threads per CTA of every kernel of libgsb200.  The
// kernels launch with these constants and gsb_block_dim() reports them, so
// the runtime's block-dim getter always names the shapes actually launched.
#pragma once

namespace gsb {
namespace launch {

constexpr int PREPROCESS = 256;          // preprocess_fwd_kernel, colours given or SH rows of any width
constexpr int PREPROCESS_SH16 = 128;     // preprocess_fwd_kernel with (P,16,3) SH rows staged per warp
constexpr int SH_COLORS_VIEWS = 128;     // sh_colors_views_kernel
constexpr int BINNING_SCAN = 256;        // compact_kernel, depth_scan_kernel
constexpr int BINNING_EMIT = 256;        // emit_binrec_kernel, emit_kernel
constexpr int RADIX_SORT = 256;          // histogram_kernel, onesweep_kernel, bin_base_kernel
constexpr int RENDER = 128;              // render_fwd_kernel, render_bwd_tile4_kernel (16x16 tile, 2 px/thread)
constexpr int RENDER_BWD = 64;           // render_bwd_tile2_kernel (16x16 tile, 4 px/thread; grids of >= 6,000 tiles)
constexpr int PREPROCESS_BWD = 256;      // preprocess_bwd_kernel, no SH or SH rows of any width
constexpr int PREPROCESS_BWD_SH16 = 128; // preprocess_bwd_kernel with (P,16,3) SH rows staged per warp
constexpr int SH_BACKWARD_VIEWS = 128;   // sh_backward_views_kernel
constexpr int SSIM = 256;                // ssim_fwd_kernel, ssim_bwd_kernel (fused H+V passes)
constexpr int KNN = 256;                 // morton, gather/leaf boxes, box reductions, search (a warp per leaf)
constexpr int ADAM = 256;                // adam_kernel, densify_stats_kernel

}  // namespace launch
}  // namespace gsb
