/*
 * gsb200.h -- C ABI of libgsb200.so, the sm_100a kernels behind gswarp_b200.
 *
 * Every entry point takes plain device pointers, sizes and scalars plus a
 * cudaStream_t (passed as void*), enqueues its kernels on that stream and
 * returns an int status (GSB_OK or a negative GSB_ERR_* code; the message is
 * available from gsb_last_error() on the calling thread).  The library never
 * allocates device memory: every output and workspace buffer is provided by
 * the caller, sized with the *_workspace_bytes() queries.  It keeps no state
 * between calls and is safe to call from several host threads on different
 * streams.
 *
 * Each entry point replaces a stage of gswarp v1.1.0 (fancifulland2718/gswarp);
 * the reference interface it stands in for is cited beside it, by file:line
 * inside that project.
 *
 * Floating point conventions: view/proj matrices are 16 floats read as
 * flat[c*4+r] (the transposed 3DGS world_view_transform / full_proj_transform,
 * exactly what the reference kernels read, preprocess_kernels.py:134).
 */
#ifndef GSB200_H
#define GSB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GSB_ABI_VERSION 16

#define GSB_OK 0
#define GSB_ERR_INVALID (-1)  /* bad argument: ValueError in Python          */
#define GSB_ERR_OVERFLOW (-2) /* int32 pair-count overflow: OverflowError    */
#define GSB_ERR_CUDA (-3)     /* CUDA launch / runtime error: RuntimeError   */
#define GSB_ERR_TIMEOUT (-4)  /* a bounded device-side wait gave up          */

/* Tile-coverage modes (gswarp/_internal/coverage.py:80-84). */
#define GSB_COVERAGE_SNUGBOX 0
#define GSB_COVERAGE_ACCUTILE 1
#define GSB_COVERAGE_CONIC_RECT 2

/* Per-Gaussian render record written by preprocess and read by the render
 * kernels: 12 floats = 48 bytes, three float4:
 *   [0..3]  x, y, conic_a, conic_b
 *   [4..7]  conic_c, opacity, depth, clamped bits (uint32 bit c = channel c)
 *   [8..11] r, g, b, 0
 * Per-Gaussian render-gradient accumulator (filled by gsb_render_bwd):
 * 12 floats = 48 bytes:
 *   [0..3]  dL/dx, dL/dy, dL/ddepth, 0
 *   [4..7]  dL/dconic_a, dL/dconic_b, dL/dconic_c, dL/dopacity
 *   [8..11] dL/dr, dL/dg, dL/db, 0                                         */
#define GSB_RECORD_FLOATS 12
#define GSB_GRAD_FLOATS 12

int gsb_abi_version(void);
const char* gsb_last_error(void);

/* Threads per CTA that the library launches for a kernel class (0 for an
 * unknown name).  Stands in for get_tuned_block_dim (gswarp/_tuning.py:342):
 * the sm_100a launch shapes are fixed at compile time, and this reports the
 * shapes actually launched.  Classes: preprocess, preprocess_sh16,
 * sh_colors_views, binning_scan, binning_emit, radix_sort, render_forward,
 * render_backward (grids of 6,000 tiles and more), render_backward_small_grid,
 * backward_preprocess, backward_preprocess_sh16, sh_backward_views, ssim_fwd, ssim_bwd (and the reference's ssim_fwd_h,
 * ssim_fwd_v, ssim_bwd_h, ssim_bwd_v), knn_morton, knn_gather,
 * knn_box_minmax, knn_box_dist, knn_search, adam. */
int gsb_block_dim(const char* kernel_class);

/* Measurement microkernels (no counterpart in the reference; used by the
 * benchmark for the compute roofline of the render kernels).  gsb_peak_fp32
 * runs packed f32x2 fused multiply-adds, gsb_peak_ex2 MUFU ex2.approx, in
 * `blocks` CTAs of independent chains for `iters` iterations; `out` (blocks
 * floats) only keeps the results live.  gsb_peak_work returns one launch's
 * FLOP (which = 0) or ex2 evaluations (which = 1). */
int gsb_peak_fp32(int blocks, int iters, float* out, void* stream);
int gsb_peak_ex2(int blocks, int iters, float* out, void* stream);
long long gsb_peak_work(int which, int blocks, int iters);

/* ------------------------------------------------------------------------ */
/* Preprocess forward.  Replaces preprocess_gaussians                        */
/* (gswarp/_internal/backends/warp/preprocess_ops.py:289-581): the fused     */
/* projection/cov3d/EWA cov2d/conic/radius/AccuTile kernel                  */
/* (preprocess_kernels.py:83-269), its cov3D_precomp variant (:345-476,     */
/* :630-672) and the SH colour kernel (:272-342).                            */
/* ------------------------------------------------------------------------ */
typedef struct {
  int P, W, H;
  const float* means;          /* (P,3) */
  const float* scales;         /* (P,3) or NULL when cov3d_precomp is given */
  const float* rotations;      /* (P,4) or NULL */
  const float* cov3d_precomp;  /* (P,6) or NULL */
  float scale_modifier;
  const float* opacities;      /* (P) */
  const float* viewmatrix;     /* 16 floats, device */
  const float* projmatrix;     /* 16 floats, device */
  const float* campos;         /* 3 floats, device */
  float tanfovx, tanfovy, focal_x, focal_y;
  const float* sh;             /* (P,K,3) or NULL */
  int sh_degree, sh_coeffs;    /* degree and K */
  const float* colors_precomp; /* (P,3) or NULL (exactly one of sh/colors) */
  int coverage_mode;           /* GSB_COVERAGE_* */
  /* outputs (all (P,...) device arrays) */
  int* radii;
  float* proj_2d;       /* (P,2), or NULL (not written) */
  float* conic_2d;      /* (P,3), or NULL (not written) */
  float* conic_2d_inv;  /* (P,3), or NULL (not written; the binning emit needs it
                           unless bin_records are used) */
  float* depths;        /* (P) */
  int* tiles_touched;   /* (P) */
  float* records;       /* (P,12) render records */
  float* cov3d_out;     /* (P,6) 3D covariance of the scale/rotation path, or NULL
                           (only the packed raw-compat geometry buffer needs it) */
  float* bin_records;   /* (P,8) 16-byte aligned, or NULL: per Gaussian with tiles, a
                           32-byte record of its covered tiles (clipped rect plus the
                           AccuTile interval of each band, or the conic_rect tile mask),
                           written while counting so the binning emit only replays it
                           (written only where tiles_touched > 0; needs both tile-grid
                           dimensions below 65536) */
  int sparse_records;   /* 1: write render records only where radius > 0 (nothing reads
                           the others: render and the id-list backward skip them) */
  int colors_clamp_signed; /* 1: colors_precomp holds SH colours from gsb_sh_colors_views:
                           a channel stored as -0.0 was clamped at zero (its record clamp
                           bit is set and its colour is +0.0), so the records equal those
                           of the SH path bit for bit */
} gsb_preprocess_args;

int gsb_preprocess_fwd(const gsb_preprocess_args* a, void* stream);

/* markVisible (preprocess_ops.py:584-595 / preprocess_kernels.py:603-627). */
int gsb_mark_visible(int P, const float* means, const float* viewmatrix, uint8_t* out,
                     void* stream);

/* ------------------------------------------------------------------------ */
/* Binning.  Replaces _build_binning_state (binning_ops.py:84-431) with two  */
/* calls separated by one host read of the pair count.                       */
/* gsb_bin_count: order-preserving compaction of the V Gaussians with      */
/* tiles, stable sort of them by depth float bits (ties by index), depth-   */
/* ordered inclusive scan of tiles_touched (binning_ops.py:152-224).        */
/* status_out[0] = int64 pair total, [1] = device error word, [2] = V.       */
/* ------------------------------------------------------------------------ */
typedef struct {
  int P;
  const float* depths;        /* (P) */
  const int* radii;           /* (P) */
  const int* tiles_touched;   /* (P) */
  int* depth_order;           /* out (P): first V entries = ids with tiles, in depth order */
  int* point_offsets;         /* out (P): first V entries = inclusive scan in depth order */
  int* binned_ids;            /* optional out (P): first V entries = ids with tiles, ascending */
  long long* status_out;      /* out, device, 3 words: [0]=pair total, [1]=error word, [2]=V */
  void* workspace;
  size_t workspace_bytes;
} gsb_bin_count_args;

size_t gsb_bin_count_workspace_bytes(int P);
int gsb_bin_count(const gsb_bin_count_args* a, void* stream);

/* gsb_bin_emit_sort: emit (tile id, point id) pairs in depth order with the  */
/* same AccuTile sweep as the count (binning_kernels.py:126-216,410-451),   */
/* stable radix sort by tile id (memory.py:571-600 semantics), identify     */
/* ranges (binning_kernels.py:467-487).  Result order: ascending (tile,     */
/* depth bits, point id).  ranges is zero-filled here first.                */
typedef struct {
  int P, W, H;
  long long num_rendered;
  int coverage_mode;
  const int* depth_order;      /* from gsb_bin_count */
  const int* point_offsets;    /* from gsb_bin_count */
  const int* radii;
  const float* records;        /* (P,12) */
  const float* conic_2d_inv;   /* (P,3) */
  const int* tiles_touched;
  int* point_list;             /* out (num_rendered) */
  int* ranges;                 /* out (tiles,2) */
  long long* error_word;       /* device word; OR-ed with error bits */
  void* workspace;
  size_t workspace_bytes;
  const float* bin_records;    /* (P,8) from gsb_preprocess_fwd, or NULL: with it the emit
                                  reads one 32-byte record per Gaussian (radii, conic_2d_inv
                                  and tiles_touched are then not read; records only for
                                  footprints of more than 5 tile bands) */
  const long long* bin_status; /* status_out of gsb_bin_count (device; V is read from [2]) */
} gsb_bin_sort_args;

size_t gsb_bin_sort_workspace_bytes(long long num_rendered, int W, int H);
int gsb_bin_emit_sort(const gsb_bin_sort_args* a, void* stream);

/* ------------------------------------------------------------------------ */
/* Render forward.  Replaces _render_tiles_warp (render_ops.py:16-93) /     */
/* _render_tiles_tiled256_warp_kernel (render_kernels.py:15-147).           */
/* ------------------------------------------------------------------------ */
typedef struct {
  int W, H;
  int compute_depth;
  const int* ranges;
  const int* point_list;
  const float* records;
  const float* background;  /* 3 floats, device */
  float* out_color;         /* (3,H,W) */
  float* out_depth;         /* (1,H,W) */
  float* out_alpha;         /* (1,H,W) */
  int* n_contrib;           /* (H*W) */
  int top_k;                /* > 0: flow render auxiliary outputs (flow_kernels.py:14-180): */
  int* gs_per_pixel;        /*   (K,H,W) ids of the first K contributors, -1 where none */
  float* weight_per_gs_pixel; /* (K,H,W) their compositing weights alpha * T */
  float* x_mu;              /*   (2,K,H,W) offsets centre - pixel (dx planes, then dy) */
  float* aux_scratch;       /* optional (K,H,W,4) floats, 16-byte aligned: the render writes each
                               slot as one 16-byte (id, weight, dx, dy) record here, and a second
                               kernel splits the records into the three outputs with coalesced
                               stores (a quarter of the store transactions of writing the
                               outputs directly); NULL: the outputs are written directly */
} gsb_render_fwd_args;

int gsb_render_fwd(const gsb_render_fwd_args* a, void* stream);

/* Render backward.  Replaces _backward_render_tiles_warp                    */
/* (backward_ops.py:183-290) / _backward_render_tiles_warp32_kernel         */
/* (backward_kernels.py:538-707).  grad_acc must be zero-filled (P,12).     */
typedef struct {
  int W, H, P;
  int compute_depth;
  const int* ranges;
  const int* point_list;
  const float* records;
  const float* background;
  const float* out_alpha;
  const int* n_contrib;
  const float* grad_color;  /* (3,H,W) */
  const float* grad_depth;  /* (1,H,W) or NULL (zero gradient) */
  const float* grad_alpha;  /* (1,H,W) or NULL (zero gradient) */
  float* grad_acc;          /* (P,12), accumulated with atomics */
} gsb_render_bwd_args;

int gsb_render_bwd(const gsb_render_bwd_args* a, void* stream);

/* ------------------------------------------------------------------------ */
/* Preprocess + SH backward.  Replaces the tail of                           */
/* _rasterize_gaussians_backward_python (backward_ops.py:525-744): the SH   */
/* backward (backward_kernels.py:297-536), the fused preprocess backward    */
/* (:52-295) and the cov3D_precomp kernels (:709-949).                       */
/* ------------------------------------------------------------------------ */
typedef struct {
  int P, W, H;
  const float* means;
  const int* radii;
  const float* scales;         /* or NULL */
  const float* rotations;      /* or NULL */
  const float* cov3d_precomp;  /* or NULL */
  float scale_modifier;
  const float* viewmatrix;
  const float* projmatrix;
  const float* campos;
  float tanfovx, tanfovy, focal_x, focal_y;
  const float* sh;             /* (P,K,3) or NULL */
  int sh_degree, sh_coeffs;
  const float* records;        /* forward records (clamped bits) */
  const float* grad_acc;       /* (P,12) from gsb_render_bwd */
  const float* grad_proj_2d;   /* (P,2) user gradient of proj_2D, or NULL (zero) */
  const float* grad_conic_2d;  /* (P,3) or NULL */
  const float* grad_conic_2d_inv; /* (P,3) or NULL */
  int accumulate;              /* 1: add into the outputs instead of storing */
  /* outputs (NULL where not applicable) */
  float* grad_means3d;   /* (P,3) */
  float* grad_means2d;   /* (P,3) */
  float* grad_scales;    /* (P,3) */
  float* grad_rotations; /* (P,4) */
  float* grad_opacity;   /* (P) */
  float* grad_sh;        /* (P,K,3) */
  float* grad_colors;    /* (P,3) colors_precomp gradient */
  float* grad_cov3d;     /* (P,6) cov3D_precomp gradient */
  const int* ids;        /* optional (accumulate mode only): process just these Gaussians,
                            e.g. the binned_ids of gsb_bin_count (the others get no
                            render gradient and are left untouched); NULL = all P */
  int num_ids;
  int clear_grad_acc;    /* 1: zero each processed Gaussian's grad_acc entry after reading it,
                            so a persistent accumulator is ready for the next view without a
                            full memset (the render backward only touches binned Gaussians) */
  float* densify_grad_accum; /* optional (P): += |d loss / d means2D (x, y)| per processed
                            Gaussian (3DGS add_densification_stats' gradient norm) */
  int grad_colors_clamped; /* 1: grad_colors receives the colour gradient through the
                            forward's clamp (0 for the channels whose record clamp bit is
                            set): the input gsb_sh_backward_views takes */
} gsb_preprocess_bwd_args;

int gsb_preprocess_bwd(const gsb_preprocess_bwd_args* a, void* stream);

/* ------------------------------------------------------------------------ */
/* SH colour over several views (B200 addition for multi-view steps).       */
/* Every view of a data-parallel step renders the same Gaussians, so the   */
/* SH rows (up to 192 B per Gaussian) are read once per step instead of    */
/* once per view in the forward and three times per view in the backward:  */
/* gsb_sh_colors_views writes each view's clamped SH colour                 */
/* (preprocess_kernels.py:272-342; fed to gsb_preprocess_fwd with           */
/* colors_clamp_signed), and gsb_sh_backward_views turns the views' colour */
/* gradients (gsb_preprocess_bwd with grad_colors_clamped) into the SH      */
/* gradient and the view-direction term of the means gradient              */
/* (backward_kernels.py:297-536), summed over the views in view order.      */
/* ------------------------------------------------------------------------ */
typedef struct {
  int P, num_views;
  int sh_degree, sh_coeffs;    /* degree and K (1..16) */
  const float* means;          /* (P,3) */
  const float* sh;             /* (P,K,3) */
  const float* campos;         /* (num_views,3), device */
  /* gsb_sh_colors_views */
  float* colors;               /* out (num_views,P,3): max(SH colour + 0.5, 0) of every
                                  Gaussian from each camera; clamped channels are -0.0 */
  /* gsb_sh_backward_views */
  float* grad_colors;          /* (num_views,P,3) clamped colour gradients; entries that are
                                  not zero are reset to zero after reading when
                                  clear_grad_colors is set */
  int clear_grad_colors;
  float* grad_sh;              /* out (P,K,3): stored (every row, zero where no view
                                  contributes), or added to when accumulate is set */
  float* grad_means3d;         /* (P,3): the direction term is added */
  int accumulate;
  int begin, end;              /* gsb_sh_backward_views: the Gaussians [begin, end) only
                                  (0, 0 = all P), so a caller can start reducing one range
                                  across GPUs while the next is computed */
} gsb_sh_views_args;

int gsb_sh_colors_views(const gsb_sh_views_args* a, void* stream);
int gsb_sh_backward_views(const gsb_sh_views_args* a, void* stream);

/* ------------------------------------------------------------------------ */
/* Fused SSIM.  Replaces FusedSSIMMap (gswarp/fused_ssim.py:1074-1150) and   */
/* its four separable kernels (:461-638, :831-1067).                         */
/* ------------------------------------------------------------------------ */
typedef struct {
  int B, C, H, W;
  int valid;              /* 0: 'same' padding, 1: 'valid' */
  float C1, C2;
  const float* img1;
  const float* img2;
  float* dm;              /* (3,B,C,H,W) workspace kept for backward, or NULL (inference) */
  float* partials;        /* gsb_ssim_partials_count() floats, workspace */
  float* loss;            /* 1 float out: mean SSIM */
} gsb_ssim_fwd_args;

int gsb_ssim_partials_count(int B, int C, int H, int W);
int gsb_ssim_fwd(const gsb_ssim_fwd_args* a, void* stream);

typedef struct {
  int B, C, H, W;
  int valid;
  const float* img1;
  const float* img2;
  const float* dm;        /* from gsb_ssim_fwd */
  const float* upstream;  /* 1 float, device: dL/dloss */
  float* grad_img1;       /* (B,C,H,W) */
} gsb_ssim_bwd_args;

int gsb_ssim_bwd(const gsb_ssim_bwd_args* a, void* stream);

/* Photometric training loss (B200 addition; the reference composes it in
 * Python from an L1 term and its fused SSIM, docs/ssim.md:22,91):
 *   L = w_l1 * mean|img - target| + w_ssim * (1 - SSIM(img, target)),
 * 'same' padding, 11x11 Gaussian window.  Forward writes loss_out[0] = L,
 * loss_out[1] = mean L1, loss_out[2] = mean SSIM, and the dm maps backward
 * needs; backward writes upstream * dL/dimg. */
typedef struct {
  int B, C, H, W;
  float C1, C2;
  float w_l1, w_ssim;
  const float* img;       /* (B,C,H,W) rendered */
  const float* target;    /* (B,C,H,W) */
  float* dm;              /* (3,B,C,H,W) workspace kept for backward */
  float* partials;        /* 2 * gsb_ssim_partials_count() floats, workspace */
  float* loss_out;        /* 3 floats out (device) */
} gsb_photo_loss_fwd_args;

int gsb_photo_loss_fwd(const gsb_photo_loss_fwd_args* a, void* stream);

typedef struct {
  int B, C, H, W;
  float w_l1, w_ssim;
  float upstream;         /* dTotal/dL, host scalar (1 for a plain training step) */
  const float* img;
  const float* target;
  const float* dm;        /* from gsb_photo_loss_fwd */
  float* grad_img;        /* (B,C,H,W) */
} gsb_photo_loss_bwd_args;

int gsb_photo_loss_bwd(const gsb_photo_loss_bwd_args* a, void* stream);

/* Allocation-free SSIM forward.  No counterpart in the reference: it exists
 * for callers that cannot provide device memory (a process whose device
 * memory is reserved up front by another allocator, a plain C/FFI caller
 * without a device allocator, or a loop that cannot afford a cudaMalloc /
 * cudaFree round trip).  Same result as gsb_ssim_fwd (mean SSIM into *loss,
 * dm maps if dm is non-NULL), but its scratch is a fixed 256 KiB device array
 * inside the library, so B*C*ceil(H/40)*ceil(W/32) must not exceed
 * GSB_SSIM_NOALLOC_MAX_PARTIALS (larger inputs return GSB_ERR_INVALID).
 * All calls on a device share that array: calls whose kernels overlap on the
 * GPU race.  The first call on a device looks up the array's address (again
 * after the device's context is replaced, e.g. by cudaDeviceReset); make it
 * before any stream capture begins. */
#define GSB_SSIM_NOALLOC_MAX_PARTIALS 65536
int gsb_ssim_fwd_noalloc(int B, int C, int H, int W, int valid, float C1, float C2,
                         const float* img1, const float* img2, float* dm, float* loss,
                         void* stream);

/* ------------------------------------------------------------------------ */
/* Optimizer step after the training step's gradient all-reduce (B200       */
/* addition; the reference leaves the optimizer to the training script).    */
/* Fused Adam over the flat gradient buffer [means 3P | scales 3P |         */
/* rotations 4P | opacities P | SH 3KP] with torch.optim.Adam's arithmetic  */
/* (weight_decay 0, no amsgrad) and the six 3DGS learning-rate groups.      */
/* ------------------------------------------------------------------------ */
typedef struct {
  int P, sh_coeffs;
  float* params[5];       /* means (P,3), scales (P,3), rotations (P,4), opacities (P), sh (P,K,3) */
  const float* grad;      /* flat, 11P + 3KP floats */
  float* exp_avg;         /* flat, same layout */
  float* exp_avg_sq;      /* flat, same layout */
  double lr[6];           /* means, scales, rotations, opacities, SH DC (coefficient 0), SH rest */
  double beta1, beta2, eps;
  int step;               /* this update's step number, >= 1 (bias corrections) */
} gsb_adam_args;

int gsb_adam_step(const gsb_adam_args* a, void* stream);

/* Densification statistics: for radius > 0, denom += 1 and
 * max_radii = max(max_radii, radius) (3DGS add_densification_stats /
 * max_radii2D); the gradient-norm sum comes from gsb_preprocess_bwd. */
int gsb_densify_stats(int P, const int* radii, float* denom, float* max_radii, void* stream);

/* ------------------------------------------------------------------------ */
/* KNN initialiser.  Replaces distCUDA2 (gswarp/knn.py:264-410).             */
/* out[i] = mean squared distance of point i to its three nearest others.   */
/* ------------------------------------------------------------------------ */
typedef struct {
  int P;                 /* >= 4 */
  const float* points;   /* (P,3) */
  float* out;            /* (P) */
  long long* error_word; /* device word */
  void* workspace;
  size_t workspace_bytes;
} gsb_knn_args;

size_t gsb_knn_workspace_bytes(int P);
int gsb_knn(const gsb_knn_args* a, void* stream);

/* Correctly rounded binary32 log of every input (the AccuTile threshold   */
/* primitive); exported so tests can pin device and host bit for bit.       */
int gsb_selftest_threshold_log(const float* in, float* out, long long n, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GSB200_H */
