// render.cu -- 16x16-tile front-to-back alpha blending and its backward.
//
// Forward restates _render_tiles_tiled256_warp_kernel
// (render_kernels.py:15-147): integer pixel coordinates, 256-Gaussian rounds
// with a CTA-wide done vote, alpha = min(0.99, op*exp(power)), skip below
// 1/255, stop (without adding the pair) once T*(1-alpha) < 1e-4.
// Backward restates _backward_render_tiles_warp32_kernel
// (backward_kernels.py:538-707): per-pixel back-to-front recurrence from
// n_contrib with T_final = 1 - alpha, 3DGS accum_rec / last_alpha /
// last_color (and depth) terms, gradients of xy (scaled by W/2, H/2), conic,
// opacity, colour and depth.
//
// B200 design (both directions): one 256-thread CTA per tile; each warp owns
// an 8x4 pixel block (squarer than the reference's 16x2 rows, so a small
// Gaussian touches fewer warps); Gaussians are staged per batch in shared
// memory from the 48-byte render records (three 16-byte loads per Gaussian);
// exp is one MUFU.EX2.  Backward: the CTA walks its list from the CTA-wide
// maximum contributor down, each warp skips positions above its own maximum,
// a warp vote skips Gaussians no lane of the warp uses, and the ten gradient
// terms are reduced across the warp with a 12-shuffle transpose reduction
// (instead of 10 x 5 butterfly shuffles); 10 lanes then issue one float
// atomic each into the per-Gaussian accumulator.
#include "gsb_common.cuh"

namespace gsb {
namespace {

constexpr int THREADS = 256;
constexpr int FWD_BATCH = 256;
constexpr int BWD_BATCH = 128;
constexpr unsigned FULL = 0xffffffffu;

__device__ __forceinline__ void pixel_of(int tile, int gx, int& px, int& py) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tx = tile % gx, ty = tile / gx;
  px = tx * BLOCK_X + (warp & 1) * 8 + (lane & 7);
  py = ty * BLOCK_Y + (warp >> 1) * 4 + (lane >> 3);
}

template <bool DEPTH>
__global__ void __launch_bounds__(THREADS) render_fwd_kernel(const gsb_render_fwd_args a, int gx) {
  __shared__ float2 s_xy[FWD_BATCH];
  __shared__ float4 s_cop[FWD_BATCH];   // conic a, b, c, opacity
  __shared__ float4 s_rgbd[FWD_BATCH];  // r, g, b, depth
  const int tile = blockIdx.x;
  int pxi, pyi;
  pixel_of(tile, gx, pxi, pyi);
  const bool inside = pxi < a.W && pyi < a.H;
  const int2 range = reinterpret_cast<const int2*>(a.ranges)[tile];
  const float4* rec = reinterpret_cast<const float4*>(a.records);
  const float fx = (float)pxi, fy = (float)pyi;

  float T = 1.0f, c0 = 0.0f, c1 = 0.0f, c2 = 0.0f, wsum = 0.0f, dacc = 0.0f;
  int last = 0;
  bool done = !inside;
  for (int b = range.x; b < range.y; b += FWD_BATCH) {
    if (__syncthreads_count(done) == THREADS) break;
    const int i = b + threadIdx.x;
    if (i < range.y) {
      const int id = a.point_list[i];
      const float4 q0 = __ldg(rec + (size_t)id * 3 + 0);
      const float4 q1 = __ldg(rec + (size_t)id * 3 + 1);
      const float4 q2 = __ldg(rec + (size_t)id * 3 + 2);
      s_xy[threadIdx.x] = make_float2(q0.x, q0.y);
      s_cop[threadIdx.x] = make_float4(q0.z, q0.w, q1.x, q1.y);
      s_rgbd[threadIdx.x] = make_float4(q2.x, q2.y, q2.z, q1.z);
    }
    __syncthreads();
    const int cnt = min(FWD_BATCH, range.y - b);
    if (!done) {
      for (int j = 0; j < cnt; ++j) {
        const float2 xy = s_xy[j];
        const float4 co = s_cop[j];
        const float dx = xy.x - fx, dy = xy.y - fy;
        const float power = -0.5f * (co.x * dx * dx + co.z * dy * dy) - co.y * dx * dy;
        if (power > 0.0f) continue;
        const float alpha = fminf(0.99f, co.w * fast_exp(power));
        if (alpha < (1.0f / 255.0f)) continue;
        const float test_T = T * (1.0f - alpha);
        if (test_T < 0.0001f) {
          done = true;
          break;
        }
        const float contrib = alpha * T;
        const float4 cd = s_rgbd[j];
        c0 += cd.x * contrib;
        c1 += cd.y * contrib;
        c2 += cd.z * contrib;
        wsum += contrib;
        if (DEPTH) dacc += cd.w * contrib;
        T = test_T;
        last = b - range.x + j + 1;
      }
    }
  }
  if (inside) {
    const long long npix = (long long)a.W * a.H;
    const long long pix = (long long)pyi * a.W + pxi;
    a.n_contrib[pix] = last;
    a.out_color[pix] = c0 + T * a.background[0];
    a.out_color[npix + pix] = c1 + T * a.background[1];
    a.out_color[2 * npix + pix] = c2 + T * a.background[2];
    a.out_alpha[pix] = wsum;
    a.out_depth[pix] = dacc;
  }
}

// Transpose reduction of ten per-lane values over a warp (12 shuffles).
// On return, lane pairs (2k, 2k+1) hold the warp total of one value; the
// returned index is that value's index (0..9) or -1 for lanes without one.
__device__ __forceinline__ int warp_reduce10(const float (&v)[10], float& out) {
  const int lane = threadIdx.x & 31;
  const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4, b1 = lane & 2;
  float a5[5];
#pragma unroll
  for (int k = 0; k < 5; ++k) {
    const float send = b4 ? v[k] : v[5 + k];
    const float keep = b4 ? v[5 + k] : v[k];
    a5[k] = keep + __shfl_xor_sync(FULL, send, 16);
  }
  float c[3];
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const float hiv = (k + 3 < 5) ? a5[(k + 3) % 5] : 0.0f;
    const float send = b3 ? a5[k] : hiv;
    const float keep = b3 ? hiv : a5[k];
    c[k] = keep + __shfl_xor_sync(FULL, send, 8);
  }
  float d0, d1;
  {
    const float send0 = b2 ? c[0] : c[2];
    const float keep0 = b2 ? c[2] : c[0];
    d0 = keep0 + __shfl_xor_sync(FULL, send0, 4);
    const float send1 = b2 ? c[1] : 0.0f;
    const float keep1 = b2 ? 0.0f : c[1];
    d1 = keep1 + __shfl_xor_sync(FULL, send1, 4);
  }
  float e;
  {
    const float send = b1 ? d0 : d1;
    const float keep = b1 ? d1 : d0;
    e = keep + __shfl_xor_sync(FULL, send, 2);
  }
  e += __shfl_xor_sync(FULL, e, 1);
  out = e;
  int off;
  if (!b3)
    off = b2 ? (b1 ? -1 : 2) : (b1 ? 1 : 0);
  else
    off = b2 ? -1 : (b1 ? 4 : 3);
  return off < 0 ? -1 : (b4 ? 5 : 0) + off;
}

template <bool DEPTH>
__global__ void __launch_bounds__(THREADS) render_bwd_kernel(const gsb_render_bwd_args a, int gx) {
  __shared__ int s_id[BWD_BATCH];
  __shared__ float2 s_xy[BWD_BATCH];
  __shared__ float4 s_cop[BWD_BATCH];
  __shared__ float4 s_rgbd[BWD_BATCH];
  __shared__ int s_max[THREADS / 32];
  const int tile = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int pxi, pyi;
  pixel_of(tile, gx, pxi, pyi);
  const bool inside = pxi < a.W && pyi < a.H;
  const int2 range = reinterpret_cast<const int2*>(a.ranges)[tile];
  const int n = range.y - range.x;
  const float4* rec = reinterpret_cast<const float4*>(a.records);

  const long long npix = (long long)a.W * a.H;
  const long long pix = (long long)pyi * a.W + pxi;
  int lc = 0;
  float T_final = 0.0f, g0 = 0.0f, g1 = 0.0f, g2 = 0.0f, gd = 0.0f, ga = 0.0f, bg_dot = 0.0f;
  if (inside && n > 0) {
    lc = a.n_contrib[pix];
    T_final = 1.0f - a.out_alpha[pix];
    g0 = a.grad_color[pix];
    g1 = a.grad_color[npix + pix];
    g2 = a.grad_color[2 * npix + pix];
    if (DEPTH) gd = a.grad_depth[pix];
    ga = a.grad_alpha[pix];
    bg_dot = a.background[0] * g0 + a.background[1] * g1 + a.background[2] * g2;
  }
  const int warp_max = __reduce_max_sync(FULL, lc);
  if (lane == 0) s_max[warp] = warp_max;
  __syncthreads();
  int cta_max = 0;
#pragma unroll
  for (int w = 0; w < THREADS / 32; ++w) cta_max = max(cta_max, s_max[w]);
  cta_max = min(cta_max, n);  // n_contrib never exceeds the tile's list
  if (cta_max <= 0) return;

  const float ddelx_dx = 0.5f * (float)a.W;
  const float ddely_dy = 0.5f * (float)a.H;
  const float fx = (float)pxi, fy = (float)pyi;
  float T = T_final;
  float ar0 = 0.0f, ar1 = 0.0f, ar2 = 0.0f, adr = 0.0f, aar = 0.0f;
  float la = 0.0f, lc0 = 0.0f, lc1 = 0.0f, lc2 = 0.0f, ld = 0.0f;

  for (int hi = cta_max; hi > 0; hi -= BWD_BATCH) {
    const int lo = max(0, hi - BWD_BATCH);
    __syncthreads();
    for (int k = threadIdx.x; k < hi - lo; k += THREADS) {
      const int id = a.point_list[range.x + lo + k];
      const float4 q0 = __ldg(rec + (size_t)id * 3 + 0);
      const float4 q1 = __ldg(rec + (size_t)id * 3 + 1);
      const float4 q2 = __ldg(rec + (size_t)id * 3 + 2);
      s_id[k] = id;
      s_xy[k] = make_float2(q0.x, q0.y);
      s_cop[k] = make_float4(q0.z, q0.w, q1.x, q1.y);
      s_rgbd[k] = make_float4(q2.x, q2.y, q2.z, q1.z);
    }
    __syncthreads();
    const int top = min(hi, warp_max);
    for (int pos = top - 1; pos >= lo; --pos) {
      const int j = pos - lo;
      float v[10];
#pragma unroll
      for (int k = 0; k < 10; ++k) v[k] = 0.0f;
      bool contrib = false;
      if (pos < lc) {
        const float2 xy = s_xy[j];
        const float4 co = s_cop[j];
        const float dx = xy.x - fx, dy = xy.y - fy;
        const float power = -0.5f * (co.x * dx * dx + co.z * dy * dy) - co.y * dx * dy;
        if (power <= 0.0f) {
          const float G = fast_exp(power);
          const float alpha = fminf(0.99f, co.w * G);
          if (alpha >= (1.0f / 255.0f)) {
            contrib = true;
            const float oma = fmaxf(1.0f - alpha, 1.0e-5f);
            const float inv_oma = __frcp_rn(oma);
            T = T * inv_oma;
            const float dchannel = alpha * T;
            const float4 cd = s_rgbd[j];
            ar0 = la * lc0 + (1.0f - la) * ar0;
            ar1 = la * lc1 + (1.0f - la) * ar1;
            ar2 = la * lc2 + (1.0f - la) * ar2;
            lc0 = cd.x;
            lc1 = cd.y;
            lc2 = cd.z;
            float dL_dopa = (cd.x - ar0) * g0 + (cd.y - ar1) * g1 + (cd.z - ar2) * g2;
            v[7] = dchannel * g0;
            v[8] = dchannel * g1;
            v[9] = dchannel * g2;
            if (DEPTH) {
              adr = la * ld + (1.0f - la) * adr;
              ld = cd.w;
              dL_dopa += (cd.w - adr) * gd;
              v[2] = dchannel * gd;
            }
            aar = la + (1.0f - la) * aar;
            dL_dopa += (1.0f - aar) * ga;
            dL_dopa *= T;
            la = alpha;
            dL_dopa += (-T_final * inv_oma) * bg_dot;
            const float dL_dG = co.w * dL_dopa;
            const float gdx = G * dx, gdy = G * dy;
            const float dG_ddelx = -gdx * co.x - gdy * co.y;
            const float dG_ddely = -gdy * co.z - gdx * co.y;
            v[0] = dL_dG * dG_ddelx * ddelx_dx;
            v[1] = dL_dG * dG_ddely * ddely_dy;
            v[3] = -0.5f * gdx * dx * dL_dG;
            v[4] = -0.5f * gdx * dy * dL_dG;
            v[5] = -0.5f * gdy * dy * dL_dG;
            v[6] = G * dL_dopa;
          }
        }
      }
      if (__any_sync(FULL, contrib)) {
        float sum;
        const int slot = warp_reduce10(v, sum);
        if (!(lane & 1) && slot >= 0) {
          const int off = slot < 3 ? slot : slot + 1;
          atomicAdd(a.grad_acc + (size_t)s_id[j] * GSB_GRAD_FLOATS + off, sum);
        }
      }
    }
  }
}

}  // namespace
}  // namespace gsb

using namespace gsb;

GSB_EXPORT int gsb_render_fwd(const gsb_render_fwd_args* a, void* stream) {
  if (!a || a->W <= 0 || a->H <= 0 || !a->ranges || !a->records || !a->background ||
      !a->out_color || !a->out_depth || !a->out_alpha || !a->n_contrib) {
    set_error("gsb_render_fwd: invalid arguments");
    return GSB_ERR_INVALID;
  }
  const int gx = div_up(a->W, BLOCK_X), gy = div_up(a->H, BLOCK_Y);
  cudaStream_t s = (cudaStream_t)stream;
  if (a->compute_depth)
    render_fwd_kernel<true><<<gx * gy, THREADS, 0, s>>>(*a, gx);
  else
    render_fwd_kernel<false><<<gx * gy, THREADS, 0, s>>>(*a, gx);
  return check_launch("render_fwd_kernel");
}

GSB_EXPORT int gsb_render_bwd(const gsb_render_bwd_args* a, void* stream) {
  if (!a || a->W <= 0 || a->H <= 0 || a->P < 0 || !a->ranges || !a->records ||
      !a->background || !a->out_alpha || !a->n_contrib || !a->grad_color || !a->grad_alpha ||
      (a->compute_depth && !a->grad_depth) || !a->grad_acc) {
    set_error("gsb_render_bwd: invalid arguments");
    return GSB_ERR_INVALID;
  }
  if (a->P == 0) return GSB_OK;
  const int gx = div_up(a->W, BLOCK_X), gy = div_up(a->H, BLOCK_Y);
  cudaStream_t s = (cudaStream_t)stream;
  if (a->compute_depth)
    render_bwd_kernel<true><<<gx * gy, THREADS, 0, s>>>(*a, gx);
  else
    render_bwd_kernel<false><<<gx * gy, THREADS, 0, s>>>(*a, gx);
  return check_launch("render_bwd_kernel");
}
