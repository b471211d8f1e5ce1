// render.cu -- 16x16-tile front-to-back alpha blending and its backward.
//
// Forward restates _render_tiles_tiled256_warp_kernel
// (render_kernels.py:15-147): integer pixel coordinates, Gaussian rounds
// with a CTA-wide done vote, alpha = min(0.99, op*exp(power)), skip below
// 1/255, stop (without adding the pair) once T*(1-alpha) < 1e-4.
// Backward restates _backward_render_tiles_warp32_kernel
// (backward_kernels.py:538-707): per-pixel back-to-front recurrence from
// n_contrib with T_final = 1 - alpha, 3DGS accum_rec / last_alpha /
// last_color (and depth) terms, gradients of xy (scaled by W/2, H/2), conic,
// opacity, colour and depth.
//
// B200 design (both directions): one 128-thread CTA per 16x16 tile; each
// thread owns TWO pixels (rows y and y+4 of its warp's 8x8 block), so every
// Gaussian staged in shared memory is read once per two pixels and the
// per-(warp, Gaussian) control work covers 64 pixels.  Gaussians are staged
// per batch from the 48-byte render records (three 16-byte loads per
// Gaussian); exp is one MUFU.EX2, 1/(1-alpha) one MUFU.RCP.  Backward: the
// CTA walks its list from the CTA-wide maximum contributor down, each warp
// skips positions above its own maximum, a warp vote skips Gaussians no lane
// uses, and the ten gradient terms (already summed over the thread's two
// pixels) are reduced across the warp with a 12-shuffle transpose reduction
// (instead of 10 x 5 butterfly shuffles); 10 lanes then issue one float atomic
// each into the per-Gaussian accumulator.
#include "gsb_common.cuh"

namespace gsb {
namespace {

constexpr int THREADS = 128;
constexpr int BATCH = 128;
constexpr unsigned FULL = 0xffffffffu;

// Pixel coordinates of the thread's two pixels.
__device__ __forceinline__ void pixels_of(int tile, int gx, int& px, int& py0) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tx = tile % gx, ty = tile / gx;
  px = tx * BLOCK_X + (warp & 1) * 8 + (lane & 7);
  py0 = ty * BLOCK_Y + (warp >> 1) * 8 + (lane >> 3);
}

__device__ __forceinline__ float fast_rcp(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Conservative screen box of the pixels where this Gaussian can reach
// alpha >= 1/255: op*exp(-q/2) >= 1/255  <=>  q = d^T conic d <= t with
// t = 2 ln(255 op); the ellipse {q <= t} has half-extents sqrt(t*cov_xx),
// sqrt(t*cov_yy) (cov = conic^-1).  Widened by 1% + 0.5 px so rounding in
// the per-pixel test can never reach outside it.  A conic that is not
// positive definite gets an unbounded box (never culled); t <= 0 (opacity
// below 1/255) an empty one.
__device__ __forceinline__ float4 alpha_box(float x, float y, float a, float b, float c, float op) {
  const float det = a * c - b * b;
  const float inf = __int_as_float(0x7f800000);
  if (!(a > 0.0f) || !(det > 0.0f)) return make_float4(-inf, inf, -inf, inf);
  const float t = 2.0f * __logf(255.0f * op);
  if (!(t > 0.0f)) return make_float4(inf, -inf, inf, -inf);
  const float inv = 1.0f / det;
  const float ex = sqrtf(t * c * inv) * 1.01f + 0.5f;
  const float ey = sqrtf(t * a * inv) * 1.01f + 0.5f;
  return make_float4(x - ex, x + ex, y - ey, y + ey);
}

__device__ __forceinline__ bool box_hits(const float4 b, float x0, float x1, float y0, float y1) {
  return b.x <= x1 && b.y >= x0 && b.z <= y1 && b.w >= y0;
}

template <bool DEPTH>
__global__ void __launch_bounds__(THREADS) render_fwd_kernel(const gsb_render_fwd_args a, int gx) {
  __shared__ float2 s_xy[BATCH];
  __shared__ float4 s_cop[BATCH];   // conic a, b, c, opacity
  __shared__ float4 s_rgbd[BATCH];  // r, g, b, depth
  __shared__ float4 s_box[BATCH];   // alpha_box
  const int tile = blockIdx.x;
  const int lane = threadIdx.x & 31;
  int pxi, py0;
  pixels_of(tile, gx, pxi, py0);
  const int2 range = reinterpret_cast<const int2*>(a.ranges)[tile];
  const float4* rec = reinterpret_cast<const float4*>(a.records);
  const float fx = (float)pxi;
  // the warp's 8x8 pixel block
  const float bx0 = (float)(__shfl_sync(FULL, pxi, 0)), by0 = (float)(__shfl_sync(FULL, py0, 0));
  const float bx1 = bx0 + 7.0f, by1 = by0 + 7.0f;
  float fy[2], T[2], c0[2], c1[2], c2[2], wsum[2], dacc[2];
  int last[2];
  bool inside[2], done[2];
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const int py = py0 + 4 * p;
    fy[p] = (float)py;
    inside[p] = pxi < a.W && py < a.H;
    done[p] = !inside[p];
    T[p] = 1.0f;
    c0[p] = c1[p] = c2[p] = wsum[p] = dacc[p] = 0.0f;
    last[p] = 0;
  }
  for (int b = range.x; b < range.y; b += BATCH) {
    if (__syncthreads_count(done[0] && done[1]) == THREADS) break;
    const int i = b + threadIdx.x;
    if (i < range.y) {
      const int id = a.point_list[i];
      const float4 q0 = __ldg(rec + (size_t)id * 3 + 0);
      const float4 q1 = __ldg(rec + (size_t)id * 3 + 1);
      const float4 q2 = __ldg(rec + (size_t)id * 3 + 2);
      s_xy[threadIdx.x] = make_float2(q0.x, q0.y);
      s_cop[threadIdx.x] = make_float4(q0.z, q0.w, q1.x, q1.y);
      s_rgbd[threadIdx.x] = make_float4(q2.x, q2.y, q2.z, q1.z);
      s_box[threadIdx.x] = alpha_box(q0.x, q0.y, q0.z, q0.w, q1.x, q1.y);
    }
    __syncthreads();
    const int cnt = min(BATCH, range.y - b);
    // Each lane tests one staged Gaussian against the warp's block; the warp
    // then visits only the hits, in front-to-back order.
    for (int cb = 0; cb < cnt; cb += 32) {
      if (__all_sync(FULL, done[0] && done[1])) break;
      const int g = cb + lane;
      unsigned hits = __ballot_sync(FULL, g < cnt && box_hits(s_box[g], bx0, bx1, by0, by1));
      while (hits) {
      const int j = cb + __ffs(hits) - 1;
      hits &= hits - 1;
      if (done[0] && done[1]) continue;
      const float2 xy = s_xy[j];
      const float4 co = s_cop[j];
      const float dx = xy.x - fx;
      const float adx2 = co.x * dx * dx;
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        if (done[p]) continue;
        const float dy = xy.y - fy[p];
        const float power = -0.5f * (adx2 + co.z * dy * dy) - co.y * dx * dy;
        if (power > 0.0f) continue;
        const float alpha = fminf(0.99f, co.w * fast_exp(power));
        if (alpha < (1.0f / 255.0f)) continue;
        const float test_T = T[p] * (1.0f - alpha);
        if (test_T < 0.0001f) {
          done[p] = true;
          continue;
        }
        const float contrib = alpha * T[p];
        const float4 cd = s_rgbd[j];
        c0[p] += cd.x * contrib;
        c1[p] += cd.y * contrib;
        c2[p] += cd.z * contrib;
        wsum[p] += contrib;
        if (DEPTH) dacc[p] += cd.w * contrib;
        T[p] = test_T;
        last[p] = b - range.x + j + 1;
      }
      }
    }
  }
  const long long npix = (long long)a.W * a.H;
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    if (!inside[p]) continue;
    const long long pix = (long long)(py0 + 4 * p) * a.W + pxi;
    a.n_contrib[pix] = last[p];
    a.out_color[pix] = c0[p] + T[p] * a.background[0];
    a.out_color[npix + pix] = c1[p] + T[p] * a.background[1];
    a.out_color[2 * npix + pix] = c2[p] + T[p] * a.background[2];
    a.out_alpha[pix] = wsum[p];
    a.out_depth[pix] = dacc[p];
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

// Back-to-front state of one pixel (backward_kernels.py:606-625).
struct BwdPixel {
  int lc;
  float fy, T, T_final, g0, g1, g2, gd, ga, bg_dot;
  float ar0, ar1, ar2, adr, aar, la, lc0, lc1, lc2, ld;
};

// One pixel's contribution of the Gaussian at this position, added to v[]
// (backward_kernels.py:637-685).  Returns whether the pixel contributed.
template <bool DEPTH>
__device__ __forceinline__ bool bwd_pixel(BwdPixel& s, float dx, float adx2, const float2 xy,
                                          const float4 co, const float4 cd, float ddelx_dx,
                                          float ddely_dy, float (&v)[10]) {
  const float dy = xy.y - s.fy;
  const float power = -0.5f * (adx2 + co.z * dy * dy) - co.y * dx * dy;
  if (power > 0.0f) return false;
  const float G = fast_exp(power);
  const float alpha = fminf(0.99f, co.w * G);
  if (alpha < (1.0f / 255.0f)) return false;
  const float oma = fmaxf(1.0f - alpha, 1.0e-5f);
  const float inv_oma = fast_rcp(oma);
  s.T = s.T * inv_oma;
  const float dchannel = alpha * s.T;
  s.ar0 = s.la * s.lc0 + (1.0f - s.la) * s.ar0;
  s.ar1 = s.la * s.lc1 + (1.0f - s.la) * s.ar1;
  s.ar2 = s.la * s.lc2 + (1.0f - s.la) * s.ar2;
  s.lc0 = cd.x;
  s.lc1 = cd.y;
  s.lc2 = cd.z;
  float dL_dopa = (cd.x - s.ar0) * s.g0 + (cd.y - s.ar1) * s.g1 + (cd.z - s.ar2) * s.g2;
  v[7] += dchannel * s.g0;
  v[8] += dchannel * s.g1;
  v[9] += dchannel * s.g2;
  if (DEPTH) {
    s.adr = s.la * s.ld + (1.0f - s.la) * s.adr;
    s.ld = cd.w;
    dL_dopa += (cd.w - s.adr) * s.gd;
    v[2] += dchannel * s.gd;
  }
  s.aar = s.la + (1.0f - s.la) * s.aar;
  dL_dopa += (1.0f - s.aar) * s.ga;
  dL_dopa *= s.T;
  s.la = alpha;
  dL_dopa += (-s.T_final * inv_oma) * s.bg_dot;
  const float dL_dG = co.w * dL_dopa;
  const float gdx = G * dx, gdy = G * dy;
  const float dG_ddelx = -gdx * co.x - gdy * co.y;
  const float dG_ddely = -gdy * co.z - gdx * co.y;
  v[0] += dL_dG * dG_ddelx * ddelx_dx;
  v[1] += dL_dG * dG_ddely * ddely_dy;
  v[3] += -0.5f * gdx * dx * dL_dG;
  v[4] += -0.5f * gdx * dy * dL_dG;
  v[5] += -0.5f * gdy * dy * dL_dG;
  v[6] += G * dL_dopa;
  return true;
}

template <bool DEPTH>
__global__ void __launch_bounds__(THREADS) render_bwd_kernel(const gsb_render_bwd_args a, int gx) {
  __shared__ int s_id[BATCH];
  __shared__ float2 s_xy[BATCH];
  __shared__ float4 s_cop[BATCH];
  __shared__ float4 s_rgbd[BATCH];
  __shared__ float4 s_box[BATCH];
  __shared__ int s_max[THREADS / 32];
  const int tile = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int pxi, py0;
  pixels_of(tile, gx, pxi, py0);
  const int2 range = reinterpret_cast<const int2*>(a.ranges)[tile];
  const int n = range.y - range.x;
  const float4* rec = reinterpret_cast<const float4*>(a.records);
  const long long npix = (long long)a.W * a.H;

  BwdPixel px[2];
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    BwdPixel& s = px[p];
    const int py = py0 + 4 * p;
    s.fy = (float)py;
    s.lc = 0;
    s.T_final = s.g0 = s.g1 = s.g2 = s.gd = s.ga = s.bg_dot = 0.0f;
    if (pxi < a.W && py < a.H && n > 0) {
      const long long pix = (long long)py * a.W + pxi;
      s.lc = a.n_contrib[pix];
      s.T_final = 1.0f - a.out_alpha[pix];
      s.g0 = a.grad_color[pix];
      s.g1 = a.grad_color[npix + pix];
      s.g2 = a.grad_color[2 * npix + pix];
      if (DEPTH && a.grad_depth) s.gd = a.grad_depth[pix];
      if (a.grad_alpha) s.ga = a.grad_alpha[pix];
      s.bg_dot = a.background[0] * s.g0 + a.background[1] * s.g1 + a.background[2] * s.g2;
    }
    s.T = s.T_final;
    s.ar0 = s.ar1 = s.ar2 = s.adr = s.aar = s.la = s.lc0 = s.lc1 = s.lc2 = s.ld = 0.0f;
  }
  const int warp_max = __reduce_max_sync(FULL, max(px[0].lc, px[1].lc));
  if (lane == 0) s_max[warp] = warp_max;
  __syncthreads();
  int cta_max = 0;
#pragma unroll
  for (int w = 0; w < THREADS / 32; ++w) cta_max = max(cta_max, s_max[w]);
  cta_max = min(cta_max, n);  // n_contrib never exceeds the tile's list
  if (cta_max <= 0) return;

  const float ddelx_dx = 0.5f * (float)a.W;
  const float ddely_dy = 0.5f * (float)a.H;
  const float fx = (float)pxi;
  const float bx0 = (float)(__shfl_sync(FULL, pxi, 0)), by0 = (float)(__shfl_sync(FULL, py0, 0));
  const float bx1 = bx0 + 7.0f, by1 = by0 + 7.0f;

  for (int hi = cta_max; hi > 0; hi -= BATCH) {
    const int lo = max(0, hi - BATCH);
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
      s_box[k] = alpha_box(q0.x, q0.y, q0.z, q0.w, q1.x, q1.y);
    }
    __syncthreads();
    const int top = min(hi, warp_max);
    // Lanes test staged Gaussians against the warp's 8x8 block; the warp
    // visits only the hits below its own maximum, back to front.
    for (int cb = ((top - lo - 1) >> 5) << 5; cb >= 0 && top > lo; cb -= 32) {
      const int g = cb + lane;
      unsigned hits = __ballot_sync(FULL, g < top - lo && box_hits(s_box[g], bx0, bx1, by0, by1));
      while (hits) {
      const int j = cb + 31 - __clz(hits);
      hits &= ~(1u << (j - cb));
      const int pos = lo + j;
      float v[10];
#pragma unroll
      for (int k = 0; k < 10; ++k) v[k] = 0.0f;
      bool contrib = false;
      if (pos < px[0].lc || pos < px[1].lc) {
        const float2 xy = s_xy[j];
        const float4 co = s_cop[j];
        const float4 cd = s_rgbd[j];
        const float dx = xy.x - fx;
        const float adx2 = co.x * dx * dx;
        if (pos < px[0].lc) contrib |= bwd_pixel<DEPTH>(px[0], dx, adx2, xy, co, cd, ddelx_dx, ddely_dy, v);
        if (pos < px[1].lc) contrib |= bwd_pixel<DEPTH>(px[1], dx, adx2, xy, co, cd, ddelx_dx, ddely_dy, v);
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
      !a->background || !a->out_alpha || !a->n_contrib || !a->grad_color || !a->grad_acc) {
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
