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
// B200 design.  Forward: one 128-thread CTA per 16x16 tile; each thread owns
// TWO pixels (rows y and y+4 of its warp's 8x8 block), so every Gaussian
// staged in shared memory is read once per two pixels and the per-(warp,
// Gaussian) control work covers 64 pixels.  Backward, on grids of 6,000
// tiles or more: one 64-thread CTA per tile; each warp owns an 8x16 column
// block and each thread FOUR pixels (rows y, y+4, y+8, y+12) as two packed
// pairs, so the per-(warp, Gaussian) work that does not scale with pixels --
// culling, operand loads, the 10-term warp reduction and the atomics --
// covers 128 pixels (a Gaussian that reaches both 8x8 blocks of a column
// costs one hit, not two).  On smaller grids, where the heaviest tile sets
// the kernel's length, the backward keeps the forward's four warps per tile
// and two pixels per thread.  Both directions stage Gaussians
// per batch from the 48-byte render records (three 16-byte loads per
// Gaussian); exp is one MUFU.EX2, 1/(1-alpha) one MUFU.RCP.  Backward: the
// CTA walks its list from the CTA-wide maximum contributor down, each warp
// skips positions above its own maximum, tests each Gaussian against the
// halves of its block that hold whole pixel pairs (so a pair the Gaussian
// cannot reach is skipped warp-wide), a warp vote skips
// Gaussians no lane uses, and the ten gradient terms (already summed over the
// thread's pixels) are reduced across the warp with a 12-shuffle transpose
// reduction (instead of 10 x 5 butterfly shuffles); 10 lanes then issue one
// float atomic each into the per-Gaussian accumulator.
#include "gsb_common.cuh"

namespace gsb {
namespace {

constexpr int THREADS = launch::RENDER;
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

// Ellipse data for the exact block test: conic (a, b, c) and the culling
// threshold on q = a dx^2 + 2b dx dy + c dy^2.  alpha >= 1/255 needs
// q <= t = 2 ln(255 op); the test uses t * 1.02 + 0.05 (alpha 2.5% below the
// cut-off at the edge, far above the rounding of the per-pixel evaluation),
// and +inf for a conic that is not positive definite (never culled).
__device__ __forceinline__ float4 cull_ellipse(float a, float b, float c, float op) {
  const float inf = __int_as_float(0x7f800000);
  if (!(a > 0.0f) || !(a * c - b * b > 0.0f)) return make_float4(a, b, c, inf);
  const float t = 2.0f * __logf(255.0f * op);
  return make_float4(a, b, c, t * 1.02f + 0.05f);
}

// Whether the ellipse {q <= e.w} around (cx, cy) reaches the pixel block
// [x0, x1] x [y0, y1] (d = centre - pixel, as in the per-pixel evaluation).
// Outside the block the minimum of the convex q lies on an edge; each edge
// minimum is the clamped stationary point.
__device__ __forceinline__ bool ellipse_hits(float cx, float cy, const float4 e, float x0, float x1,
                                             float y0, float y1) {
  if (!(e.w < __int_as_float(0x7f800000))) return true;
  const float X0 = cx - x1, X1 = cx - x0, Y0 = cy - y1, Y1 = cy - y0;
  if (X0 <= 0.0f && X1 >= 0.0f && Y0 <= 0.0f && Y1 >= 0.0f) return true;
  const float ia = fast_rcp(e.x), ic = fast_rcp(e.z);
  float q = __int_as_float(0x7f800000);
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const float X = k ? X1 : X0;
    const float dy = fminf(fmaxf(-e.y * X * ic, Y0), Y1);
    q = fminf(q, e.x * X * X + (2.0f * e.y * X + e.z * dy) * dy);
    const float Y = k ? Y1 : Y0;
    const float dx = fminf(fmaxf(-e.y * Y * ia, X0), X1);
    q = fminf(q, e.z * Y * Y + (2.0f * e.y * Y + e.x * dx) * dx);
  }
  return q <= e.w;
}

// Exponent of a Gaussian at pixel offset (dx, dy) in log2 units, from the
// staged coefficients cf = (-a/2, -b, -c/2) * log2(e):
//   power2 = cf.x dx^2 + (cf.z dy + cf.y dx) dy = log2(e) * (-(a dx^2 + c dy^2)/2 - b dx dy),
// so exp(power) = ex2(power2).  ax = cf.x dx^2 and bx = cf.y dx are shared by
// the thread's two pixels (same column).  Forward and backward evaluate it
// through power2_of2 with explicit FMAs, so they make the same alpha
// decisions bit for bit.
__device__ __forceinline__ float4 power_coefs(float a, float b, float c) {
  const float L2E = 1.4426950408889634f;
  return make_float4(-0.5f * L2E * a, -L2E * b, -0.5f * L2E * c, 0.0f);
}
__device__ __forceinline__ void column_terms(const float4 cf, float dx, float& ax, float& bx) {
  ax = __fmul_rn(__fmul_rn(cf.x, dx), dx);
  bx = __fmul_rn(cf.y, dx);
}
// The exponent for the thread's two pixels (dy = (dy0, dy1)) as one packed
// stream: per component fma(fma(cf.z, dy, bx), dy, ax), each rounded once.
__device__ __forceinline__ float2 power2_of2(const float4 cf, float ax, float bx, float2 dy) {
  return __ffma2_rn(__ffma2_rn(make_float2(cf.z, cf.z), dy, make_float2(bx, bx)), dy, make_float2(ax, ax));
}
// 1 - v per component, rounded once (fma(v, -1, 1) is the subtraction).
__device__ __forceinline__ float2 one_minus2(float2 v) {
  return __ffma2_rn(v, make_float2(-1.0f, -1.0f), make_float2(1.0f, 1.0f));
}
__device__ __forceinline__ float half_of(float2 v, int p) { return p ? v.y : v.x; }
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// AUX: also record the first top_k contributors of every pixel in
// front-to-back order -- Gaussian id, compositing weight alpha * T and the
// offset (dx, dy) = centre - pixel -- the flow render's auxiliary outputs
// (flow_kernels.py:14-180); slots left empty are written -1 / 0 / 0.
template <bool DEPTH, bool AUX>
__global__ void __launch_bounds__(THREADS, 10) render_fwd_kernel(const gsb_render_fwd_args a, int gx) {
  __shared__ int s_id[AUX ? BATCH : 1];
  __shared__ float2 s_xy[BATCH];
  __shared__ float4 s_cf[BATCH];    // power coefficients, opacity in .w
  __shared__ float4 s_rgbd[BATCH];  // r, g, b, depth
  __shared__ float4 s_box[BATCH];   // alpha_box
  __shared__ float4 s_el[BATCH];    // cull_ellipse
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
  // The thread's two pixels (same column, rows py0 and py0 + 4) share every
  // Gaussian operand, so their arithmetic runs as packed f32x2 operations
  // (__ffma2_rn / __fmul2_rn / __fadd2_rn: each rounds per component like
  // the scalar __fmaf_rn / __fmul_rn / __fadd_rn, but the compiler may fuse
  // a packed multiply into the add it feeds, so composed expressions match a
  // scalar build to rounding, not bit for bit).
  float fy[2];
  float2 T = make_float2(1.0f, 1.0f), c0 = make_float2(0.0f, 0.0f), c1 = c0, c2 = c0, wsum = c0, dacc = c0;
  int last[2] = {0, 0}, nsucc[2] = {0, 0};
  bool inside[2], done[2];
  const long long npix = (long long)a.W * a.H;
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const int py = py0 + 4 * p;
    fy[p] = (float)py;
    inside[p] = pxi < a.W && py < a.H;
    done[p] = !inside[p];
  }
  const float2 nfy = make_float2(-fy[0], -fy[1]);
  for (int b = range.x; b < range.y; b += BATCH) {
    if (__syncthreads_count(done[0] && done[1]) == THREADS) break;
    const int i = b + threadIdx.x;
    if (i < range.y) {
      const int id = a.point_list[i];
      const float4 q0 = __ldg(rec + (size_t)id * 3 + 0);
      const float4 q1 = __ldg(rec + (size_t)id * 3 + 1);
      const float4 q2 = __ldg(rec + (size_t)id * 3 + 2);
      if (AUX) s_id[threadIdx.x] = id;
      s_xy[threadIdx.x] = make_float2(q0.x, q0.y);
      float4 cf = power_coefs(q0.z, q0.w, q1.x);
      cf.w = q1.y;
      s_cf[threadIdx.x] = cf;
      s_rgbd[threadIdx.x] = make_float4(q2.x, q2.y, q2.z, q1.z);
      s_box[threadIdx.x] = alpha_box(q0.x, q0.y, q0.z, q0.w, q1.x, q1.y);
      s_el[threadIdx.x] = cull_ellipse(q0.z, q0.w, q1.x, q1.y);
    }
    __syncthreads();
    const int cnt = min(BATCH, range.y - b);
    // Each lane tests one staged Gaussian against the warp's block; the warp
    // then visits only the hits, in front-to-back order.
    for (int cb = 0; cb < cnt; cb += 32) {
      if (__all_sync(FULL, done[0] && done[1])) break;
      const int g = cb + lane;
      bool hit = false;
      if (g < cnt) {
        const float4 bb = s_box[g];
        hit = bb.x <= bx1 && bb.y >= bx0 && bb.z <= by1 && bb.w >= by0;
      }
      if (__any_sync(FULL, hit) && hit) {
        const float2 cxy = s_xy[g];
        hit = ellipse_hits(cxy.x, cxy.y, s_el[g], bx0, bx1, by0, by1);
      }
      unsigned hits = __ballot_sync(FULL, hit);
      while (hits) {
      const int j = cb + __ffs(hits) - 1;
      hits &= hits - 1;
      if (done[0] && done[1]) continue;
      const float2 xy = s_xy[j];
      const float4 cf = s_cf[j];
      const float dx = xy.x - fx;
      float ax, bx;
      column_terms(cf, dx, ax, bx);
      // Both pixels' exponent, alpha and transmittance run straight through
      // as one packed stream; the per-pixel decisions only select.
      const float2 dy = __fadd2_rn(make_float2(xy.y, xy.y), nfy);
      const float2 pw = power2_of2(cf, ax, bx, dy);
      float2 al = __fmul2_rn(make_float2(cf.w, cf.w), make_float2(ex2_approx(pw.x), ex2_approx(pw.y)));
      al.x = fminf(0.99f, al.x);
      al.y = fminf(0.99f, al.y);
      const float2 tt = __fmul2_rn(T, one_minus2(al));
      const bool ok0 = !done[0] && !(pw.x > 0.0f) && !(al.x < (1.0f / 255.0f));
      const bool ok1 = !done[1] && !(pw.y > 0.0f) && !(al.y < (1.0f / 255.0f));
      // a pixel whose transmittance would drop below 1e-4 stops before this Gaussian
      const bool st0 = ok0 && tt.x < 0.0001f, st1 = ok1 && tt.y < 0.0001f;
      const bool acc[2] = {ok0 && !st0, ok1 && !st1};
      done[0] = done[0] || st0;
      done[1] = done[1] || st1;
      float2 cm = __fmul2_rn(al, T);  // alpha * T, zero where the pixel does not take the Gaussian
      cm.x = acc[0] ? cm.x : 0.0f;
      cm.y = acc[1] ? cm.y : 0.0f;
      const float4 cd = s_rgbd[j];
      c0 = __ffma2_rn(make_float2(cd.x, cd.x), cm, c0);
      c1 = __ffma2_rn(make_float2(cd.y, cd.y), cm, c1);
      c2 = __ffma2_rn(make_float2(cd.z, cd.z), cm, c2);
      wsum = __fadd2_rn(wsum, cm);
      if (DEPTH) dacc = __ffma2_rn(make_float2(cd.w, cd.w), cm, dacc);
      T.x = acc[0] ? tt.x : T.x;
      T.y = acc[1] ? tt.y : T.y;
      const int idx = b - range.x + j + 1;
      last[0] = acc[0] ? idx : last[0];
      last[1] = acc[1] ? idx : last[1];
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        if (!acc[p]) continue;
        const float contrib = p ? cm.y : cm.x;
        if (AUX) {
          if (nsucc[p] < a.top_k) {
            const long long o = (long long)nsucc[p] * npix + (long long)(py0 + 4 * p) * a.W + pxi;
            if (a.aux_scratch) {
              reinterpret_cast<float4*>(a.aux_scratch)[o] =
                  make_float4(__int_as_float(s_id[j]), contrib, dx, xy.y - fy[p]);
            } else {
              a.gs_per_pixel[o] = s_id[j];
              a.weight_per_gs_pixel[o] = contrib;
              a.x_mu[o] = dx;
              a.x_mu[(long long)a.top_k * npix + o] = xy.y - fy[p];
            }
          }
          ++nsucc[p];
        }
      }
      }
    }
  }
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    if (!inside[p]) continue;
    const long long pix = (long long)(py0 + 4 * p) * a.W + pxi;
    if (AUX)
      for (int k = nsucc[p]; k < a.top_k; ++k) {
        const long long o = (long long)k * npix + pix;
        if (a.aux_scratch) {
          reinterpret_cast<float4*>(a.aux_scratch)[o] = make_float4(__int_as_float(-1), 0.0f, 0.0f, 0.0f);
        } else {
          a.gs_per_pixel[o] = -1;
          a.weight_per_gs_pixel[o] = 0.0f;
          a.x_mu[o] = 0.0f;
          a.x_mu[(long long)a.top_k * npix + o] = 0.0f;
        }
      }
    const float Tp = half_of(T, p);
    a.n_contrib[pix] = last[p];
    a.out_color[pix] = half_of(c0, p) + Tp * a.background[0];
    a.out_color[npix + pix] = half_of(c1, p) + Tp * a.background[1];
    a.out_color[2 * npix + pix] = half_of(c2, p) + Tp * a.background[2];
    a.out_alpha[pix] = half_of(wsum, p);
    a.out_depth[pix] = half_of(dacc, p);
  }
}

// Splits the (K,H,W) 16-byte slot records into the flow outputs: one thread
// per (slot, pixel), coalesced loads and stores.
__global__ void flow_aux_split_kernel(long long n, long long kn, const float4* __restrict__ scratch,
                                      int* __restrict__ ids, float* __restrict__ weights,
                                      float* __restrict__ x_mu) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float4 r = scratch[i];
  ids[i] = __float_as_int(r.x);
  weights[i] = r.y;
  x_mu[i] = r.z;
  x_mu[kn + i] = r.w;
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

// One halving stage of a transpose reduction: lanes whose `bit` is clear keep
// the first ceil(N/2) values and send the rest (zero-padded), lanes whose bit
// is set keep the rest and send the first, to the lane `xmask` apart.  The
// adds run two outputs per packed f32x2 add (per component the scalar sum).
template <int N>
__device__ __forceinline__ void halve(const float (&in)[N], float (&out)[(N + 1) / 2], bool bit, int xmask) {
  constexpr int H = (N + 1) / 2;
  float keep[H], recv[H];
#pragma unroll
  for (int k = 0; k < H; ++k) {
    const float lo = in[k];
    const float hi = (k + H < N) ? in[k + H] : 0.0f;
    keep[k] = bit ? hi : lo;
    recv[k] = __shfl_xor_sync(FULL, bit ? lo : hi, xmask);
  }
#pragma unroll
  for (int k = 0; k + 1 < H; k += 2) {
    const float2 sum = __fadd2_rn(make_float2(keep[k], keep[k + 1]), make_float2(recv[k], recv[k + 1]));
    out[k] = sum.x;
    out[k + 1] = sum.y;
  }
  if (H & 1) out[H - 1] = keep[H - 1] + recv[H - 1];
}

// Transpose reduction of N (17..32) per-lane values over a warp in five
// halving stages (N + 2 shuffles or fewer; two ten-value reductions take 24):
// on return each value's warp total sits in one lane; the returned index is
// the value held (0..N-1), or -1 for the lanes left with padding.
template <int N>
__device__ __forceinline__ int warp_reduce_n(const float (&v)[N], float& out) {
  static_assert(N > 16 && N <= 32, "five halving stages");
  constexpr int N1 = (N + 1) / 2, N2 = (N1 + 1) / 2, N3 = (N2 + 1) / 2, N4 = (N3 + 1) / 2;
  static_assert(N4 == 2, "five halving stages end in one value");
  const int lane = threadIdx.x & 31;
  float a[N1], b[N2], c[N3], d[N4], e[1];
  halve<N>(v, a, lane & 16, 16);
  halve<N1>(a, b, lane & 8, 8);
  halve<N2>(b, c, lane & 4, 4);
  halve<N3>(c, d, lane & 2, 2);
  halve<N4>(d, e, lane & 1, 1);
  out = e[0];
  // the original index of the kept value: each stage halves the slots and
  // keeps the upper half (offset ceil(slots/2)) where the lane's bit is set;
  // real values fill the lowest slots, so n counts those still held
  int idx = 0, n = N, slots = N;
  const int bits[5] = {lane & 16, lane & 8, lane & 4, lane & 2, lane & 1};
#pragma unroll
  for (int st = 0; st < 5; ++st) {
    const int h = (slots + 1) / 2;
    if (bits[st]) {
      idx += h;
      n -= h;
    } else {
      n = n < h ? n : h;
    }
    slots = h;
  }
  return n >= 1 ? idx : -1;
}

// Gradient terms per hit in the paired reduction: all ten, or without the
// depth term (index 2) when no depth gradient is asked for.
template <bool DEPTH>
__device__ __forceinline__ int pair_term_slot(int t) { return (DEPTH || t < 2) ? t : t + 1; }

// Back-to-front state of the thread's two pixels (backward_kernels.py:
// 606-625), one f32x2 component per pixel.  The colour part of accum_rec
// only enters dL/dalpha through its dot product with the pixel's colour
// gradient g, so the state keeps that dot product S = accum_rec . g.  The
// reference advances accum_rec / last_alpha / last_color lazily, at the next
// contributing Gaussian; here S (and the depth / alpha accumulators) advance
// eagerly at the end of each contributing Gaussian -- the same operands in
// the same expression, so the same values -- which leaves no last_* state:
// with alpha masked to zero where a pixel does not take the Gaussian, the
// update fma(0, ., S) leaves S unchanged and needs no per-pixel select.
struct BwdPair {
  int lc0, lc1;
  float2 nfy, T, nTf, g0, g1, g2, gd, ga, bg_dot;
  float2 S, adr, aar;
};

// Gradient sums of one Gaussian over the thread's pixels.  The per-pixel
// terms of backward_kernels.py:637-685 are, with u = G * dL/dalpha,
//   d/dx   = -op * W/2 * u (a dx + b dy)     d/dconic_a = -op/2 * u dx^2
//   d/dy   = -op * H/2 * u (c dy + b dx)     d/dconic_b = -op/2 * u dx dy
//   d/dop  = u                               d/dconic_c = -op/2 * u dy^2
// so each pixel only accumulates the moments U = sum u, UY = sum u dy,
// UYY = sum u dy^2 (dx is the thread's column); the Gaussian's constants
// (op, a, b, c, W/2, H/2, -1/2) are applied once, after the warp reduction.
struct BwdSums {
  float U, UY, UYY, dcol0, dcol1, dcol2, ddepth;
};

// The two pixels' contributions of the Gaussian at this position (3DGS
// recurrences accum_rec / last_alpha / last_color, backward_kernels.py:
// 637-671), written to m; c0 / c1 tell whether each pixel contributed.  The
// arithmetic runs straight through as one packed stream (both pixels share
// the Gaussian's operands); the per-pixel decisions only mask alpha and G.
// For a contributing pixel every value is the same expression as a scalar
// evaluation of that pixel, to rounding.
// One Gaussian at this position applied to a pixel pair back to front (3DGS
// recurrences accum_rec / last_alpha / last_color, backward_kernels.py:
// 637-671): updates the pair's state and returns the per-pixel terms the
// gradient sums are made of; c0 / c1 tell whether each pixel contributed.
// The arithmetic runs straight through as one packed stream (both pixels
// share the Gaussian's operands); the per-pixel decisions only mask alpha
// and G.  For a contributing pixel every value is the same expression as a
// scalar evaluation of that pixel, to rounding.  A pixel that does not take
// the Gaussian gets zero terms and an unchanged state.
struct PairTerms {
  float2 u, uy, dy, dch;
};

template <bool DEPTH, bool GA>
__device__ __forceinline__ PairTerms bwd_pair_core(BwdPair& s, bool e0, bool e1, const float4 cf, float ax,
                                                   float bx, float y, const float4 cd, bool has_bg, bool& c0,
                                                   bool& c1) {
  const float2 neg1 = make_float2(-1.0f, -1.0f);
  const float2 dy = __fadd2_rn(make_float2(y, y), s.nfy);
  const float2 pw = power2_of2(cf, ax, bx, dy);
  const float2 G = make_float2(ex2_approx(pw.x), ex2_approx(pw.y));
  float2 al = __fmul2_rn(make_float2(cf.w, cf.w), G);
  al.x = fminf(0.99f, al.x);
  al.y = fminf(0.99f, al.y);
  c0 = e0 && !(pw.x > 0.0f) && !(al.x < (1.0f / 255.0f));
  c1 = e1 && !(pw.y > 0.0f) && !(al.y < (1.0f / 255.0f));
  const float2 am = make_float2(c0 ? al.x : 0.0f, c1 ? al.y : 0.0f);
  // alpha <= 0.99, so 1 - alpha >= 0.01 (the reference's 1e-5 floor never binds)
  const float2 oma = one_minus2(am);
  const float2 inv = make_float2(fast_rcp(oma.x), fast_rcp(oma.y));
  const float2 T = __fmul2_rn(s.T, inv);
  const float2 dch = __fmul2_rn(am, T);
  const float2 cg = __ffma2_rn(make_float2(cd.z, cd.z), s.g2,
                               __ffma2_rn(make_float2(cd.y, cd.y), s.g1, __fmul2_rn(make_float2(cd.x, cd.x), s.g0)));
  float2 dL = __ffma2_rn(s.S, neg1, cg);  // cg - S
  const float2 cdw = make_float2(cd.w, cd.w);
  if (DEPTH) dL = __ffma2_rn(__ffma2_rn(s.adr, neg1, cdw), s.gd, dL);
  if (GA) dL = __ffma2_rn(one_minus2(s.aar), s.ga, dL);
  dL = __fmul2_rn(dL, T);
  if (has_bg) dL = __ffma2_rn(__fmul2_rn(s.nTf, inv), s.bg_dot, dL);
  const float2 u = __fmul2_rn(make_float2(c0 ? G.x : 0.0f, c1 ? G.y : 0.0f), dL);
  const float2 uy = __fmul2_rn(u, dy);
  // state: transmittance behind the next Gaussian, accumulators advanced eagerly
  s.T.x = c0 ? T.x : s.T.x;
  s.T.y = c1 ? T.y : s.T.y;
  s.S = __ffma2_rn(am, __ffma2_rn(s.S, neg1, cg), s.S);
  if (DEPTH) s.adr = __ffma2_rn(am, __ffma2_rn(s.adr, neg1, cdw), s.adr);
  if (GA) s.aar = __ffma2_rn(one_minus2(am), s.aar, am);
  return PairTerms{u, uy, dy, dch};
}


// The pair's sums (BwdSums), accumulated as pixel 0 then pixel 1.
template <bool DEPTH, bool GA>
__device__ __forceinline__ void bwd_pair(BwdPair& s, bool e0, bool e1, const float4 cf, float ax, float bx,
                                         float y, const float4 cd, bool has_bg, BwdSums& m, bool& c0, bool& c1) {
  const PairTerms t = bwd_pair_core<DEPTH, GA>(s, e0, e1, cf, ax, bx, y, cd, has_bg, c0, c1);
  m.U = t.u.x + t.u.y;
  m.UY = t.uy.x + t.uy.y;
  m.UYY = __fmaf_rn(t.uy.y, t.dy.y, __fmul_rn(t.uy.x, t.dy.x));
  m.dcol0 = __fmaf_rn(t.dch.y, s.g0.y, __fmul_rn(t.dch.x, s.g0.x));
  m.dcol1 = __fmaf_rn(t.dch.y, s.g1.y, __fmul_rn(t.dch.x, s.g1.x));
  m.dcol2 = __fmaf_rn(t.dch.y, s.g2.y, __fmul_rn(t.dch.x, s.g2.x));
  if (DEPTH) m.ddepth = __fmaf_rn(t.dch.y, s.gd.y, __fmul_rn(t.dch.x, s.gd.x));
}

// Sums of several pairs kept per pixel slot (packed): the first pair stores
// its terms, later pairs add theirs, and one horizontal add per sum ends the
// hit -- for two pairs 16 instructions where two BwdSums and their addition
// take 26.
struct BwdSums2 {
  float2 U, UY, UYY, d0, d1, d2, dd;
};

template <bool DEPTH, bool FIRST>
__device__ __forceinline__ void sums2_add(BwdSums2& m, const PairTerms& t, const BwdPair& s) {
  if (FIRST) {
    m.U = t.u;
    m.UY = t.uy;
    m.UYY = __fmul2_rn(t.uy, t.dy);
    m.d0 = __fmul2_rn(t.dch, s.g0);
    m.d1 = __fmul2_rn(t.dch, s.g1);
    m.d2 = __fmul2_rn(t.dch, s.g2);
    if (DEPTH) m.dd = __fmul2_rn(t.dch, s.gd);
  } else {
    m.U = __fadd2_rn(m.U, t.u);
    m.UY = __fadd2_rn(m.UY, t.uy);
    m.UYY = __ffma2_rn(t.uy, t.dy, m.UYY);
    m.d0 = __ffma2_rn(t.dch, s.g0, m.d0);
    m.d1 = __ffma2_rn(t.dch, s.g1, m.d1);
    m.d2 = __ffma2_rn(t.dch, s.g2, m.d2);
    if (DEPTH) m.dd = __ffma2_rn(t.dch, s.gd, m.dd);
  }
}

template <bool DEPTH>
__device__ __forceinline__ void sums2_reduce(const BwdSums2& m2, BwdSums& m) {
  m.U = m2.U.x + m2.U.y;
  m.UY = m2.UY.x + m2.UY.y;
  m.UYY = m2.UYY.x + m2.UYY.y;
  m.dcol0 = m2.d0.x + m2.d0.y;
  m.dcol1 = m2.d1.x + m2.d1.y;
  m.dcol2 = m2.d2.x + m2.d2.y;
  if (DEPTH) m.ddepth = m2.dd.x + m2.dd.y;
}

// Backward launch shape: two warps per 16x16 tile, each owning an 8-column x
// 16-row block with FOUR pixels per thread (rows r, r+4, r+8, r+12 of its
// column), run as two packed f32x2 pairs that share every Gaussian operand
// (the column offset dx included).  Against a warp per 8x8 block, a Gaussian
// that covers both blocks of a column costs one hit -- one cull, one
// operand load, one 10-term warp reduction and one set of atomics -- for
// twice the pixels.  Culling is per 8x8 half (the rows of one pixel pair of
// every lane): a half the Gaussian cannot reach is a pair the warp skips;
// testing the four 8x4 quarters instead only masked pixels the per-pixel
// alpha test rejects anyway, and cost 4% more time.
constexpr int BWD_THREADS = launch::RENDER_BWD;
// Grids of at least this many tiles use the two-warp kernel (more pixels per
// hit); smaller ones the four-warp kernel (a shorter heaviest tile).  Render
// backward, 1M / 3M / 6M Gaussians, two-warp against four-warp kernel (ms):
// 1245x825 (4,056 tiles) 0.63/0.61, 0.86/0.83, 0.85/0.83; 1600x1063 (6,700)
// 0.76/0.74, 1.04/1.05, 1.02/1.05; 1920x1080 (8,160) 0.75/0.78, 1.05/1.11,
// 1.04/1.11; 2560x1440 (14,400) 0.98/1.08, 1.40/1.55, 1.40/1.56.
constexpr int BWD_TILE2_MIN_TILES = 6000;

// The thread's column and first row (slot k is row py0 + 4k).
__device__ __forceinline__ void bwd_pixels_of(int tile, int gx, int& px, int& py0) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tx = tile % gx, ty = tile / gx;
  px = tx * BLOCK_X + warp * 8 + (lane & 7);
  py0 = ty * BLOCK_Y + (lane >> 3);
}

// Which 8x8 halves (rows y0..y0+7, y0+8..y0+15) of the warp's 8x16 block
// staged Gaussian g can reach: box test, then the exact ellipse test per
// half (the forward's block test, same widened threshold).  A half decides
// whether its pixel pair runs; a pixel inside a reached half that the
// Gaussian does not reach fails the per-pixel alpha test and is left as is.
__device__ __forceinline__ void cull_halves8(int g, int cnt, const float4* s_box, const float2* s_xy,
                                             const float4* s_el, float x0, float x1, float y0, bool& top,
                                             bool& bot) {
  top = bot = false;
  if (g < cnt) {
    const float4 b = s_box[g];
    const bool xs = b.x <= x1 && b.y >= x0;
    top = xs && b.z <= y0 + 7.0f && b.w >= y0;
    bot = xs && b.z <= y0 + 15.0f && b.w >= y0 + 8.0f;
  }
  if (__any_sync(FULL, top || bot) && (top || bot)) {
    const float2 c = s_xy[g];
    const float4 e = s_el[g];
    if (top) top = ellipse_hits(c.x, c.y, e, x0, x1, y0, y0 + 7.0f);
    if (bot) bot = ellipse_hits(c.x, c.y, e, x0, x1, y0 + 8.0f, y0 + 15.0f);
  }
}

// DEPTH: compute_depth with a depth gradient given; GA: an alpha gradient
// given.  Without them those terms are exactly zero and are not evaluated.
template <bool DEPTH, bool GA>
__global__ void __launch_bounds__(BWD_THREADS, 11) render_bwd_tile2_kernel(const gsb_render_bwd_args a, int gx) {
  __shared__ int s_id[BATCH];
  __shared__ float2 s_xy[BATCH];
  __shared__ float4 s_cf[BATCH];    // power coefficients, opacity in .w
  __shared__ float4 s_con[BATCH];   // conic a, b, c
  __shared__ float4 s_rgbd[BATCH];
  __shared__ float4 s_box[BATCH];
  __shared__ float4 s_el[BATCH];
  __shared__ int s_max[BWD_THREADS / 32];
  const int tile = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int pxi, py0;
  bwd_pixels_of(tile, gx, pxi, py0);
  const int2 range = reinterpret_cast<const int2*>(a.ranges)[tile];
  const int n = range.y - range.x;
  const float4* rec = reinterpret_cast<const float4*>(a.records);
  const long long npix = (long long)a.W * a.H;
  const bool has_bg = a.background[0] != 0.0f || a.background[1] != 0.0f || a.background[2] != 0.0f;

  // pair 0: slots 0 and 1 (rows py0, py0 + 4); pair 1: slots 2 and 3 (rows py0 + 8, py0 + 12)
  BwdPair px[2];
  int lc_max = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float Tf[2], g0[2], g1[2], g2[2], gd[2], ga[2];
    int lc[2];
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const int py = py0 + 8 * h + 4 * p;
      lc[p] = 0;
      Tf[p] = g0[p] = g1[p] = g2[p] = gd[p] = ga[p] = 0.0f;
      if (pxi < a.W && py < a.H && n > 0) {
        const long long pix = (long long)py * a.W + pxi;
        lc[p] = a.n_contrib[pix];
        Tf[p] = 1.0f - a.out_alpha[pix];
        g0[p] = a.grad_color[pix];
        g1[p] = a.grad_color[npix + pix];
        g2[p] = a.grad_color[2 * npix + pix];
        if (DEPTH) gd[p] = a.grad_depth[pix];
        if (GA) ga[p] = a.grad_alpha[pix];
      }
    }
    BwdPair& s = px[h];
    s.lc0 = lc[0];
    s.lc1 = lc[1];
    lc_max = max(lc_max, max(lc[0], lc[1]));
    s.nfy = make_float2(-(float)(py0 + 8 * h), -(float)(py0 + 8 * h + 4));
    s.T = make_float2(Tf[0], Tf[1]);
    s.nTf = make_float2(-Tf[0], -Tf[1]);
    s.g0 = make_float2(g0[0], g0[1]);
    s.g1 = make_float2(g1[0], g1[1]);
    s.g2 = make_float2(g2[0], g2[1]);
    s.gd = make_float2(gd[0], gd[1]);
    s.ga = make_float2(ga[0], ga[1]);
    s.bg_dot = make_float2(a.background[0] * g0[0] + a.background[1] * g1[0] + a.background[2] * g2[0],
                           a.background[0] * g0[1] + a.background[1] * g1[1] + a.background[2] * g2[1]);
    s.S = s.adr = s.aar = make_float2(0.0f, 0.0f);
  }
  const int warp_max = __reduce_max_sync(FULL, lc_max);
  if (lane == 0) s_max[warp] = warp_max;
  __syncthreads();
  int cta_max = max(s_max[0], s_max[1]);
  cta_max = min(cta_max, n);  // n_contrib never exceeds the tile's list
  if (cta_max <= 0) return;

  const float half_w = 0.5f * (float)a.W;
  const float half_h = 0.5f * (float)a.H;
  // Which reduced term this lane writes (a lane constant): its accumulator
  // offset and the Gaussian-constant factor op * my_mul_op + my_mul_one
  // (-op W/2 for x, -op H/2 for y, -op/2 for the conic, 1 otherwise).
  bool my_writer;
  int my_off;
  float my_mul_op, my_mul_one;
  {
    float dummy[10] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
    float unused;
    const int slot = warp_reduce10(dummy, unused);
    my_writer = !(lane & 1) && slot >= 0 && (DEPTH || slot != 2);
    my_off = slot < 3 ? slot : slot + 1;
    my_mul_op = slot == 0 ? -half_w : slot == 1 ? -half_h : (slot >= 3 && slot <= 5) ? -0.5f : 0.0f;
    my_mul_one = (slot == 2 || slot >= 6) ? 1.0f : 0.0f;
  }
  // the same for the paired reduction of two hits (the first hit's terms,
  // then the second's)
  constexpr int PT = DEPTH ? 10 : 9;
  bool my_writer20, my_second20;
  int my_off20;
  float my_mul_op20, my_mul_one20;
  {
    float dummy[2 * PT];
#pragma unroll
    for (int k = 0; k < 2 * PT; ++k) dummy[k] = 0.0f;
    float unused;
    const int idx = warp_reduce_n<2 * PT>(dummy, unused);
    my_second20 = idx >= PT;
    const int slot = pair_term_slot<DEPTH>(my_second20 ? idx - PT : idx);
    my_writer20 = idx >= 0;
    my_off20 = slot < 3 ? slot : slot + 1;
    my_mul_op20 = slot == 0 ? -half_w : slot == 1 ? -half_h : (slot >= 3 && slot <= 5) ? -0.5f : 0.0f;
    my_mul_one20 = (slot == 2 || slot >= 6) ? 1.0f : 0.0f;
  }
  const float fx = (float)pxi;
  const float bx0 = (float)(__shfl_sync(FULL, pxi, 0)), by0 = (float)(__shfl_sync(FULL, py0, 0));
  const float bx1 = bx0 + 7.0f;

  for (int hi = cta_max; hi > 0; hi -= BATCH) {
    const int lo = max(0, hi - BATCH);
    __syncthreads();
    for (int k = threadIdx.x; k < hi - lo; k += BWD_THREADS) {
      const int id = a.point_list[range.x + lo + k];
      const float4 q0 = __ldg(rec + (size_t)id * 3 + 0);
      const float4 q1 = __ldg(rec + (size_t)id * 3 + 1);
      const float4 q2 = __ldg(rec + (size_t)id * 3 + 2);
      s_id[k] = id;
      s_xy[k] = make_float2(q0.x, q0.y);
      float4 cf = power_coefs(q0.z, q0.w, q1.x);
      cf.w = q1.y;
      s_cf[k] = cf;
      s_con[k] = make_float4(q0.z, q0.w, q1.x, 0.0f);
      s_rgbd[k] = make_float4(q2.x, q2.y, q2.z, q1.z);
      s_box[k] = alpha_box(q0.x, q0.y, q0.z, q0.w, q1.x, q1.y);
      s_el[k] = cull_ellipse(q0.z, q0.w, q1.x, q1.y);
    }
    __syncthreads();
    const int top = min(hi, warp_max);
    // Lanes test staged Gaussians against the warp's two 8x8 halves; the warp
    // visits only the hits below its own maximum, back to front.
    for (int cb = ((top - lo - 1) >> 5) << 5; cb >= 0 && top > lo; cb -= 32) {
      bool h_top, h_bot;
      cull_halves8(cb + lane, top - lo, s_box, s_xy, s_el, bx0, bx1, by0, h_top, h_bot);
      const unsigned m0 = __ballot_sync(FULL, h_top), m2 = __ballot_sync(FULL, h_bot);
      unsigned hits = m0 | m2;
      // The hit at `bit`: the warp's pairs it reaches run back to front; its ten
      // gradient terms land in v.  Returns whether any lane contributed.
      auto eval_hit = [&](int bit, float (&v)[10]) -> bool {
        const int j = cb + bit;
        const int pos = lo + j;
        // a half the Gaussian cannot reach has alpha < 1/255 at every pixel: no state change to skip
        const bool e0 = ((m0 >> bit) & 1u) && pos < px[0].lc0;
        const bool e1 = ((m0 >> bit) & 1u) && pos < px[0].lc1;
        const bool e2 = ((m2 >> bit) & 1u) && pos < px[1].lc0;
        const bool e3 = ((m2 >> bit) & 1u) && pos < px[1].lc1;
        // which pairs the warp runs (warp-uniform; a lane whose pixels do not
        // take the Gaussian gets zero terms and keeps its state)
        const bool P0 = __any_sync(FULL, e0 || e1), P1 = __any_sync(FULL, e2 || e3);
        if (!(P0 || P1)) return false;
        const float2 xy = s_xy[j];
        const float4 cf = s_cf[j];
        const float4 cd = s_rgbd[j];
        const float dx = xy.x - fx;
        float ax, bx;
        column_terms(cf, dx, ax, bx);
        bool c0, c1, contrib;
        BwdSums2 m2;
        if (P0) {
          const PairTerms t0 = bwd_pair_core<DEPTH, GA>(px[0], e0, e1, cf, ax, bx, xy.y, cd, has_bg, c0, c1);
          contrib = c0 || c1;
          sums2_add<DEPTH, true>(m2, t0, px[0]);
          if (P1) {
            const PairTerms t1 = bwd_pair_core<DEPTH, GA>(px[1], e2, e3, cf, ax, bx, xy.y, cd, has_bg, c0, c1);
            contrib = contrib || c0 || c1;
            sums2_add<DEPTH, false>(m2, t1, px[1]);
          }
        } else {
          const PairTerms t1 = bwd_pair_core<DEPTH, GA>(px[1], e2, e3, cf, ax, bx, xy.y, cd, has_bg, c0, c1);
          contrib = c0 || c1;
          sums2_add<DEPTH, true>(m2, t1, px[1]);
        }
        if (!__any_sync(FULL, contrib)) return false;
        BwdSums m;
        sums2_reduce<DEPTH>(m2, m);
        if (!DEPTH) m.ddepth = 0.0f;
        const float4 con = s_con[j];
        const float dxU = dx * m.U;
        v[0] = con.x * dxU + con.y * m.UY;   // x: times -op W/2
        v[1] = con.z * m.UY + con.y * dxU;   // y: times -op H/2
        v[2] = m.ddepth;
        v[3] = dx * dxU;                     // conic a: times -op/2
        v[4] = dx * m.UY;                    // conic b: times -op/2
        v[5] = m.UYY;                        // conic c: times -op/2
        v[6] = m.U;                          // opacity
        v[7] = m.dcol0;
        v[8] = m.dcol1;
        v[9] = m.dcol2;
        return true;
      };
      // Contributing hits are reduced two at a time (one 20-value transpose
      // reduction instead of two 10-value ones); an unpaired last one alone.
      while (hits) {
        const int bitA = 31 - __clz(hits);
        hits &= ~(1u << bitA);
        float vA[10];
        if (!eval_hit(bitA, vA)) continue;
        int bitB = -1;
        float vB[10];
        while (hits) {
          const int bit = 31 - __clz(hits);
          hits &= ~(1u << bit);
          if (eval_hit(bit, vB)) {
            bitB = bit;
            break;
          }
        }
        const int jA = cb + bitA;
        if (bitB >= 0) {
          float v2[2 * PT];
#pragma unroll
          for (int k = 0; k < PT; ++k) {
            v2[k] = vA[pair_term_slot<DEPTH>(k)];
            v2[PT + k] = vB[pair_term_slot<DEPTH>(k)];
          }
          float sum;
          warp_reduce_n<2 * PT>(v2, sum);
          if (my_writer20) {
            const int jj = my_second20 ? cb + bitB : jA;
            const float scale = fmaf(s_cf[jj].w, my_mul_op20, my_mul_one20);
            atomicAdd(a.grad_acc + (size_t)s_id[jj] * GSB_GRAD_FLOATS + my_off20, sum * scale);
          }
        } else {
          float sum;
          warp_reduce10(vA, sum);
          if (my_writer) {
            const float scale = fmaf(s_cf[jA].w, my_mul_op, my_mul_one);
            atomicAdd(a.grad_acc + (size_t)s_id[jA] * GSB_GRAD_FLOATS + my_off, sum * scale);
          }
        }
      }
    }
  }
}

// Backward for grids of few tiles: one 128-thread CTA per tile, each warp an
// 8x8 block, each thread two pixels (rows y, y+4) as one packed pair, culled
// per block (3% faster on an 800x800 view than a test per 8x4 half).  When
// the grid holds fewer tiles than the GPU holds CTAs, the kernel lasts as
// long as its heaviest tile, and four warps per tile finish it sooner than
// two.  DEPTH: compute_depth with a depth gradient
// given; GA: an alpha gradient given.  Without them those terms are exactly
// zero and are not evaluated.
template <bool DEPTH, bool GA>
__global__ void __launch_bounds__(THREADS, 8) render_bwd_tile4_kernel(const gsb_render_bwd_args a, int gx) {
  __shared__ int s_id[BATCH];
  __shared__ float2 s_xy[BATCH];
  __shared__ float4 s_cf[BATCH];    // power coefficients, opacity in .w
  __shared__ float4 s_con[BATCH];   // conic a, b, c
  __shared__ float4 s_rgbd[BATCH];
  __shared__ float4 s_box[BATCH];
  __shared__ float4 s_el[BATCH];
  __shared__ int s_max[THREADS / 32];
  const int tile = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int pxi, py0;
  pixels_of(tile, gx, pxi, py0);
  const int2 range = reinterpret_cast<const int2*>(a.ranges)[tile];
  const int n = range.y - range.x;
  const float4* rec = reinterpret_cast<const float4*>(a.records);
  const long long npix = (long long)a.W * a.H;
  const bool has_bg = a.background[0] != 0.0f || a.background[1] != 0.0f || a.background[2] != 0.0f;

  BwdPair px;
  px.lc0 = px.lc1 = 0;
  float Tf[2], g0[2], g1[2], g2[2], gd[2], ga[2];
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const int py = py0 + 4 * p;
    int lc = 0;
    Tf[p] = g0[p] = g1[p] = g2[p] = gd[p] = ga[p] = 0.0f;
    if (pxi < a.W && py < a.H && n > 0) {
      const long long pix = (long long)py * a.W + pxi;
      lc = a.n_contrib[pix];
      Tf[p] = 1.0f - a.out_alpha[pix];
      g0[p] = a.grad_color[pix];
      g1[p] = a.grad_color[npix + pix];
      g2[p] = a.grad_color[2 * npix + pix];
      if (DEPTH) gd[p] = a.grad_depth[pix];
      if (GA) ga[p] = a.grad_alpha[pix];
    }
    if (p) px.lc1 = lc;
    else px.lc0 = lc;
  }
  px.nfy = make_float2(-(float)py0, -(float)(py0 + 4));
  px.T = make_float2(Tf[0], Tf[1]);
  px.nTf = make_float2(-Tf[0], -Tf[1]);
  px.g0 = make_float2(g0[0], g0[1]);
  px.g1 = make_float2(g1[0], g1[1]);
  px.g2 = make_float2(g2[0], g2[1]);
  px.gd = make_float2(gd[0], gd[1]);
  px.ga = make_float2(ga[0], ga[1]);
  px.bg_dot = make_float2(a.background[0] * g0[0] + a.background[1] * g1[0] + a.background[2] * g2[0],
                          a.background[0] * g0[1] + a.background[1] * g1[1] + a.background[2] * g2[1]);
  px.S = px.adr = px.aar = make_float2(0.0f, 0.0f);
  const int warp_max = __reduce_max_sync(FULL, max(px.lc0, px.lc1));
  if (lane == 0) s_max[warp] = warp_max;
  __syncthreads();
  int cta_max = 0;
#pragma unroll
  for (int w = 0; w < THREADS / 32; ++w) cta_max = max(cta_max, s_max[w]);
  cta_max = min(cta_max, n);  // n_contrib never exceeds the tile's list
  if (cta_max <= 0) return;

  const float half_w = 0.5f * (float)a.W;
  const float half_h = 0.5f * (float)a.H;
  // Which reduced term this lane writes (a lane constant): its accumulator
  // offset and the Gaussian-constant factor op * my_mul_op + my_mul_one
  // (-op W/2 for x, -op H/2 for y, -op/2 for the conic, 1 otherwise).
  bool my_writer;
  int my_off;
  float my_mul_op, my_mul_one;
  {
    float dummy[10] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
    float unused;
    const int slot = warp_reduce10(dummy, unused);
    my_writer = !(lane & 1) && slot >= 0 && (DEPTH || slot != 2);
    my_off = slot < 3 ? slot : slot + 1;
    my_mul_op = slot == 0 ? -half_w : slot == 1 ? -half_h : (slot >= 3 && slot <= 5) ? -0.5f : 0.0f;
    my_mul_one = (slot == 2 || slot >= 6) ? 1.0f : 0.0f;
  }
  // the same for the paired reduction of two hits (the first hit's terms,
  // then the second's)
  constexpr int PT = DEPTH ? 10 : 9;
  bool my_writer20, my_second20;
  int my_off20;
  float my_mul_op20, my_mul_one20;
  {
    float dummy[2 * PT];
#pragma unroll
    for (int k = 0; k < 2 * PT; ++k) dummy[k] = 0.0f;
    float unused;
    const int idx = warp_reduce_n<2 * PT>(dummy, unused);
    my_second20 = idx >= PT;
    const int slot = pair_term_slot<DEPTH>(my_second20 ? idx - PT : idx);
    my_writer20 = idx >= 0;
    my_off20 = slot < 3 ? slot : slot + 1;
    my_mul_op20 = slot == 0 ? -half_w : slot == 1 ? -half_h : (slot >= 3 && slot <= 5) ? -0.5f : 0.0f;
    my_mul_one20 = (slot == 2 || slot >= 6) ? 1.0f : 0.0f;
  }
  const float fx = (float)pxi;
  const float bx0 = (float)(__shfl_sync(FULL, pxi, 0)), by0 = (float)(__shfl_sync(FULL, py0, 0));
  const float bx1 = bx0 + 7.0f;

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
      float4 cf = power_coefs(q0.z, q0.w, q1.x);
      cf.w = q1.y;
      s_cf[k] = cf;
      s_con[k] = make_float4(q0.z, q0.w, q1.x, 0.0f);
      s_rgbd[k] = make_float4(q2.x, q2.y, q2.z, q1.z);
      s_box[k] = alpha_box(q0.x, q0.y, q0.z, q0.w, q1.x, q1.y);
      s_el[k] = cull_ellipse(q0.z, q0.w, q1.x, q1.y);
    }
    __syncthreads();
    const int top = min(hi, warp_max);
    // Lanes test staged Gaussians against the warp's 8x8 block; the warp
    // visits only the hits below its own maximum, back to front.
    for (int cb = ((top - lo - 1) >> 5) << 5; cb >= 0 && top > lo; cb -= 32) {
      // one test over the warp's 8x8 block: both of a lane's pixels lie in
      // it, so a half-block test would only mask pixels the alpha test rejects
      const int g = cb + lane;
      bool hit = false;
      if (g < top - lo) {
        const float4 bb = s_box[g];
        hit = bb.x <= bx1 && bb.y >= bx0 && bb.z <= by0 + 7.0f && bb.w >= by0;
      }
      if (__any_sync(FULL, hit) && hit) hit = ellipse_hits(s_xy[g].x, s_xy[g].y, s_el[g], bx0, bx1, by0, by0 + 7.0f);
      const unsigned top_h = __ballot_sync(FULL, hit), bot_h = top_h;
      unsigned hits = top_h;
      // The hit at `bit`: this lane's pixels that take it run back to front;
      // its ten gradient terms land in v.  Returns whether any lane contributed.
      auto eval_hit = [&](int bit, float (&v)[10]) -> bool {
        const int j = cb + bit;
        const int pos = lo + j;
        BwdSums m = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
        bool contrib = false;
        float dx = 0.0f;
        // a half the Gaussian cannot reach has alpha < 1/255 at every pixel: no state change to skip
        const bool e0 = ((top_h >> bit) & 1u) && pos < px.lc0;
        const bool e1 = ((bot_h >> bit) & 1u) && pos < px.lc1;
        if (e0 || e1) {
          const float2 xy = s_xy[j];
          const float4 cf = s_cf[j];
          const float4 cd = s_rgbd[j];
          dx = xy.x - fx;
          float ax, bx;
          column_terms(cf, dx, ax, bx);
          bool c0, c1;
          bwd_pair<DEPTH, GA>(px, e0, e1, cf, ax, bx, xy.y, cd, has_bg, m, c0, c1);
          contrib = c0 || c1;
        }
        if (!__any_sync(FULL, contrib)) return false;
        const float4 con = s_con[j];
        const float dxU = dx * m.U;
        v[0] = con.x * dxU + con.y * m.UY;   // x: times -op W/2
        v[1] = con.z * m.UY + con.y * dxU;   // y: times -op H/2
        v[2] = m.ddepth;
        v[3] = dx * dxU;                     // conic a: times -op/2
        v[4] = dx * m.UY;                    // conic b: times -op/2
        v[5] = m.UYY;                        // conic c: times -op/2
        v[6] = m.U;                          // opacity
        v[7] = m.dcol0;
        v[8] = m.dcol1;
        v[9] = m.dcol2;
        return true;
      };
      // contributing hits are reduced two at a time, an unpaired last one alone
      while (hits) {
        const int bitA = 31 - __clz(hits);
        hits &= ~(1u << bitA);
        float vA[10];
        if (!eval_hit(bitA, vA)) continue;
        int bitB = -1;
        float vB[10];
        while (hits) {
          const int bit = 31 - __clz(hits);
          hits &= ~(1u << bit);
          if (eval_hit(bit, vB)) {
            bitB = bit;
            break;
          }
        }
        const int jA = cb + bitA;
        if (bitB >= 0) {
          float v2[2 * PT];
#pragma unroll
          for (int k = 0; k < PT; ++k) {
            v2[k] = vA[pair_term_slot<DEPTH>(k)];
            v2[PT + k] = vB[pair_term_slot<DEPTH>(k)];
          }
          float sum;
          warp_reduce_n<2 * PT>(v2, sum);
          if (my_writer20) {
            const int jj = my_second20 ? cb + bitB : jA;
            const float scale = fmaf(s_cf[jj].w, my_mul_op20, my_mul_one20);
            atomicAdd(a.grad_acc + (size_t)s_id[jj] * GSB_GRAD_FLOATS + my_off20, sum * scale);
          }
        } else {
          float sum;
          warp_reduce10(vA, sum);
          if (my_writer) {
            const float scale = fmaf(s_cf[jA].w, my_mul_op, my_mul_one);
            atomicAdd(a.grad_acc + (size_t)s_id[jA] * GSB_GRAD_FLOATS + my_off, sum * scale);
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
  const bool aux = a->top_k > 0;
  if (aux && (!a->gs_per_pixel || !a->weight_per_gs_pixel || !a->x_mu)) {
    set_error("gsb_render_fwd: top_k > 0 needs gs_per_pixel, weight_per_gs_pixel and x_mu");
    return GSB_ERR_INVALID;
  }
  if (aux && a->aux_scratch && (reinterpret_cast<uintptr_t>(a->aux_scratch) & 15)) {
    set_error("gsb_render_fwd: aux_scratch needs 16-byte alignment");
    return GSB_ERR_INVALID;
  }
  if (a->compute_depth)
    aux ? render_fwd_kernel<true, true><<<gx * gy, THREADS, 0, s>>>(*a, gx)
        : render_fwd_kernel<true, false><<<gx * gy, THREADS, 0, s>>>(*a, gx);
  else
    aux ? render_fwd_kernel<false, true><<<gx * gy, THREADS, 0, s>>>(*a, gx)
        : render_fwd_kernel<false, false><<<gx * gy, THREADS, 0, s>>>(*a, gx);
  if (aux && a->aux_scratch) {
    const long long kn = (long long)a->top_k * a->W * a->H;
    flow_aux_split_kernel<<<(unsigned)((kn + 255) / 256), 256, 0, s>>>(
        kn, kn, reinterpret_cast<const float4*>(a->aux_scratch), a->gs_per_pixel, a->weight_per_gs_pixel, a->x_mu);
  }
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
  const bool depth = a->compute_depth && a->grad_depth;
  const bool ga = a->grad_alpha != nullptr;
  const int blocks = gx * gy;
  if (blocks >= BWD_TILE2_MIN_TILES) {
    if (depth && ga)
      render_bwd_tile2_kernel<true, true><<<blocks, BWD_THREADS, 0, s>>>(*a, gx);
    else if (depth)
      render_bwd_tile2_kernel<true, false><<<blocks, BWD_THREADS, 0, s>>>(*a, gx);
    else if (ga)
      render_bwd_tile2_kernel<false, true><<<blocks, BWD_THREADS, 0, s>>>(*a, gx);
    else
      render_bwd_tile2_kernel<false, false><<<blocks, BWD_THREADS, 0, s>>>(*a, gx);
  } else {
    if (depth && ga)
      render_bwd_tile4_kernel<true, true><<<blocks, THREADS, 0, s>>>(*a, gx);
    else if (depth)
      render_bwd_tile4_kernel<true, false><<<blocks, THREADS, 0, s>>>(*a, gx);
    else if (ga)
      render_bwd_tile4_kernel<false, true><<<blocks, THREADS, 0, s>>>(*a, gx);
    else
      render_bwd_tile4_kernel<false, false><<<blocks, THREADS, 0, s>>>(*a, gx);
  }
  return check_launch("render_bwd_kernel");
}
