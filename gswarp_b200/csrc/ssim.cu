// ssim.cu -- fused separable 11x11 SSIM forward and backward.
//
// Restates gswarp's fused_ssim.py: Gaussian window sigma 1.5 (:47-57);
// forward _fwd_h (:461-518) + _fwd_v_train_tiled (:522-638) ('same') or
// _fwd_v_train_valid (:760-828) ('valid'); backward _bwd_h_scalar
// (:831-874) / _bwd_h_scalar_valid (:878-935) + _bwd_v_tiled (:985-1067) /
// _bwd_v (:938-981).  The reference runs each direction as two kernels with
// four (forward) or three (backward) full-size intermediate maps in HBM; here
// each direction is ONE kernel per 32x40 output tile: the input tile plus a
// 5-pixel halo is staged in shared memory, the horizontal pass writes shared
// memory only, and the vertical pass produces the outputs; both passes slide
// their 11-tap windows over values held in registers.  Forward writes
// only what backward needs (dm0, dm1, dm2) plus one partial SSIM sum per CTA;
// a last tiny kernel turns the partial sums into the mean.
//
// Out-of-image taps are zero-filled in shared memory; adding g*0 is exact, so
// this equals the reference's explicit bounds checks.  The 'valid' vertical
// pass pairs symmetric taps g*(top+bottom) as the reference does there.
#include "gsb_common.cuh"

namespace gsb {
namespace {

constexpr int TX = 32, TY = 40;
constexpr int HALO = 5;
constexpr int RX = TX + 2 * HALO;  // 42
constexpr int RY = TY + 2 * HALO;  // 50
constexpr int THREADS = launch::SSIM;
// Register blocking: a thread runs the horizontal pass over RH consecutive
// outputs of one row (its 11-tap windows slide over RH + 10 values held in
// registers) and the vertical pass over RV consecutive outputs of one column,
// so each staged value is read from shared memory about once per thread
// instead of once per tap.  Row strides are odd: the warps' accesses hit 32
// different banks.
constexpr int RH = 8;
constexpr int HSEG = TX / RH;         // row segments: 4
constexpr int H_ITEMS = RY * HSEG;    // 200 horizontal work items
constexpr int RV = 5;
constexpr int VSEG = TY / RV;         // column segments: 8
static_assert(TX * VSEG == THREADS, "one vertical work item per thread");
static_assert(H_ITEMS <= THREADS, "one horizontal work item per thread at most");
constexpr int STAGE_ITERS = (RY * RX + THREADS - 1) / THREADS;  // staged values per thread: 9

__constant__ float GW[11] = {0.001028380123898387f, 0.0075987582094967365f,
                             0.036000773310661316f,  0.10936068743467331f,
                             0.21300552785396576f,   0.26601171493530273f,
                             0.21300552785396576f,   0.10936068743467331f,
                             0.036000773310661316f,  0.0075987582094967365f,
                             0.001028380123898387f};

// WITH_L1 also sums |img1 - img2| over the tile's pixels into
// partials[gridDim.x + blockIdx.x] (the photometric training loss).
template <bool WITH_L1>
__global__ void __launch_bounds__(THREADS) ssim_fwd_kernel(const gsb_ssim_fwd_args a, int tiles_x,
                                                           int tiles_y) {
  __shared__ float2 s_p[RY][RX + 1];      // (img1, img2)
  __shared__ float2 s_h[2][RY][TX + 1];   // horizontal sums: (x, y) and (x^2 + y^2, x y)
  __shared__ float s_red[THREADS / 32];
  __shared__ float s_red_l1[THREADS / 32];
  const int H = a.H, W = a.W;
  const int tile = blockIdx.x;
  const int tx = tile % tiles_x;
  const int ty = (tile / tiles_x) % tiles_y;
  const int plane = tile / (tiles_x * tiles_y);
  const int x0 = tx * TX, y0 = ty * TY;
  const size_t pbase = (size_t)plane * H * W;
  const float* img1 = a.img1 + pbase;
  const float* img2 = a.img2 + pbase;

  // Staging: all of a thread's loads are issued before its shared-memory
  // stores, so their latencies overlap instead of adding up.
  {
    float v1[STAGE_ITERS], v2[STAGE_ITERS];
#pragma unroll
    for (int it = 0; it < STAGE_ITERS; ++it) {
      const int i = threadIdx.x + it * THREADS;
      const int r = i / RX, c = i % RX;
      const int gy = y0 - HALO + r, gxp = x0 - HALO + c;
      v1[it] = v2[it] = 0.0f;
      if (i < RY * RX && gy >= 0 && gy < H && gxp >= 0 && gxp < W) {
        v1[it] = __ldg(img1 + (size_t)gy * W + gxp);
        v2[it] = __ldg(img2 + (size_t)gy * W + gxp);
      }
    }
#pragma unroll
    for (int it = 0; it < STAGE_ITERS; ++it) {
      const int i = threadIdx.x + it * THREADS;
      if (i < RY * RX) s_p[i / RX][i % RX] = make_float2(v1[it], v2[it]);
    }
  }
  __syncthreads();
  // Horizontal pass (fused_ssim.py:477-511): symmetric tap pairs, then centre.
  // The four filtered quantities go as two packed f32x2 pairs, (x, y) and
  // (x^2 + y^2, x y): per component the same taps, weights and fused
  // multiply-adds as four scalar chains.  Consecutive lanes take
  // consecutive rows (odd row stride: conflict-free 8-byte accesses).
  if (threadIdx.x < H_ITEMS) {
    const int r = threadIdx.x % RY, c0 = (threadIdx.x / RY) * RH;
    // x^2 + y^2 and x*y once per window value (each is used by up to 11 outputs)
    float2 p[RH + 10], sq[RH + 10];
#pragma unroll
    for (int q = 0; q < RH + 10; ++q) {
      p[q] = s_p[r][c0 + q];
      sq[q] = make_float2(p[q].x * p[q].x + p[q].y * p[q].y, p[q].x * p[q].y);
    }
#pragma unroll
    for (int j = 0; j < RH; ++j) {
      float2 a01 = make_float2(0.0f, 0.0f), a23 = a01;
#pragma unroll
      for (int k = 0; k < 5; ++k) {
        const float2 g = make_float2(GW[k], GW[k]);
        const int l = j + k, rr = j + 10 - k;
        a01 = __ffma2_rn(g, __fadd2_rn(p[l], p[rr]), a01);
        a23 = __ffma2_rn(g, __fadd2_rn(sq[l], sq[rr]), a23);
      }
      const float2 g5 = make_float2(GW[5], GW[5]);
      s_h[0][r][c0 + j] = __ffma2_rn(g5, p[j + 5], a01);
      s_h[1][r][c0 + j] = __ffma2_rn(g5, sq[j + 5], a23);
    }
  }
  __syncthreads();
  // Vertical pass: column c, rows r0 .. r0 + RV - 1 of the tile.
  const int c = threadIdx.x % TX, r0 = (threadIdx.x / TX) * RV;
  float s4[RV][4];
#pragma unroll
  for (int m = 0; m < 2; ++m) {
    float2 w[RV + 10];
#pragma unroll
    for (int q = 0; q < RV + 10; ++q) w[q] = s_h[m][r0 + q][c];
#pragma unroll
    for (int j = 0; j < RV; ++j) {
      float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int k = 0; k < 5; ++k) {
        const float2 g = make_float2(GW[k], GW[k]);
        const float2 top = w[j + k], bot = w[j + 10 - k];
        if (a.valid) {
          acc = __ffma2_rn(g, __fadd2_rn(top, bot), acc);
        } else {
          acc = __ffma2_rn(g, top, acc);
          acc = __ffma2_rn(g, bot, acc);
        }
      }
      acc = __ffma2_rn(make_float2(GW[5], GW[5]), w[j + 5], acc);
      s4[j][2 * m] = acc.x;
      s4[j][2 * m + 1] = acc.y;
    }
  }
  float local_sum = 0.0f, local_l1 = 0.0f;
  const size_t npix = (size_t)a.B * a.C * H * W;
  const int gxp = x0 + c;
#pragma unroll
  for (int j = 0; j < RV; ++j) {
    const int gy = y0 + r0 + j;
    if (gy >= H || gxp >= W) continue;
    if (a.valid && (gy < 5 || gy >= H - 5 || gxp < 5 || gxp >= W - 5)) continue;
    const float mu1 = s4[j][0], mu2 = s4[j][1];
    const float mu1_sq = mu1 * mu1, mu2_sq = mu2 * mu2, mu1mu2 = mu1 * mu2;
    const float Av = mu1_sq + mu2_sq + a.C1;
    const float Bv = s4[j][2] - mu1_sq - mu2_sq + a.C2;
    const float Cv = 2.0f * mu1mu2 + a.C1;
    const float Dv = 2.0f * (s4[j][3] - mu1mu2) + a.C2;
    const float rA = 1.0f / Av, rB = 1.0f / Bv, rAB = rA * rB;
    const float m = Cv * Dv * rAB;
    local_sum += m;
    if (WITH_L1) {
      const float2 v = s_p[r0 + j + HALO][c + HALO];
      local_l1 += fabsf(v.x - v.y);
    }
    if (a.dm) {
      const size_t o = pbase + (size_t)gy * W + gxp;
      a.dm[o] = 2.0f * (mu2 * (Dv - Cv) * rAB + mu1 * m * (rB - rA));
      a.dm[npix + o] = -m * rB;
      a.dm[2 * npix + o] = 2.0f * Cv * rAB;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) local_sum += __shfl_xor_sync(0xffffffffu, local_sum, o);
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = local_sum;
  if (WITH_L1) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) local_l1 += __shfl_xor_sync(0xffffffffu, local_l1, o);
    if ((threadIdx.x & 31) == 0) s_red_l1[threadIdx.x >> 5] = local_l1;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
#pragma unroll
    for (int w = 0; w < THREADS / 32; ++w) t += s_red[w];
    a.partials[blockIdx.x] = t;
    if (WITH_L1) {
      float u = 0.0f;
#pragma unroll
      for (int w = 0; w < THREADS / 32; ++w) u += s_red_l1[w];
      a.partials[gridDim.x + blockIdx.x] = u;
    }
  }
}

__global__ void __launch_bounds__(1024) ssim_mean_kernel(const float* __restrict__ partials, int n,
                                                         double inv_count, float* __restrict__ loss) {
  __shared__ double s[32];
  double acc = 0.0;
  for (int i = threadIdx.x; i < n; i += 1024) acc += (double)partials[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) s[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < 32; ++w) t += s[w];
    *loss = (float)(t * inv_count);
  }
}

// upstream_host != 0 replaces the device upstream scalar (the photometric
// loss passes -w_ssim); WITH_L1 adds l1_scale * sign(img1 - img2).
template <bool WITH_L1>
__global__ void __launch_bounds__(THREADS) ssim_bwd_kernel(const gsb_ssim_bwd_args a, int tiles_x,
                                                           int tiles_y, float inv_n, float upstream_host,
                                                           float l1_scale) {
  // maps 0 and 1 as packed f32x2 pairs, map 2 alone
  __shared__ float2 s_dm01[RY][RX + 1];
  __shared__ float s_dm2[RY][RX + 1];
  __shared__ float2 s_t01[RY][TX + 1];
  __shared__ float s_t2[RY][TX + 1];
  const int H = a.H, W = a.W;
  const int tile = blockIdx.x;
  const int tx = tile % tiles_x;
  const int ty = (tile / tiles_x) % tiles_y;
  const int plane = tile / (tiles_x * tiles_y);
  const int x0 = tx * TX, y0 = ty * TY;
  const size_t pbase = (size_t)plane * H * W;
  const size_t npix = (size_t)a.B * a.C * H * W;
  const float scale = inv_n * (WITH_L1 ? upstream_host : a.upstream[0]);
  const int lo_y = a.valid ? 5 : 0, hi_y = a.valid ? H - 5 : H;
  const int lo_x = a.valid ? 5 : 0, hi_x = a.valid ? W - 5 : W;
  {
    float d[3][STAGE_ITERS];
#pragma unroll
    for (int it = 0; it < STAGE_ITERS; ++it) {
      const int i = threadIdx.x + it * THREADS;
      const int r = i / RX, c = i % RX;
      const int gy = y0 - HALO + r, gxp = x0 - HALO + c;
      d[0][it] = d[1][it] = d[2][it] = 0.0f;
      if (i < RY * RX && gy >= lo_y && gy < hi_y && gxp >= lo_x && gxp < hi_x) {
        const size_t o = pbase + (size_t)gy * W + gxp;
        d[0][it] = __ldg(a.dm + o);
        d[1][it] = __ldg(a.dm + npix + o);
        d[2][it] = __ldg(a.dm + 2 * npix + o);
      }
    }
#pragma unroll
    for (int it = 0; it < STAGE_ITERS; ++it) {
      const int i = threadIdx.x + it * THREADS;
      if (i < RY * RX) {
        s_dm01[i / RX][i % RX] = make_float2(d[0][it], d[1][it]);
        s_dm2[i / RX][i % RX] = d[2][it];
      }
    }
  }
  __syncthreads();
  // Horizontal pass of dm * (upstream / N) (fused_ssim.py:844-868): maps 0
  // and 1 as one packed f32x2 chain (per component the scalar chain's
  // fused multiply-adds), then map 2.  Consecutive lanes take
  // consecutive rows.
  if (threadIdx.x < H_ITEMS) {
    const int r = threadIdx.x % RY, c0 = (threadIdx.x / RY) * RH;
    {
      float2 dv[RH + 10];
#pragma unroll
      for (int q = 0; q < RH + 10; ++q) dv[q] = s_dm01[r][c0 + q];
#pragma unroll
      for (int j = 0; j < RH; ++j) {
        float2 t = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int k = 0; k < 5; ++k) {
          const float gs = GW[k] * scale;
          const float2 g = make_float2(gs, gs);
          t = __ffma2_rn(g, dv[j + k], t);
          t = __ffma2_rn(g, dv[j + 10 - k], t);
        }
        const float g5 = GW[5] * scale;
        s_t01[r][c0 + j] = __ffma2_rn(make_float2(g5, g5), dv[j + 5], t);
      }
    }
    {
      float dv[RH + 10];
#pragma unroll
      for (int q = 0; q < RH + 10; ++q) dv[q] = s_dm2[r][c0 + q];
#pragma unroll
      for (int j = 0; j < RH; ++j) {
        float t = 0.0f;
#pragma unroll
        for (int k = 0; k < 5; ++k) {
          const float gs = GW[k] * scale;
          t += gs * dv[j + k];
          t += gs * dv[j + 10 - k];
        }
        t += GW[5] * scale * dv[j + 5];
        s_t2[r][c0 + j] = t;
      }
    }
  }
  __syncthreads();
  const int c = threadIdx.x % TX, r0 = (threadIdx.x / TX) * RV;
  float acc3[RV][3];
  {
    float2 w[RV + 10];
#pragma unroll
    for (int q = 0; q < RV + 10; ++q) w[q] = s_t01[r0 + q][c];
#pragma unroll
    for (int j = 0; j < RV; ++j) {
      float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int k = 0; k < 5; ++k) {
        const float2 g = make_float2(GW[k], GW[k]);
        acc = __ffma2_rn(g, w[j + k], acc);
        acc = __ffma2_rn(g, w[j + 10 - k], acc);
      }
      acc = __ffma2_rn(make_float2(GW[5], GW[5]), w[j + 5], acc);
      acc3[j][0] = acc.x;
      acc3[j][1] = acc.y;
    }
  }
  {
    float w[RV + 10];
#pragma unroll
    for (int q = 0; q < RV + 10; ++q) w[q] = s_t2[r0 + q][c];
#pragma unroll
    for (int j = 0; j < RV; ++j) {
      float acc = 0.0f;
#pragma unroll
      for (int k = 0; k < 5; ++k) {
        const float g = GW[k];
        acc += g * w[j + k];
        acc += g * w[j + 10 - k];
      }
      acc += GW[5] * w[j + 5];
      acc3[j][2] = acc;
    }
  }
  const int gxp = x0 + c;
#pragma unroll
  for (int j = 0; j < RV; ++j) {
    const int gy = y0 + r0 + j;
    if (gy >= H || gxp >= W) continue;
    const size_t o = pbase + (size_t)gy * W + gxp;
    const float x1 = __ldg(a.img1 + o), x2 = __ldg(a.img2 + o);
    float gv = acc3[j][0] + 2.0f * x1 * acc3[j][1] + x2 * acc3[j][2];
    if (WITH_L1) {
      const float d = x1 - x2;
      gv = gv + (d > 0.0f ? l1_scale : (d < 0.0f ? -l1_scale : 0.0f));
    }
    a.grad_img1[o] = gv;
  }
}

// Photometric loss mean: partials[0,n) hold SSIM sums, [n,2n) |d| sums.
__global__ void __launch_bounds__(1024) photo_mean_kernel(const float* __restrict__ partials, int n,
                                                          double inv_count, float w_l1, float w_ssim,
                                                          float* __restrict__ out) {
  __shared__ double s[2][32];
  double acc_s = 0.0, acc_l = 0.0;
  for (int i = threadIdx.x; i < n; i += 1024) {
    acc_s += (double)partials[i];
    acc_l += (double)partials[n + i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    acc_s += __shfl_xor_sync(0xffffffffu, acc_s, o);
    acc_l += __shfl_xor_sync(0xffffffffu, acc_l, o);
  }
  if ((threadIdx.x & 31) == 0) {
    s[0][threadIdx.x >> 5] = acc_s;
    s[1][threadIdx.x >> 5] = acc_l;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double ts = 0.0, tl = 0.0;
    for (int w = 0; w < 32; ++w) {
      ts += s[0][w];
      tl += s[1][w];
    }
    const double ssim = ts * inv_count, l1 = tl * inv_count;
    out[0] = (float)((double)w_l1 * l1 + (double)w_ssim * (1.0 - ssim));
    out[1] = (float)l1;
    out[2] = (float)ssim;
  }
}

inline void tiles_of(int H, int W, int& tx, int& ty) {
  tx = div_up(W, TX);
  ty = div_up(H, TY);
}

}  // namespace
}  // namespace gsb

using namespace gsb;

GSB_EXPORT int gsb_ssim_partials_count(int B, int C, int H, int W) {
  int tx, ty;
  tiles_of(H, W, tx, ty);
  return B * C * tx * ty;
}

GSB_EXPORT int gsb_ssim_fwd(const gsb_ssim_fwd_args* a, void* stream) {
  if (!a || a->B <= 0 || a->C <= 0 || a->H <= 0 || a->W <= 0 || !a->img1 || !a->img2 ||
      !a->partials || !a->loss) {
    set_error("gsb_ssim_fwd: invalid arguments");
    return GSB_ERR_INVALID;
  }
  if (a->valid && (a->H < 11 || a->W < 11)) {
    set_error("gsb_ssim_fwd: padding='valid' requires image height and width of at least 11");
    return GSB_ERR_INVALID;
  }
  int tx, ty;
  tiles_of(a->H, a->W, tx, ty);
  const int blocks = a->B * a->C * tx * ty;
  cudaStream_t s = (cudaStream_t)stream;
  ssim_fwd_kernel<false><<<blocks, THREADS, 0, s>>>(*a, tx, ty);
  const double count = a->valid ? (double)a->B * a->C * (a->H - 10) * (a->W - 10)
                                 : (double)a->B * a->C * a->H * a->W;
  ssim_mean_kernel<<<1, 1024, 0, s>>>(a->partials, blocks, 1.0 / count, a->loss);
  return check_launch("ssim_fwd_kernel");
}

GSB_EXPORT int gsb_ssim_bwd(const gsb_ssim_bwd_args* a, void* stream) {
  if (!a || a->B <= 0 || a->C <= 0 || a->H <= 0 || a->W <= 0 || !a->img1 || !a->img2 ||
      !a->dm || !a->upstream || !a->grad_img1) {
    set_error("gsb_ssim_bwd: invalid arguments");
    return GSB_ERR_INVALID;
  }
  int tx, ty;
  tiles_of(a->H, a->W, tx, ty);
  const double count = a->valid ? (double)a->B * a->C * (a->H - 10) * (a->W - 10)
                                 : (double)a->B * a->C * a->H * a->W;
  const float inv_n = (float)(1.0 / count);
  ssim_bwd_kernel<false><<<a->B * a->C * tx * ty, THREADS, 0, (cudaStream_t)stream>>>(*a, tx, ty, inv_n,
                                                                                      0.0f, 0.0f);
  return check_launch("ssim_bwd_kernel");
}

// ---------------------------------------------------------------------------
// Photometric training loss  L = w_l1 * mean|img - target|
//                               + w_ssim * (1 - SSIM(img, target))
// ('same' padding), the loss the reference's SSIM documentation pairs its
// fused SSIM with (docs/ssim.md:22, :91).  The L1 term rides on the SSIM
// kernels' tile loads: forward adds one |d| partial per tile, backward adds
// l1_scale * sign(d) to the SSIM gradient, so the whole loss costs the same
// two image passes as SSIM alone.
// ---------------------------------------------------------------------------
GSB_EXPORT int gsb_photo_loss_fwd(const gsb_photo_loss_fwd_args* a, void* stream) {
  if (!a || a->B <= 0 || a->C <= 0 || a->H <= 0 || a->W <= 0 || !a->img || !a->target || !a->dm ||
      !a->partials || !a->loss_out) {
    set_error("gsb_photo_loss_fwd: invalid arguments");
    return GSB_ERR_INVALID;
  }
  int tx, ty;
  tiles_of(a->H, a->W, tx, ty);
  const int blocks = a->B * a->C * tx * ty;
  gsb_ssim_fwd_args f{};
  f.B = a->B;
  f.C = a->C;
  f.H = a->H;
  f.W = a->W;
  f.valid = 0;
  f.C1 = a->C1;
  f.C2 = a->C2;
  f.img1 = a->img;
  f.img2 = a->target;
  f.dm = a->dm;
  f.partials = a->partials;
  f.loss = a->loss_out;
  cudaStream_t s = (cudaStream_t)stream;
  ssim_fwd_kernel<true><<<blocks, THREADS, 0, s>>>(f, tx, ty);
  const double count = (double)a->B * a->C * a->H * a->W;
  photo_mean_kernel<<<1, 1024, 0, s>>>(a->partials, blocks, 1.0 / count, a->w_l1, a->w_ssim, a->loss_out);
  return check_launch("gsb_photo_loss_fwd");
}

GSB_EXPORT int gsb_photo_loss_bwd(const gsb_photo_loss_bwd_args* a, void* stream) {
  if (!a || a->B <= 0 || a->C <= 0 || a->H <= 0 || a->W <= 0 || !a->img || !a->target || !a->dm ||
      !a->grad_img) {
    set_error("gsb_photo_loss_bwd: invalid arguments");
    return GSB_ERR_INVALID;
  }
  int tx, ty;
  tiles_of(a->H, a->W, tx, ty);
  const double count = (double)a->B * a->C * a->H * a->W;
  const float inv_n = (float)(1.0 / count);
  gsb_ssim_bwd_args b{};
  b.B = a->B;
  b.C = a->C;
  b.H = a->H;
  b.W = a->W;
  b.valid = 0;
  b.img1 = a->img;
  b.img2 = a->target;
  b.dm = a->dm;
  b.upstream = nullptr;
  b.grad_img1 = a->grad_img;
  // Same float products as autograd forms for the two terms:
  // SSIM: inv_n * (-w_ssim * upstream); L1: (w_l1 * upstream) * inv_n.
  const float ssim_up = -(a->w_ssim * a->upstream);
  const float l1_scale = (a->w_l1 * a->upstream) * inv_n;
  ssim_bwd_kernel<true><<<a->B * a->C * tx * ty, THREADS, 0, (cudaStream_t)stream>>>(b, tx, ty, inv_n,
                                                                                     ssim_up, l1_scale);
  return check_launch("gsb_photo_loss_bwd");
}

// ---------------------------------------------------------------------------
// Allocation-free SSIM forward.
//
// Some callers cannot hand this library a workspace: a host process whose
// device memory is reserved up front by another allocator (a framework's
// caching pool that owns the whole device), a plain C / FFI caller with no
// device allocator of its own, or a latency-critical loop in which a
// cudaMalloc/cudaFree round trip (cudaFree synchronizes the device) is not
// acceptable.  This entry point computes the same mean SSIM (and, if `dm` is
// given, the same dm maps) as gsb_ssim_fwd but keeps its only scratch -- one
// partial sum per 32x40 output tile -- in a fixed device array that lives in
// this library for as long as it is loaded (256 KiB on every GPU that loads
// it), so it allocates nothing.
//
// Limits and sharing rules:
//  * at most GSB_SSIM_NOALLOC_MAX_PARTIALS tiles, i.e. B*C*ceil(H/40)*
//    ceil(W/32) <= 65536 (four 3x1080x1920 images need 19,440); larger
//    inputs are rejected with GSB_ERR_INVALID;
//  * every call on a device shares the one array and it keeps the last
//    call's partial sums; each call writes every slot it later reads, so
//    nothing has to start at zero, but two calls whose kernels overlap on
//    the GPU (different streams without ordering) race on the array;
//  * the array's device address is looked up once per device and CUDA
//    context, on the first call made with that device current (and again
//    after the context is replaced, e.g. by cudaDeviceReset); make the first
//    call on a device before any stream capture begins.
// ---------------------------------------------------------------------------
#include <cuda.h>

#include <mutex>

namespace gsb {
namespace {
constexpr int NOALLOC_MAX_PARTIALS = GSB_SSIM_NOALLOC_MAX_PARTIALS;
static __device__ __align__(256) float g_noalloc_partials[NOALLOC_MAX_PARTIALS];
constexpr int NOALLOC_MAX_DEVICES = 64;
struct NoallocSlot {
  unsigned long long ctx_id;  // context the address belongs to (0: unknown)
  float* ptr;
};
NoallocSlot g_noalloc_slot[NOALLOC_MAX_DEVICES] = {};
std::mutex g_noalloc_mutex;

// Unique id of the calling thread's current CUDA context (driver
// cuCtxGetCurrent + cuCtxGetId, fetched through the runtime so the library
// does not link libcuda); 0 when it cannot be told, in which case the
// address is looked up again on every call.
unsigned long long current_context_id() {
  using GetCurrent = CUresult (*)(CUcontext*);
  using GetId = CUresult (*)(CUcontext, unsigned long long*);
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  static bool resolved = false;
  if (!resolved) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = (GetCurrent)f;
    f = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = (GetId)f;
    resolved = true;
  }
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS)
    return 0;
  return id;
}

// Device address of the fixed scratch array on the current device.
int noalloc_scratch(float** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= NOALLOC_MAX_DEVICES) {
    set_error("gsb_ssim_fwd_noalloc: no usable current device (%s)", cudaGetErrorString(e));
    return GSB_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  NoallocSlot& slot = g_noalloc_slot[dev];
  const unsigned long long ctx = current_context_id();
  if (!slot.ptr || ctx == 0 || ctx != slot.ctx_id) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_partials);
    if (e != cudaSuccess || !p) {
      set_error("gsb_ssim_fwd_noalloc: cudaGetSymbolAddress failed (%s)", cudaGetErrorString(e));
      slot = NoallocSlot{};
      return GSB_ERR_CUDA;
    }
    slot.ptr = (float*)p;
    // the lookup makes the device's context current if it was not yet
    slot.ctx_id = ctx ? ctx : current_context_id();
  }
  *out = slot.ptr;
  return GSB_OK;
}
}  // namespace
}  // namespace gsb

GSB_EXPORT int gsb_ssim_fwd_noalloc(int B, int C, int H, int W, int valid, float C1, float C2,
                                    const float* img1, const float* img2, float* dm, float* loss,
                                    void* stream) {
  if (B <= 0 || C <= 0 || H <= 0 || W <= 0 || !img1 || !img2 || !loss) {
    set_error("gsb_ssim_fwd_noalloc: invalid arguments");
    return GSB_ERR_INVALID;
  }
  if (valid && (H < 11 || W < 11)) {
    set_error("gsb_ssim_fwd_noalloc: padding='valid' requires image height and width of at least 11");
    return GSB_ERR_INVALID;
  }
  int tx, ty;
  tiles_of(H, W, tx, ty);
  const long long blocks = (long long)B * C * tx * ty;
  if (blocks > NOALLOC_MAX_PARTIALS) {
    set_error("gsb_ssim_fwd_noalloc: %lld output tiles exceed the fixed scratch of %d "
              "(B*C*ceil(H/40)*ceil(W/32) must be <= %d); use gsb_ssim_fwd with a workspace",
              blocks, NOALLOC_MAX_PARTIALS, NOALLOC_MAX_PARTIALS);
    return GSB_ERR_INVALID;
  }
  float* partials = nullptr;
  const int st = noalloc_scratch(&partials);
  if (st != GSB_OK) return st;
  gsb_ssim_fwd_args a{};
  a.B = B;
  a.C = C;
  a.H = H;
  a.W = W;
  a.valid = valid;
  a.C1 = C1;
  a.C2 = C2;
  a.img1 = img1;
  a.img2 = img2;
  a.dm = dm;
  a.partials = partials;
  a.loss = loss;
  cudaStream_t s = (cudaStream_t)stream;
  ssim_fwd_kernel<false><<<(int)blocks, THREADS, 0, s>>>(a, tx, ty);
  const double count = valid ? (double)B * C * (H - 10) * (W - 10) : (double)B * C * H * W;
  ssim_mean_kernel<<<1, 1024, 0, s>>>(partials, (int)blocks, 1.0 / count, loss);
  return check_launch("gsb_ssim_fwd_noalloc");
}
