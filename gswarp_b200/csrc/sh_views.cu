// sh_views.cu -- SH backward over the views of a data-parallel step
// (gsb_sh_backward_views).
//
// Every view of a step renders the same Gaussians, so the views' colour
// gradients (gsb_preprocess_bwd with grad_colors_clamped, one (P,3) plane per
// view) become the SH gradient and the view-direction term of the means
// gradient in one pass after the last view: each SH row is read once per
// step instead of once per view, and the SH gradient is stored once instead
// of read-modified-written per view.
//
// Math: the SH backward of backward_kernels.py:297-536, restated.  With
// d = (mean - campos) / |mean - campos| and colour_c = sum_k sh[k][c] Y_k(d),
//   dL/dsh[k][c] = Y_k(d) g_c
//   dL/dd        = sum_k t_k dY_k/dd,   t_k = sum_c g_c sh[k][c]
// and dL/dmean is the normalisation's Jacobian applied to dL/dd.  The
// channels are contracted first (t_k), so every basis derivative is applied
// once rather than once per channel.  Views are summed in view order from
// zero.  Compiled with FMA contraction: equal to the per-view SH backward
// within float rounding.
#include "gsb_common.cuh"
#include "gsb_shrows.cuh"

namespace gsb {
namespace {

// Real SH normalisation constants, degrees 0-3.
constexpr float C0 = 0.28209479177387814f;
constexpr float C1 = 0.4886025119029199f;
constexpr float C2_0 = 1.0925484305920792f, C2_1 = -1.0925484305920792f, C2_2 = 0.31539156525252005f,
                C2_3 = -1.0925484305920792f, C2_4 = 0.5462742152960396f;
constexpr float C3_0 = -0.5900435899266435f, C3_1 = 2.890611442640554f, C3_2 = -0.4570457994644658f,
                C3_3 = 0.3731763325901154f, C3_4 = -0.4570457994644658f, C3_5 = 1.445305721320277f,
                C3_6 = -0.5900435899266435f;

constexpr int SHV_THREADS = launch::SH_BACKWARD_VIEWS;
constexpr int SHV_ROW_F = 49;  // 48 floats padded: per-thread scalar reads of a warp hit 32 banks

// Adds one view's contribution: accum[3k+c] += Y_k g_c for the USED
// coefficients the degree uses, and returns dL/dmean.
template <int USED>
__device__ __forceinline__ void sh_view_grad(const float* row, const float mean[3], const float cam[3],
                                             const float g[3], float (&accum)[48], float gmean[3]) {
  constexpr int used = USED;
  const float vx = mean[0] - cam[0], vy = mean[1] - cam[1], vz = mean[2] - cam[2];
  const float sum2 = vx * vx + vy * vy + vz * vz;
  // 1/|v| (rsqrt: within 2 ulp); |v| is clamped at 1e-10 as the reference clamps |v|^2 at 1e-20
  const float inv_len = rsqrtf(fmx(sum2, 1.0e-20f));
  const float x = vx * inv_len, y = vy * inv_len, z = vz * inv_len;
  float Y[16], t[16];
  Y[0] = C0;
  Y[1] = -C1 * y;
  Y[2] = C1 * z;
  Y[3] = -C1 * x;
  const float xx = x * x, yy = y * y, zz = z * z, xy = x * y, yz = y * z, xz = x * z;
  Y[4] = C2_0 * xy;
  Y[5] = C2_1 * yz;
  Y[6] = C2_2 * (2.0f * zz - xx - yy);
  Y[7] = C2_3 * xz;
  Y[8] = C2_4 * (xx - yy);
  Y[9] = C3_0 * y * (3.0f * xx - yy);
  Y[10] = C3_1 * xy * z;
  Y[11] = C3_2 * y * (4.0f * zz - xx - yy);
  Y[12] = C3_3 * z * (2.0f * zz - 3.0f * xx - 3.0f * yy);
  Y[13] = C3_4 * x * (4.0f * zz - xx - yy);
  Y[14] = C3_5 * z * (xx - yy);
  Y[15] = C3_6 * x * (xx - 3.0f * yy);
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    t[k] = 0.0f;
    if (k < used) {
      const float s0 = row[3 * k], s1 = row[3 * k + 1], s2 = row[3 * k + 2];
      t[k] = g[0] * s0 + g[1] * s1 + g[2] * s2;
#pragma unroll
      for (int c = 0; c < 3; ++c) accum[3 * k + c] += Y[k] * g[c];
    }
  }
  // dL/dd; t_k = 0 above the degree, so every term can be summed
  float dx = -C1 * t[3], dy = -C1 * t[1], dz = C1 * t[2];
  dx += C2_0 * y * t[4] - 2.0f * C2_2 * x * t[6] + C2_3 * z * t[7] + 2.0f * C2_4 * x * t[8];
  dy += C2_0 * x * t[4] + C2_1 * z * t[5] - 2.0f * C2_2 * y * t[6] - 2.0f * C2_4 * y * t[8];
  dz += C2_1 * y * t[5] + 4.0f * C2_2 * z * t[6] + C2_3 * x * t[7];
  dx += 6.0f * C3_0 * xy * t[9] + C3_1 * yz * t[10] - 2.0f * C3_2 * xy * t[11] - 6.0f * C3_3 * xz * t[12] +
        C3_4 * (4.0f * zz - 3.0f * xx - yy) * t[13] + 2.0f * C3_5 * xz * t[14] + 3.0f * C3_6 * (xx - yy) * t[15];
  dy += 3.0f * C3_0 * (xx - yy) * t[9] + C3_1 * xz * t[10] + C3_2 * (4.0f * zz - xx - 3.0f * yy) * t[11] -
        6.0f * C3_3 * yz * t[12] - 2.0f * C3_4 * xy * t[13] - 2.0f * C3_5 * yz * t[14] - 6.0f * C3_6 * xy * t[15];
  dz += C3_1 * xy * t[10] + 8.0f * C3_2 * yz * t[11] + 3.0f * C3_3 * (2.0f * zz - xx - yy) * t[12] +
        8.0f * C3_4 * xz * t[13] + C3_5 * (xx - yy) * t[14];
  // through the normalisation (math_kernels.py:89-97): (|v|^2 g - v (v.g)) / |v|^3
  const float inv32 = inv_len * inv_len * inv_len;
  const float vg = vx * dx + vy * dy + vz * dz;
  gmean[0] = (sum2 * dx - vx * vg) * inv32;
  gmean[1] = (sum2 * dy - vy * vg) * inv32;
  gmean[2] = (sum2 * dz - vz * vg) * inv32;
}

// One thread per Gaussian, 128-thread CTAs.  Each warp first stages the
// colour gradients of its 32 Gaussians for up to VCHUNK views in shared
// memory (per view one contiguous span of 96 floats: coalesced, independent
// loads, entries reset to zero as they are read), then the SH rows of the
// Gaussians with a non-zero gradient (coalesced), so the per-view loop runs
// from shared memory only.  The (K,3) gradient row is summed in registers
// and leaves through shared memory with coalesced stores.
constexpr int VCHUNK = 8;
constexpr int WARPS = SHV_THREADS / 32;

template <int USED>
__global__ void __launch_bounds__(SHV_THREADS, 4) sh_backward_views_kernel(const gsb_sh_views_args a) {
  __shared__ float s_rows[SHV_THREADS * SHV_ROW_F];
  __shared__ float s_g[WARPS][VCHUNK][96];
  // Gaussians [first, last): the warps start at `first` (a multiple of 32
  // is not required: rows are addressed from the warp's own base).
  const int first = a.begin, last = a.end;
  const int idx = first + blockIdx.x * blockDim.x + threadIdx.x;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int base = idx - lane;
  if (base >= last) return;  // whole warp past the range
  const bool live = idx < last;
  const int K = a.sh_coeffs, RF = K * 3;
  const int rows_here = min(32, last - base);
  const int n_here = rows_here * 3;
  float* rows = s_rows + warp * SHV_ROW_F * 32;
  const size_t plane = (size_t)a.P * 3;
  float(*sg)[96] = s_g[warp];
  // The SH rows are loaded only after the colour gradients are staged, and
  // the means gradient is read back at the end: their lines are requested
  // now (the warp's rows are one contiguous span).
  {
    const float* span = a.sh + (size_t)base * RF;
    const int nf = rows_here * RF;
    // one address per 128 bytes and the span's last float (a misaligned
    // start leaves a partial line at the end); all inside the span
    for (int l = lane; l * 32 < nf; l += 32) asm volatile("prefetch.global.L2 [%0];" ::"l"(span + (size_t)l * 32));
    if (lane == 31) asm volatile("prefetch.global.L2 [%0];" ::"l"(span + (nf - 1)));
    if (live) {
      asm volatile("prefetch.global.L1 [%0];" ::"l"(a.means + (size_t)idx * 3));
      asm volatile("prefetch.global.L1 [%0];" ::"l"(a.grad_means3d + (size_t)idx * 3));
    }
  }

  // One chunk of views' colour gradients into shared memory.  Every load is
  // issued before any reset store: the compiler cannot tell the views' planes
  // apart, so a load placed after a store would wait for it.
  auto stage = [&](int v0, int nv) {
    float val[VCHUNK][3];
#pragma unroll
    for (int v = 0; v < VCHUNK; ++v) {
      const float* src = a.grad_colors + (size_t)(v0 + v) * plane + (size_t)base * 3;
#pragma unroll
      for (int q = 0; q < 3; ++q) {
        const int j = lane + 32 * q;
        val[v][q] = (v < nv && j < n_here) ? src[j] : 0.0f;
      }
    }
#pragma unroll
    for (int v = 0; v < VCHUNK; ++v) {
      float* src = a.grad_colors + (size_t)(v0 + v) * plane + (size_t)base * 3;
#pragma unroll
      for (int q = 0; q < 3; ++q) {
        const int j = lane + 32 * q;
        sg[v][j] = val[v][q];
        if (a.clear_grad_colors && val[v][q] != 0.0f) src[j] = 0.0f;  // non-zero only where v < nv, j < n_here
      }
    }
  };

  const int nv0 = min(a.num_views, VCHUNK);
  stage(0, nv0);
  __syncwarp();
  // With more views than one chunk holds, every live row is staged (the views
  // past the first chunk are not looked at yet).
  bool need = live && a.num_views > VCHUNK;
  if (live && !need)
    for (int v = 0; v < nv0; ++v) {
      const float* gv = sg[v] + lane * 3;
      need = need || !(gv[0] == 0.0f && gv[1] == 0.0f && gv[2] == 0.0f);
    }
  const unsigned need_mask = __ballot_sync(0xffffffffu, need);
  if (need_mask) sh_rows_load<SHV_ROW_F>(rows, a.sh + (size_t)base * RF, RF, rows_here, need_mask, lane);
  __syncwarp();
  float accum[48];
#pragma unroll
  for (int e = 0; e < 48; ++e) accum[e] = 0.0f;
  const float mean[3] = {live ? a.means[idx * 3 + 0] : 0.0f, live ? a.means[idx * 3 + 1] : 0.0f,
                         live ? a.means[idx * 3 + 2] : 0.0f};
  float gm[3] = {0.0f, 0.0f, 0.0f};
  const float* row = rows + lane * SHV_ROW_F;
  for (int v0 = 0; v0 < a.num_views; v0 += VCHUNK) {
    const int nv = min(a.num_views - v0, VCHUNK);
    if (v0 > 0) {
      __syncwarp();  // every lane is done with the previous chunk
      stage(v0, nv);
      __syncwarp();
    }
    if (need)
      for (int v = 0; v < nv; ++v) {
        const float* gv = sg[v] + lane * 3;
        const float g[3] = {gv[0], gv[1], gv[2]};
        if (g[0] == 0.0f && g[1] == 0.0f && g[2] == 0.0f) continue;
        const float* cp = a.campos + (v0 + v) * 3;
        const float cam[3] = {__ldg(cp), __ldg(cp + 1), __ldg(cp + 2)};
        float gmean[3];
        sh_view_grad<USED>(row, mean, cam, g, accum, gmean);
        gm[0] += gmean[0];
        gm[1] += gmean[1];
        gm[2] += gmean[2];
      }
  }
  if (need) {
    float* gmp = a.grad_means3d + idx * 3;
    const float o0 = gmp[0], o1 = gmp[1], o2 = gmp[2];
    gmp[0] = o0 + gm[0];
    gmp[1] = o1 + gm[1];
    gmp[2] = o2 + gm[2];
  }
  __syncwarp();  // every lane is done reading the staged SH rows
  if (need) {
    float* r = rows + lane * SHV_ROW_F;
#pragma unroll
    for (int e = 0; e < 48; ++e)
      if (e < RF) r[e] = accum[e];
  }
  __syncwarp();
  // rows without a contribution: zero (store mode) or left as they are (accumulate mode)
  const bool acc = a.accumulate != 0;
  sh_rows_store<SHV_ROW_F>(a.grad_sh + (size_t)base * RF, rows, RF, rows_here, need_mask, acc, !acc, lane);
}

}  // namespace
}  // namespace gsb

using namespace gsb;

GSB_EXPORT int gsb_sh_backward_views(const gsb_sh_views_args* a, void* stream) {
  if (!a || a->P < 0 || a->num_views < 0 || a->sh_coeffs < 1 || a->sh_coeffs > 16 || a->sh_degree < 0 ||
      a->sh_degree > 3) {
    set_error("gsb_sh_backward_views: invalid sizes (P, num_views >= 0; 1 <= sh_coeffs <= 16; degree 0..3)");
    return GSB_ERR_INVALID;
  }
  if (a->P == 0) return GSB_OK;
  if (!a->means || !a->sh || !a->campos || !a->grad_sh || !a->grad_means3d ||
      (a->num_views > 0 && !a->grad_colors)) {
    set_error("gsb_sh_backward_views: null pointer argument");
    return GSB_ERR_INVALID;
  }
  gsb_sh_views_args r = *a;
  if (r.begin == 0 && r.end == 0) r.end = r.P;
  if (r.begin < 0 || r.end > r.P || r.begin > r.end) {
    set_error("gsb_sh_backward_views: need 0 <= begin <= end <= P");
    return GSB_ERR_INVALID;
  }
  if (r.begin == r.end) return GSB_OK;
  // coefficients the degree uses (degree and K both bound it)
  int used = 1;
  if (a->sh_degree > 0 && a->sh_coeffs > 3) used = 4;
  if (a->sh_degree > 1 && a->sh_coeffs > 8) used = 9;
  if (a->sh_degree > 2 && a->sh_coeffs > 15) used = 16;
  const int blocks = div_up(r.end - r.begin, SHV_THREADS);
  cudaStream_t s = (cudaStream_t)stream;
  switch (used) {
    case 1: sh_backward_views_kernel<1><<<blocks, SHV_THREADS, 0, s>>>(r); break;
    case 4: sh_backward_views_kernel<4><<<blocks, SHV_THREADS, 0, s>>>(r); break;
    case 9: sh_backward_views_kernel<9><<<blocks, SHV_THREADS, 0, s>>>(r); break;
    default: sh_backward_views_kernel<16><<<blocks, SHV_THREADS, 0, s>>>(r); break;
  }
  return check_launch("sh_backward_views_kernel");
}
