// preprocess_bwd.cu -- per-Gaussian backward of projection, EWA covariance,
// scale/rotation (or precomputed 3D covariance) and SH colour, in one pass.
//
// Restates gswarp's _fused_backward_preprocess_accumulate_warp_kernel
// (backward_kernels.py:52-295) together with the SH backward kernels
// (:297-536), and for cov3D_precomp inputs _backward_projected_means
// (:842-875) + _backward_cov2d (:709-840) + the accumulate kernel (:34-50),
// composed as in backward_ops.py:525-744.  Built with -fmad=false: fed the
// same render gradients it reproduces the CPU oracle bit for bit.
//
// B200 layout: one thread per Gaussian.  The render gradients arrive as one
// 48-byte accumulator per Gaussian (three 16-byte loads); cov3d is recomputed
// from scale/rotation instead of being stored by the forward (same
// expressions, same bits, 48 fewer bytes of traffic per Gaussian); SH rows
// are read only where the colour gradient is non-zero and the (P,K,3)
// gradient is written in place with 16-byte stores, with none of the
// reference's (P,K,3)<->(K,P,3) transposes.
#include "gsb_common.cuh"

namespace gsb {
namespace {

__constant__ float SH_C0 = 0.28209479177387814f;
__constant__ float SH_C1 = 0.4886025119029199f;
__constant__ float SH_C2[5] = {1.0925484305920792f, -1.0925484305920792f, 0.31539156525252005f,
                               -1.0925484305920792f, 0.5462742152960396f};
__constant__ float SH_C3[7] = {-0.5900435899266435f, 2.890611442640554f, -0.4570457994644658f,
                               0.3731763325901154f,  -0.4570457994644658f, 1.445305721320277f,
                               -0.5900435899266435f};

__device__ __forceinline__ void store_or_add(float* p, float v, bool acc) {
  if (acc)
    *p += v;
  else
    *p = v;
}

// math_kernels.py:89-97
__device__ __forceinline__ void dnormvdv(const float v[3], const float g[3], float out[3]) {
  const float sum2 = v[0] * v[0] + v[1] * v[1] + v[2] * v[2];
  const float invsum32 = 1.0f / sqrtf(fmx(sum2 * sum2 * sum2, 1.0e-20f));
  out[0] = ((sum2 - v[0] * v[0]) * g[0] - v[1] * v[0] * g[1] - v[2] * v[0] * g[2]) * invsum32;
  out[1] = (-v[0] * v[1] * g[0] + (sum2 - v[1] * v[1]) * g[1] - v[2] * v[1] * g[2]) * invsum32;
  out[2] = (-v[0] * v[2] * g[0] - v[1] * v[2] * g[1] + (sum2 - v[2] * v[2]) * g[2]) * invsum32;
}

// Coefficient e (= 3 * coefficient + channel) of one SH row: from a
// register copy, or from the row staged in shared memory (read where used,
// which keeps the 48 coefficients out of registers).
struct RegRow {
  const float* v;
  __device__ __forceinline__ float operator()(int e) const { return v[e]; }
};
struct SmemRow {
  const float* p;
  __device__ __forceinline__ float operator()(int e) const { return p[e]; }
};

// SH backward (backward_kernels.py:297-536), direction-dependent part:
// basis weights w[k] (0 above the degree), the number of coefficients the
// degree uses, and the gradient through the view direction from the row's
// coefficients shv[0..47] (zero-padded past K).
template <class Src>
__device__ __forceinline__ void sh_core(int K, int degree, const Src& shv, const float mean[3],
                                        const float cam[3], const float g[3], float w[16], int& used,
                                        float gmean[3]) {
  const float dir[3] = {mean[0] - cam[0], mean[1] - cam[1], mean[2] - cam[2]};
  const float len_sq = dir[0] * dir[0] + dir[1] * dir[1] + dir[2] * dir[2];
  const float inv_len = 1.0f / sqrtf(fmx(len_sq, 1.0e-20f));
  const float x = dir[0] * inv_len, y = dir[1] * inv_len, z = dir[2] * inv_len;
  float dx[3] = {0, 0, 0}, dy[3] = {0, 0, 0}, dz[3] = {0, 0, 0};
#pragma unroll
  for (int k = 0; k < 16; ++k) w[k] = 0.0f;
  used = 0;
  if (K > 0) {
    w[0] = SH_C0;
    used = 1;
  }
  if (degree > 0 && K > 3) {
    const float c1 = SH_C1;
    w[1] = -c1 * y;
    w[2] = c1 * z;
    w[3] = -c1 * x;
    used = 4;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      dx[c] = -c1 * shv(9 + c);
      dy[c] = -c1 * shv(3 + c);
      dz[c] = c1 * shv(6 + c);
    }
    if (degree > 1 && K > 8) {
      const float xx = x * x, yy = y * y, zz = z * z, xy = x * y, yz = y * z, xz = x * z;
      w[4] = SH_C2[0] * xy;
      w[5] = SH_C2[1] * yz;
      w[6] = SH_C2[2] * (2.0f * zz - xx - yy);
      w[7] = SH_C2[3] * xz;
      w[8] = SH_C2[4] * (xx - yy);
      used = 9;
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        const float s4 = shv(12 + c), s5 = shv(15 + c), s6 = shv(18 + c);
        const float s7 = shv(21 + c), s8 = shv(24 + c);
        dx[c] = dx[c] + (SH_C2[0] * y) * s4 + (SH_C2[2] * (-2.0f * x)) * s6 + (SH_C2[3] * z) * s7 +
                (SH_C2[4] * (2.0f * x)) * s8;
        dy[c] = dy[c] + (SH_C2[0] * x) * s4 + (SH_C2[1] * z) * s5 + (SH_C2[2] * (-2.0f * y)) * s6 +
                (SH_C2[4] * (-2.0f * y)) * s8;
        dz[c] = dz[c] + (SH_C2[1] * y) * s5 + (SH_C2[2] * (4.0f * z)) * s6 + (SH_C2[3] * x) * s7;
      }
      if (degree > 2 && K > 15) {
        w[9] = SH_C3[0] * y * (3.0f * xx - yy);
        w[10] = SH_C3[1] * xy * z;
        w[11] = SH_C3[2] * y * (4.0f * zz - xx - yy);
        w[12] = SH_C3[3] * z * (2.0f * zz - 3.0f * xx - 3.0f * yy);
        w[13] = SH_C3[4] * x * (4.0f * zz - xx - yy);
        w[14] = SH_C3[5] * z * (xx - yy);
        w[15] = SH_C3[6] * x * (xx - 3.0f * yy);
        used = 16;
#pragma unroll
        for (int c = 0; c < 3; ++c) {
          const float s9 = shv(27 + c), s10 = shv(30 + c), s11 = shv(33 + c);
          const float s12 = shv(36 + c), s13 = shv(39 + c);
          const float s14 = shv(42 + c), s15 = shv(45 + c);
          dx[c] = dx[c] + (SH_C3[0] * (6.0f * xy)) * s9 + (SH_C3[1] * yz) * s10 +
                  (SH_C3[2] * (-2.0f * xy)) * s11 + (SH_C3[3] * (-6.0f * xz)) * s12 +
                  (SH_C3[4] * (-3.0f * xx + 4.0f * zz - yy)) * s13 + (SH_C3[5] * (2.0f * xz)) * s14 +
                  (SH_C3[6] * (3.0f * (xx - yy))) * s15;
          dy[c] = dy[c] + (SH_C3[0] * (3.0f * (xx - yy))) * s9 + (SH_C3[1] * xz) * s10 +
                  (SH_C3[2] * (-3.0f * yy + 4.0f * zz - xx)) * s11 + (SH_C3[3] * (-6.0f * yz)) * s12 +
                  (SH_C3[4] * (-2.0f * xy)) * s13 + (SH_C3[5] * (-2.0f * yz)) * s14 +
                  (SH_C3[6] * (-6.0f * xy)) * s15;
          dz[c] = dz[c] + (SH_C3[1] * xy) * s10 + (SH_C3[2] * (8.0f * yz)) * s11 +
                  (SH_C3[3] * (3.0f * (2.0f * zz - xx - yy))) * s12 + (SH_C3[4] * (8.0f * xz)) * s13 +
                  (SH_C3[5] * (xx - yy)) * s14;
        }
      }
    }
  }
  const float ddir[3] = {dx[0] * g[0] + dx[1] * g[1] + dx[2] * g[2],
                         dy[0] * g[0] + dy[1] * g[1] + dy[2] * g[2],
                         dz[0] * g[0] + dz[1] * g[1] + dz[2] * g[2]};
  dnormvdv(dir, ddir, gmean);
}


// Colour gradient through the clamp flags; zero when the channel was clamped.
__device__ __forceinline__ bool sh_color_grad(const float grad_rgb[3], unsigned clamp_bits, float g[3]) {
#pragma unroll
  for (int c = 0; c < 3; ++c) g[c] = grad_rgb[c] * (1.0f - (float)((clamp_bits >> c) & 1u));
  return !(g[0] == 0.0f && g[1] == 0.0f && g[2] == 0.0f);
}

// Per-thread SH backward for any K: reads the row from global memory,
// writes (or adds) the (K,3) gradient row, returns the mean gradient.
__device__ void sh_backward(const gsb_preprocess_bwd_args& a, int idx, const float mean[3],
                            const float cam[3], const float grad_rgb[3], unsigned clamp_bits,
                            float gmean[3]) {
  const int K = a.sh_coeffs;
  float g[3];
  gmean[0] = gmean[1] = gmean[2] = 0.0f;
  float* out = a.grad_sh + (size_t)idx * K * 3;
  const bool acc = a.accumulate != 0;
  if (!sh_color_grad(grad_rgb, clamp_bits, g)) {
    // Zero colour gradient: every SH gradient and the direction term vanish.
    if (!acc)
      for (int k = 0; k < K * 3; ++k) out[k] = 0.0f;
    return;
  }
  const float* sp = a.sh + (size_t)idx * K * 3;
  float shv[48];
  {
    const int n = (K < 16 ? K : 16) * 3;
#pragma unroll
    for (int k = 0; k < 48; ++k) shv[k] = k < n ? __ldg(sp + k) : 0.0f;
  }
  float w[16];
  int used = 0;
  sh_core(K, a.sh_degree, RegRow{shv}, mean, cam, g, w, used, gmean);
  for (int k = 0; k < K; ++k) {
    float wk = 0.0f;  // w[k] without dynamic register indexing
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (j == k) wk = w[j];
    for (int c = 0; c < 3; ++c) {
      const float gv = k < used ? wk * g[c] : 0.0f;
      store_or_add(out + k * 3 + c, gv, acc);
    }
  }
}

// Warp-cooperative SH backward for (P,16,3) rows.  One thread per Gaussian
// reads and writes its 48-float row with stride-48 accesses, 32 rows apart
// across a warp; here the warp moves its 32 rows (each 192 contiguous bytes)
// between global and shared memory with coalesced 16-byte global accesses,
// and each thread works on its row in shared memory, reading coefficients
// where they are used (rows padded to 49 floats: the per-thread scalar
// accesses of a warp hit 32 different banks).  Arithmetic is the same
// sh_core as the per-thread path.
constexpr int SH_ROW_F = 49;
constexpr int PB_THREADS = launch::PREPROCESS_BWD;
constexpr int PB_SH16_THREADS = launch::PREPROCESS_BWD_SH16;

__device__ __forceinline__ void sh_backward_staged(const gsb_preprocess_bwd_args& a, float* rows, int my_idx,
                                                   bool work, bool need, const float mean[3],
                                                   const float cam[3], const float g[3], float gmean[3]) {
  const int lane = threadIdx.x & 31;
  const bool acc = a.accumulate != 0;
  const unsigned need_mask = __ballot_sync(0xffffffffu, need);
  const unsigned work_mask = __ballot_sync(0xffffffffu, work);
  gmean[0] = gmean[1] = gmean[2] = 0.0f;
  if (work_mask == 0u) return;
  // Row r belongs to lane r's Gaussian (consecutive Gaussians, or the
  // Gaussians of an id list); its 12 float4 are contiguous in memory.
  const float4* src = reinterpret_cast<const float4*>(a.sh);
  if (need_mask) {
#pragma unroll 4
    for (int j = lane; j < 32 * 12; j += 32) {
      const int r = j / 12, q = j - r * 12;
      const int row_idx = __shfl_sync(0xffffffffu, my_idx, r);
      if ((need_mask >> r) & 1u) {
        const float4 v = __ldg(src + (size_t)row_idx * 12 + q);
        float* d = rows + r * SH_ROW_F + q * 4;
        d[0] = v.x;
        d[1] = v.y;
        d[2] = v.z;
        d[3] = v.w;
      }
    }
  }
  __syncwarp();
  if (need) {
    float* row = rows + lane * SH_ROW_F;
    float w[16];
    int used = 0;
    sh_core(16, a.sh_degree, SmemRow{row}, mean, cam, g, w, used, gmean);
#pragma unroll
    for (int e = 0; e < 48; ++e) row[e] = e / 3 < used ? w[e / 3] * g[e % 3] : 0.0f;
  }
  __syncwarp();
  // Written back in chunks of SH_CHUNK float4 per lane; in accumulate mode a
  // chunk's old values are all loaded before its stores (as above, so the
  // loads do not wait on earlier stores).
  float4* dst_base = reinterpret_cast<float4*>(a.grad_sh);
  constexpr int SH_CHUNK = 4;
#pragma unroll 1
  for (int j0 = 0; j0 < 12; j0 += SH_CHUNK) {
    float4 old[SH_CHUNK];
    float4* dst[SH_CHUNK];
    bool wr[SH_CHUNK], nd[SH_CHUNK];
#pragma unroll
    for (int c = 0; c < SH_CHUNK; ++c) {
      const int j = (j0 + c) * 32 + lane;
      const int r = j / 12, q = j - r * 12;
      const int row_idx = __shfl_sync(0xffffffffu, my_idx, r);
      wr[c] = (work_mask >> r) & 1u;
      nd[c] = (need_mask >> r) & 1u;
      dst[c] = dst_base + (size_t)row_idx * 12 + q;
      old[c] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      if (acc && wr[c] && nd[c]) old[c] = *dst[c];
    }
#pragma unroll
    for (int c = 0; c < SH_CHUNK; ++c) {
      const int j = (j0 + c) * 32 + lane;
      const int r = j / 12, q = j - r * 12;
      if (!wr[c]) continue;
      if (nd[c]) {
        const float* sr = rows + r * SH_ROW_F + q * 4;
        float4 v = make_float4(sr[0], sr[1], sr[2], sr[3]);
        if (acc) v = make_float4(old[c].x + v.x, old[c].y + v.y, old[c].z + v.z, old[c].w + v.w);
        *dst[c] = v;
      } else if (!acc) {
        *dst[c] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
    }
  }
  __syncwarp();
}

// backward_kernels.py:89-112 (scale/rotation path): the screen-space
// gradient (gxy0, gxy1) through the projection of the mean, plus the term of
// the view-depth gradient rgd; returns the mean's view-space depth.
__device__ __forceinline__ float proj_mean_grad(const float* pr, const float* vf, const float mean[3], float gxy0,
                                                float gxy1, float rgd, float pm[3]) {
  const float hom_x = pr[0] * mean[0] + pr[4] * mean[1] + pr[8] * mean[2] + pr[12];
  const float hom_y = pr[1] * mean[0] + pr[5] * mean[1] + pr[9] * mean[2] + pr[13];
  const float hom_w = pr[3] * mean[0] + pr[7] * mean[1] + pr[11] * mean[2] + pr[15];
  const float inv_w = 1.0f / (hom_w + 1.0e-7f);
  const float inv_w2 = inv_w * inv_w;
  const float gh = hom_x * gxy0 + hom_y * gxy1;
  pm[0] = inv_w * (pr[0] * gxy0 + pr[1] * gxy1) - pr[3] * inv_w2 * gh;
  pm[1] = inv_w * (pr[4] * gxy0 + pr[5] * gxy1) - pr[7] * inv_w2 * gh;
  pm[2] = inv_w * (pr[8] * gxy0 + pr[9] * gxy1) - pr[11] * inv_w2 * gh;
  const float zz = vf[2] * mean[0] + vf[6] * mean[1] + vf[10] * mean[2] + vf[14];
  pm[0] = pm[0] + (vf[2] - vf[3] * zz) * rgd;
  pm[1] = pm[1] + (vf[6] - vf[7] * zz) * rgd;
  pm[2] = pm[2] + (vf[10] - vf[11] * zz) * rgd;
  return zz;
}

// backward_kernels.py:124-287 (scale/rotation path, radius > 0): the
// conic gradient tc (render + user conic_2D gradient) and the user conic_2D_inv
// gradient gi through the EWA covariance to the mean (gcm), the scales (gs)
// and the rotation (gr); (x, y, z) is the mean in view space.
__device__ __forceinline__ void cov_scale_rot_grads(const float* vf, float x, float y, float z, float limx,
                                                    float limy, float focal_x, float focal_y,
                                                    float scale_modifier, const float sc_in[3], float4 rot_in,
                                                    float tc0, float tc1, float tc2, float gi0, float gi1,
                                                    float gi2, float gcm[3], float gs[3], float gr[4]) {
  const float w00 = vf[0], w01 = vf[1], w02 = vf[2], w10 = vf[4], w11 = vf[5], w12 = vf[6];
  const float w20 = vf[8], w21 = vf[9], w22 = vf[10];
  const float tz_inv = 1.0f / (z + 1.0e-7f);
  const float txtz = x * tz_inv, tytz = y * tz_inv;
  float x_mul = 1.0f, y_mul = 1.0f;
  if (txtz < -limx || txtz > limx) x_mul = 0.0f;
  if (tytz < -limy || tytz > limy) y_mul = 0.0f;
  const float tx = fclamp(txtz, -limx, limx), ty = fclamp(tytz, -limy, limy);
  const float j00 = focal_x * tz_inv;
  const float j02 = -j00 * tx;
  const float j11 = focal_y * tz_inv;
  const float j12 = -j11 * ty;
  const float t00 = w00 * j00 + w02 * j02, t10 = w10 * j00 + w12 * j02,
              t20 = w20 * j00 + w22 * j02;
  const float t01 = w01 * j11 + w02 * j12, t11 = w11 * j11 + w12 * j12,
              t21 = w21 * j11 + w22 * j12;
  const float s0 = sc_in[0] * scale_modifier;
  const float s1 = sc_in[1] * scale_modifier;
  const float s2 = sc_in[2] * scale_modifier;
  const float4 q = rot_in;
  const float rr = q.x, xq = q.y, yq = q.z, zq = q.w;
  const float r00 = 1.0f - 2.0f * (yq * yq + zq * zq);
  const float r01 = 2.0f * (xq * yq + rr * zq);
  const float r02 = 2.0f * (xq * zq - rr * yq);
  const float r10 = 2.0f * (xq * yq - rr * zq);
  const float r11 = 1.0f - 2.0f * (xq * xq + zq * zq);
  const float r12 = 2.0f * (yq * zq + rr * xq);
  const float r20 = 2.0f * (xq * zq + rr * yq);
  const float r21 = 2.0f * (yq * zq - rr * xq);
  const float r22 = 1.0f - 2.0f * (xq * xq + yq * yq);
  const float m00 = s0 * r00, m01 = s0 * r01, m02 = s0 * r02;
  const float m10 = s1 * r10, m11 = s1 * r11, m12 = s1 * r12;
  const float m20 = s2 * r20, m21 = s2 * r21, m22 = s2 * r22;
  const float v00 = m00 * m00 + m10 * m10 + m20 * m20;
  const float v01 = m00 * m01 + m10 * m11 + m20 * m21;
  const float v02 = m00 * m02 + m10 * m12 + m20 * m22;
  const float v11 = m01 * m01 + m11 * m11 + m21 * m21;
  const float v12 = m01 * m02 + m11 * m12 + m21 * m22;
  const float v22 = m02 * m02 + m12 * m12 + m22 * m22;
  const float vt0x = v00 * t00 + v01 * t10 + v02 * t20;
  const float vt0y = v01 * t00 + v11 * t10 + v12 * t20;
  const float vt0z = v02 * t00 + v12 * t10 + v22 * t20;
  const float vt1x = v00 * t01 + v01 * t11 + v02 * t21;
  const float vt1y = v01 * t01 + v11 * t11 + v12 * t21;
  const float vt1z = v02 * t01 + v12 * t11 + v22 * t21;
  const float filt = 0.0f;
  const float aa = t00 * vt0x + t10 * vt0y + t20 * vt0z + 0.3f + filt;
  const float bb = t00 * vt1x + t10 * vt1y + t20 * vt1z;
  const float cc = t01 * vt1x + t11 * vt1y + t21 * vt1z + 0.3f + filt;
  const float denom = aa * cc - bb * bb;
  const float denom2inv = 1.0f / (denom * denom + 1.0e-7f);
  float dL_da = denom2inv * (-cc * cc * tc0 + 2.0f * bb * cc * tc1 - bb * bb * tc2);
  float dL_dc = denom2inv * (-aa * aa * tc2 + 2.0f * aa * bb * tc1 - bb * bb * tc0);
  float dL_db = denom2inv * 2.0f * (bb * cc * tc0 - (aa * cc + bb * bb) * tc1 + aa * bb * tc2);
  dL_da = dL_da + gi0;
  dL_db = dL_db + gi1;
  dL_dc = dL_dc + gi2;
  const float gc0 = t00 * t00 * dL_da + t00 * t01 * dL_db + t01 * t01 * dL_dc;
  const float gc3v = t10 * t10 * dL_da + t10 * t11 * dL_db + t11 * t11 * dL_dc;
  const float gc5 = t20 * t20 * dL_da + t20 * t21 * dL_db + t21 * t21 * dL_dc;
  const float gc1 = 2.0f * t00 * t10 * dL_da + (t00 * t11 + t01 * t10) * dL_db + 2.0f * t01 * t11 * dL_dc;
  const float gc2 = 2.0f * t00 * t20 * dL_da + (t00 * t21 + t01 * t20) * dL_db + 2.0f * t01 * t21 * dL_dc;
  const float gc4 = 2.0f * t10 * t20 * dL_da + (t10 * t21 + t11 * t20) * dL_db + 2.0f * t11 * t21 * dL_dc;
  const float dT00 = 2.0f * vt0x * dL_da + vt1x * dL_db;
  const float dT01 = 2.0f * vt0y * dL_da + vt1y * dL_db;
  const float dT02 = 2.0f * vt0z * dL_da + vt1z * dL_db;
  const float dT10 = vt0x * dL_db + 2.0f * vt1x * dL_dc;
  const float dT11 = vt0y * dL_db + 2.0f * vt1y * dL_dc;
  const float dT12 = vt0z * dL_db + 2.0f * vt1z * dL_dc;
  const float dJ00 = w00 * dT00 + w10 * dT01 + w20 * dT02;
  const float dJ02 = w02 * dT00 + w12 * dT01 + w22 * dT02;
  const float dJ11 = w01 * dT10 + w11 * dT11 + w21 * dT12;
  const float dJ12 = w02 * dT10 + w12 * dT11 + w22 * dT12;
  const float dL_dtx = x_mul * -j00 * tz_inv * dJ02;
  const float dL_dty = y_mul * -j11 * tz_inv * dJ12;
  const float dL_dtz = -(j00 * dJ00 + j11 * dJ11 + 2.0f * j02 * dJ02 + 2.0f * j12 * dJ12) * tz_inv;
  gcm[0] = w00 * dL_dtx + w01 * dL_dty + w02 * dL_dtz;
  gcm[1] = w10 * dL_dtx + w11 * dL_dty + w12 * dL_dtz;
  gcm[2] = w20 * dL_dtx + w21 * dL_dty + w22 * dL_dtz;
  const float sg00 = gc0, sg01 = 0.5f * gc1, sg02 = 0.5f * gc2, sg11 = gc3v, sg12 = 0.5f * gc4,
              sg22 = gc5;
  const float dM00 = 2.0f * (m00 * sg00 + m01 * sg01 + m02 * sg02);
  const float dM01 = 2.0f * (m00 * sg01 + m01 * sg11 + m02 * sg12);
  const float dM02 = 2.0f * (m00 * sg02 + m01 * sg12 + m02 * sg22);
  const float dM10 = 2.0f * (m10 * sg00 + m11 * sg01 + m12 * sg02);
  const float dM11 = 2.0f * (m10 * sg01 + m11 * sg11 + m12 * sg12);
  const float dM12 = 2.0f * (m10 * sg02 + m11 * sg12 + m12 * sg22);
  const float dM20 = 2.0f * (m20 * sg00 + m21 * sg01 + m22 * sg02);
  const float dM21 = 2.0f * (m20 * sg01 + m21 * sg11 + m22 * sg12);
  const float dM22 = 2.0f * (m20 * sg02 + m21 * sg12 + m22 * sg22);
  gs[0] = scale_modifier * (dM00 * r00 + dM01 * r01 + dM02 * r02);
  gs[1] = scale_modifier * (dM10 * r10 + dM11 * r11 + dM12 * r12);
  gs[2] = scale_modifier * (dM20 * r20 + dM21 * r21 + dM22 * r22);
  const float dR00 = dM00 * s0, dR01 = dM01 * s0, dR02 = dM02 * s0;
  const float dR10 = dM10 * s1, dR11 = dM11 * s1, dR12 = dM12 * s1;
  const float dR20 = dM20 * s2, dR21 = dM21 * s2, dR22 = dM22 * s2;
  gr[0] = 2.0f * zq * (dR01 - dR10) + 2.0f * yq * (dR20 - dR02) + 2.0f * xq * (dR12 - dR21);
  gr[1] = 2.0f * yq * (dR10 + dR01) + 2.0f * zq * (dR20 + dR02) + 2.0f * rr * (dR12 - dR21) -
          4.0f * xq * (dR22 + dR11);
  gr[2] = 2.0f * xq * (dR10 + dR01) + 2.0f * rr * (dR20 - dR02) + 2.0f * zq * (dR12 + dR21) -
          4.0f * yq * (dR22 + dR00);
  gr[3] = 2.0f * rr * (dR01 - dR10) + 2.0f * xq * (dR20 + dR02) + 2.0f * yq * (dR12 + dR21) -
          4.0f * zq * (dR11 + dR00);
}

// SH16: SH rows of exactly 16 coefficients, 16-byte aligned, handled by
// sh_backward_staged (every lane of a warp takes part, so lanes past P or
// without work stay in the kernel and only skip their loads and stores).
// In accumulate mode a Gaussian with radius 0 got no render gradient and no
// user gradient (both only apply where radius > 0), so its contribution is
// zero and it is skipped without touching memory.
// SH handling, a template parameter so that each variant carries only the
// registers of its own SH path.
enum ShMode { SHM_NONE = 0, SHM_ANY = 1, SHM_16 = 2 };

__device__ __forceinline__ void prefetch_line(const void* p) {
  asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}

// Store mode (the autograd path, every Gaussian): the inputs are requested
// with the radius instead of after it.
__device__ __forceinline__ void prefetch_inputs(const gsb_preprocess_bwd_args& a, int gid) {
  const size_t g = (size_t)gid;
  prefetch_line(a.means + g * 3);
  prefetch_line(a.grad_acc + g * 12);
  prefetch_line(a.grad_acc + g * 12 + 11);
  if (a.scales) prefetch_line(a.scales + g * 3);
  if (a.rotations) prefetch_line(a.rotations + g * 4);
  prefetch_line(a.records + g * 12 + 7);
}

// Accumulate mode: the thread's memory is requested as soon as its id is
// known.  Its inputs would otherwise wait for the radius load, and the old
// gradient values for the whole computation (they are read just before the
// stores), each a further round trip to DRAM; prefetched lines turn those
// later loads into cache hits without holding registers across the
// computation.  The 48-byte accumulator can straddle two 128-byte lines.
__device__ __forceinline__ void prefetch_rows(const gsb_preprocess_bwd_args& a, int gid) {
  const size_t g = (size_t)gid;
  prefetch_line(a.means + g * 3);
  prefetch_line(a.grad_acc + g * 12);
  prefetch_line(a.grad_acc + g * 12 + 11);
  if (a.scales) prefetch_line(a.scales + g * 3);
  if (a.rotations) prefetch_line(a.rotations + g * 4);
  prefetch_line(a.grad_means3d + g * 3);
  if (a.grad_scales) prefetch_line(a.grad_scales + g * 3);
  if (a.grad_rotations) prefetch_line(a.grad_rotations + g * 4);
  if (a.grad_opacity) prefetch_line(a.grad_opacity + g);
  if (a.grad_colors) {
    prefetch_line(a.grad_colors + g * 3);
    if (a.grad_colors_clamped) prefetch_line(a.records + g * 12 + 7);
  }
}

template <bool PRECOMP, int SHM>
__global__ void __launch_bounds__(SHM == SHM_16 ? PB_SH16_THREADS : PB_THREADS, SHM == SHM_16 ? 6 : (SHM == SHM_NONE ? 3 : 1))
    preprocess_bwd_kernel(const gsb_preprocess_bwd_args a) {
  constexpr bool SH16 = SHM == SHM_16;
  __shared__ float s_view[16], s_proj[16], s_cam[3];
  __shared__ float s_rows[SH16 ? PB_SH16_THREADS * SH_ROW_F : 1];
  if (threadIdx.x < 16) {
    s_view[threadIdx.x] = a.viewmatrix[threadIdx.x];
    s_proj[threadIdx.x] = a.projmatrix[threadIdx.x];
  } else if (threadIdx.x < 19) {
    s_cam[threadIdx.x - 16] = a.campos ? a.campos[threadIdx.x - 16] : 0.0f;
  }
  __syncthreads();
  const int tid = blockIdx.x * blockDim.x + threadIdx.x;
  const bool acc = a.accumulate != 0;
  // With an id list, thread t handles Gaussian ids[t] (t < num_ids);
  // otherwise thread t handles Gaussian t.
  const bool live = a.ids ? tid < a.num_ids : tid < a.P;
  const int gid = a.ids ? (live ? a.ids[tid] : 0) : tid;
  if (!SH16 && acc && live) prefetch_rows(a, gid);
  if (!acc && live) prefetch_inputs(a, gid);
  const int rad = live ? a.radii[gid] : 0;
  if (SH16 && live && rad > 0) {
    // the SH row is staged only after the render gradient and clamp bits are read
    prefetch_line(a.sh + (size_t)gid * 48);
    prefetch_line(a.sh + (size_t)gid * 48 + 47);
  }
  const bool work = live && (!acc || rad > 0);
  if (!SH16 && !work) return;
  const float* pr = s_proj;
  const float* vf = s_view;
  float mean[3] = {0.0f, 0.0f, 0.0f};
  float4 gq0 = make_float4(0.0f, 0.0f, 0.0f, 0.0f), gq1 = gq0, gq2 = gq0;
  const float4* ga4 = reinterpret_cast<const float4*>(a.grad_acc) + (size_t)gid * 3;
  if (work) {
    mean[0] = a.means[gid * 3];
    mean[1] = a.means[gid * 3 + 1];
    mean[2] = a.means[gid * 3 + 2];
    gq0 = ga4[0];
    gq1 = ga4[1];
    gq2 = ga4[2];
  }
  // Scale/rotation inputs are loaded here, ahead of the SH stage's stores
  // (loads placed after those stores could not be moved above them).
  float sc_in[3] = {0.0f, 0.0f, 0.0f};
  float4 rot_in = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  if (!PRECOMP && work && rad > 0) {
    sc_in[0] = a.scales[gid * 3 + 0];
    sc_in[1] = a.scales[gid * 3 + 1];
    sc_in[2] = a.scales[gid * 3 + 2];
    rot_in = reinterpret_cast<const float4*>(a.rotations)[gid];
  }
  const float rrgb[3] = {gq2.x, gq2.y, gq2.z};

  // SH first: only its mean gradient (3 floats) stays live through the
  // projection / covariance part below, which keeps the register peak down.
  float gsm[3] = {0.0f, 0.0f, 0.0f};
  if (SH16) {
    float g[3] = {0.0f, 0.0f, 0.0f};
    bool need = false;
    if (work) {
      const unsigned clamp_bits =
          __float_as_uint(reinterpret_cast<const float4*>(a.records)[(size_t)gid * 3 + 1].w);
      need = sh_color_grad(rrgb, clamp_bits, g);
    }
    sh_backward_staged(a, s_rows + (threadIdx.x & ~31) * SH_ROW_F, gid, work, need, mean, s_cam, g,
                       gsm);
    if (!work) return;
  } else if (SHM == SHM_ANY && a.sh) {
    const unsigned clamp_bits =
        __float_as_uint(reinterpret_cast<const float4*>(a.records)[(size_t)gid * 3 + 1].w);
    sh_backward(a, gid, mean, s_cam, rrgb, clamp_bits, gsm);
  }
  const float rgx = gq0.x, rgy = gq0.y, rgd = gq0.z;
  const float rco[4] = {gq1.x, gq1.y, gq1.z, gq1.w};

  float gxy0 = rgx, gxy1 = rgy;
  if (rad > 0 && a.grad_proj_2d) {
    gxy0 = gxy0 + a.grad_proj_2d[gid * 2];
    gxy1 = gxy1 + a.grad_proj_2d[gid * 2 + 1];
  }
  float pm_x, pm_y, pm_z;
  float zz;
  if (!PRECOMP) {
    float pm[3];
    zz = proj_mean_grad(pr, vf, mean, gxy0, gxy1, rgd, pm);
    pm_x = pm[0];
    pm_y = pm[1];
    pm_z = pm[2];
  } else {
    // backward_kernels.py:853-866
    const float hom_x = pr[0] * mean[0] + pr[4] * mean[1] + pr[8] * mean[2] + pr[12];
    const float hom_y = pr[1] * mean[0] + pr[5] * mean[1] + pr[9] * mean[2] + pr[13];
    const float hom_w = pr[3] * mean[0] + pr[7] * mean[1] + pr[11] * mean[2] + pr[15];
    const float inv_w = 1.0f / (hom_w + 1.0e-7f);
    const float mul1 = hom_x * inv_w * inv_w;
    const float mul2 = hom_y * inv_w * inv_w;
    pm_x = (pr[0] * inv_w - pr[3] * mul1) * gxy0 + (pr[1] * inv_w - pr[3] * mul2) * gxy1;
    pm_y = (pr[4] * inv_w - pr[7] * mul1) * gxy0 + (pr[5] * inv_w - pr[7] * mul2) * gxy1;
    pm_z = (pr[8] * inv_w - pr[11] * mul1) * gxy0 + (pr[9] * inv_w - pr[11] * mul2) * gxy1;
    zz = vf[2] * mean[0] + vf[6] * mean[1] + vf[10] * mean[2] + vf[14];
    pm_x = pm_x + (vf[2] - vf[3] * zz) * rgd;
    pm_y = pm_y + (vf[6] - vf[7] * zz) * rgd;
    pm_z = pm_z + (vf[10] - vf[11] * zz) * rgd;
  }

  float gcm[3] = {0.0f, 0.0f, 0.0f};
  float gs[3] = {0.0f, 0.0f, 0.0f}, gr[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  float gc3[6] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
  if (rad > 0) {
    const float x = vf[0] * mean[0] + vf[4] * mean[1] + vf[8] * mean[2] + vf[12];
    const float y = vf[1] * mean[0] + vf[5] * mean[1] + vf[9] * mean[2] + vf[13];
    const float z = zz;
    const float limx = 1.3f * a.tanfovx, limy = 1.3f * a.tanfovy;
    const float w00 = vf[0], w01 = vf[1], w02 = vf[2], w10 = vf[4], w11 = vf[5], w12 = vf[6];
    const float w20 = vf[8], w21 = vf[9], w22 = vf[10];
    // A NULL user gradient is a zero gradient (x + 0 == x).
    const float* gk = a.grad_conic_2d ? a.grad_conic_2d + gid * 3 : nullptr;
    const float* gkv = a.grad_conic_2d_inv ? a.grad_conic_2d_inv + gid * 3 : nullptr;
    const float tc0 = gk ? rco[0] + gk[0] : rco[0];
    const float tc1 = gk ? rco[1] + gk[1] : rco[1];
    const float tc2 = gk ? rco[2] + gk[2] : rco[2];
    const float gi0 = gkv ? gkv[0] : 0.0f;
    const float gi1 = gkv ? gkv[1] : 0.0f;
    const float gi2 = gkv ? gkv[2] : 0.0f;
    if (!PRECOMP) {
      cov_scale_rot_grads(vf, x, y, z, limx, limy, a.focal_x, a.focal_y, a.scale_modifier, sc_in, rot_in, tc0,
                          tc1, tc2, gi0, gi1, gi2, gcm, gs, gr);
    } else {
      // backward_kernels.py:731-840
      const float* c3 = a.cov3d_precomp + (size_t)gid * 6;
      const float txtz = x / z, tytz = y / z;
      const float tx = fclamp(txtz, -limx, limx) * z;
      const float ty = fclamp(tytz, -limy, limy) * z;
      float xm = 1.0f, ym = 1.0f;
      if (txtz < -limx || txtz > limx) xm = 0.0f;
      if (tytz < -limy || tytz > limy) ym = 0.0f;
      const float j00 = a.focal_x / z;
      const float j02 = -(a.focal_x * tx) / (z * z);
      const float j11 = a.focal_y / z;
      const float j12 = -(a.focal_y * ty) / (z * z);
      const float t00 = w00 * j00 + w02 * j02, t10 = w10 * j00 + w12 * j02,
                  t20 = w20 * j00 + w22 * j02;
      const float t01 = w01 * j11 + w02 * j12, t11 = w11 * j11 + w12 * j12,
                  t21 = w21 * j11 + w22 * j12;
      const float v00 = c3[0], v01 = c3[1], v02 = c3[2], v11 = c3[3], v12 = c3[4], v22 = c3[5];
      const float vt0x = v00 * t00 + v01 * t10 + v02 * t20;
      const float vt0y = v01 * t00 + v11 * t10 + v12 * t20;
      const float vt0z = v02 * t00 + v12 * t10 + v22 * t20;
      const float vt1x = v00 * t01 + v01 * t11 + v02 * t21;
      const float vt1y = v01 * t01 + v11 * t11 + v12 * t21;
      const float vt1z = v02 * t01 + v12 * t11 + v22 * t21;
      const float filt = 0.0f;
      const float aa = t00 * vt0x + t10 * vt0y + t20 * vt0z + 0.3f + filt;
      const float bb = t00 * vt1x + t10 * vt1y + t20 * vt1z;
      const float cc = t01 * vt1x + t11 * vt1y + t21 * vt1z + 0.3f + filt;
      const float denom = aa * cc - bb * bb;
      const float d2i = 1.0f / (denom * denom + 1.0e-7f);
      float dL_da = d2i * (-cc * cc * tc0 + 2.0f * bb * cc * tc1 + (denom - aa * cc) * tc2);
      float dL_dc = d2i * (-aa * aa * tc2 + 2.0f * aa * bb * tc1 + (denom - aa * cc) * tc0);
      float dL_db = d2i * 2.0f * (bb * cc * tc0 - (denom + 2.0f * bb * bb) * tc1 + aa * bb * tc2);
      dL_da = dL_da + gi0;
      dL_db = dL_db + gi1;
      dL_dc = dL_dc + gi2;
      gc3[0] = t00 * t00 * dL_da + t00 * t01 * dL_db + t01 * t01 * dL_dc;
      gc3[3] = t10 * t10 * dL_da + t10 * t11 * dL_db + t11 * t11 * dL_dc;
      gc3[5] = t20 * t20 * dL_da + t20 * t21 * dL_db + t21 * t21 * dL_dc;
      gc3[1] = 2.0f * t00 * t10 * dL_da + (t00 * t11 + t01 * t10) * dL_db + 2.0f * t01 * t11 * dL_dc;
      gc3[2] = 2.0f * t00 * t20 * dL_da + (t00 * t21 + t01 * t20) * dL_db + 2.0f * t01 * t21 * dL_dc;
      gc3[4] = 2.0f * t10 * t20 * dL_da + (t10 * t21 + t11 * t20) * dL_db + 2.0f * t11 * t21 * dL_dc;
      const float dT00 = 2.0f * (t00 * v00 + t10 * v01 + t20 * v02) * dL_da + (t01 * v00 + t11 * v01 + t21 * v02) * dL_db;
      const float dT01 = 2.0f * (t00 * v01 + t10 * v11 + t20 * v12) * dL_da + (t01 * v01 + t11 * v11 + t21 * v12) * dL_db;
      const float dT02 = 2.0f * (t00 * v02 + t10 * v12 + t20 * v22) * dL_da + (t01 * v02 + t11 * v12 + t21 * v22) * dL_db;
      const float dT10 = 2.0f * (t01 * v00 + t11 * v01 + t21 * v02) * dL_dc + (t00 * v00 + t10 * v01 + t20 * v02) * dL_db;
      const float dT11 = 2.0f * (t01 * v01 + t11 * v11 + t21 * v12) * dL_dc + (t00 * v01 + t10 * v11 + t20 * v12) * dL_db;
      const float dT12 = 2.0f * (t01 * v02 + t11 * v12 + t21 * v22) * dL_dc + (t00 * v02 + t10 * v12 + t20 * v22) * dL_db;
      const float dJ00 = w00 * dT00 + w10 * dT01 + w20 * dT02;
      const float dJ02 = w02 * dT00 + w12 * dT01 + w22 * dT02;
      const float dJ11 = w01 * dT10 + w11 * dT11 + w21 * dT12;
      const float dJ12 = w02 * dT10 + w12 * dT11 + w22 * dT12;
      const float tz_inv = 1.0f / z;
      const float tz2 = tz_inv * tz_inv;
      const float tz3 = tz2 * tz_inv;
      const float dL_dtx = xm * -a.focal_x * tz2 * dJ02;
      const float dL_dty = ym * -a.focal_y * tz2 * dJ12;
      const float dL_dtz = -a.focal_x * tz2 * dJ00 - a.focal_y * tz2 * dJ11 +
                           (2.0f * a.focal_x * tx) * tz3 * dJ02 + (2.0f * a.focal_y * ty) * tz3 * dJ12;
      gcm[0] = vf[0] * dL_dtx + vf[1] * dL_dty + vf[2] * dL_dtz;
      gcm[1] = vf[4] * dL_dtx + vf[5] * dL_dty + vf[6] * dL_dtz;
      gcm[2] = vf[8] * dL_dtx + vf[9] * dL_dty + vf[10] * dL_dtz;
    }
  }
  float m0 = pm_x + gcm[0], m1 = pm_y + gcm[1], m2 = pm_z + gcm[2];
  if (SH16 || (SHM == SHM_ANY && a.sh)) {
    m0 = m0 + gsm[0];
    m1 = m1 + gsm[1];
    m2 = m2 + gsm[2];
  }
  // Accumulate mode: every old value is loaded before any store.  The output
  // pointers may alias as far as the compiler knows, so interleaved
  // read-modify-writes would each wait for the previous store to retire.
  const bool has2 = a.grad_means2d != nullptr;
  const bool hass = !PRECOMP && a.grad_scales != nullptr;
  const bool hasr = !PRECOMP && a.grad_rotations != nullptr;
  const bool hasc = PRECOMP && a.grad_cov3d != nullptr;
  const bool haso = a.grad_opacity != nullptr;
  float om[3] = {0.0f, 0.0f, 0.0f}, o2[3] = {0.0f, 0.0f, 0.0f}, os[3] = {0.0f, 0.0f, 0.0f};
  float orr[4] = {0.0f, 0.0f, 0.0f, 0.0f}, oc[6] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f}, oo = 0.0f;
  if (acc) {
#pragma unroll
    for (int k = 0; k < 3; ++k) om[k] = a.grad_means3d[gid * 3 + k];
    if (has2)
#pragma unroll
      for (int k = 0; k < 3; ++k) o2[k] = a.grad_means2d[gid * 3 + k];
    if (hass)
#pragma unroll
      for (int k = 0; k < 3; ++k) os[k] = a.grad_scales[gid * 3 + k];
    if (hasr)
#pragma unroll
      for (int k = 0; k < 4; ++k) orr[k] = a.grad_rotations[gid * 4 + k];
    if (hasc)
#pragma unroll
      for (int k = 0; k < 6; ++k) oc[k] = a.grad_cov3d[gid * 6 + k];
    if (haso) oo = a.grad_opacity[gid];
  }
  // *p += v is *p = *p + v: the same sum in the same order.
  const float mv[3] = {m0, m1, m2};
#pragma unroll
  for (int k = 0; k < 3; ++k) a.grad_means3d[gid * 3 + k] = acc ? om[k] + mv[k] : mv[k];
  if (has2) {
    const float v2[3] = {rgx, rgy, 0.0f};
#pragma unroll
    for (int k = 0; k < 3; ++k) a.grad_means2d[gid * 3 + k] = acc ? o2[k] + v2[k] : v2[k];
  }
  if (hass)
#pragma unroll
    for (int k = 0; k < 3; ++k) a.grad_scales[gid * 3 + k] = acc ? os[k] + gs[k] : gs[k];
  if (hasr)
#pragma unroll
    for (int k = 0; k < 4; ++k) a.grad_rotations[gid * 4 + k] = acc ? orr[k] + gr[k] : gr[k];
  if (hasc)
#pragma unroll
    for (int k = 0; k < 6; ++k) a.grad_cov3d[gid * 6 + k] = acc ? oc[k] + gc3[k] : gc3[k];
  if (haso) a.grad_opacity[gid] = acc ? oo + rco[3] : rco[3];
  if (a.densify_grad_accum) a.densify_grad_accum[gid] += sqrtf(rgx * rgx + rgy * rgy);
  if (a.clear_grad_acc) {
    // last, so the zero stores do not hold back any load above
    float4* w4 = const_cast<float4*>(ga4);
    const float4 z = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    w4[0] = z;
    w4[1] = z;
    w4[2] = z;
  }
  if (a.grad_colors) {
    // grad_colors_clamped: the gradient past the forward's clamp, the g the SH backward uses
    const unsigned cb =
        a.grad_colors_clamped ? __float_as_uint(reinterpret_cast<const float4*>(a.records)[(size_t)gid * 3 + 1].w)
                              : 0u;
    float gc[3];
    sh_color_grad(rrgb, cb, gc);
    float* gcp = a.grad_colors + gid * 3;
    const float o0 = acc ? gcp[0] : 0.0f, o1 = acc ? gcp[1] : 0.0f, o2 = acc ? gcp[2] : 0.0f;
    gcp[0] = acc ? o0 + gc[0] : gc[0];
    gcp[1] = acc ? o1 + gc[1] : gc[1];
    gcp[2] = acc ? o2 + gc[2] : gc[2];
  }
}

}  // namespace
}  // namespace gsb

using namespace gsb;

GSB_EXPORT int gsb_preprocess_bwd(const gsb_preprocess_bwd_args* a, void* stream) {
  if (!a || a->P < 0 || a->W <= 0 || a->H <= 0) {
    set_error("gsb_preprocess_bwd: invalid sizes");
    return GSB_ERR_INVALID;
  }
  if (a->P == 0) return GSB_OK;
  if (a->ids && (!a->accumulate || a->num_ids < 0 || a->num_ids > a->P)) {
    set_error("gsb_preprocess_bwd: an id list needs accumulate mode and 0 <= num_ids <= P");
    return GSB_ERR_INVALID;
  }
  const int threads_needed = a->ids ? a->num_ids : a->P;
  if (threads_needed == 0) return GSB_OK;
  const bool precomp = a->cov3d_precomp != nullptr;
  if (!precomp && (!a->scales || !a->rotations)) {
    set_error("gsb_preprocess_bwd: scales/rotations or cov3d_precomp required");
    return GSB_ERR_INVALID;
  }
  if (!a->means || !a->radii || !a->viewmatrix || !a->projmatrix || !a->records ||
      !a->grad_acc ||
      !a->grad_means3d || (a->sh && (!a->grad_sh || !a->campos || a->sh_coeffs <= 0))) {
    set_error("gsb_preprocess_bwd: null pointer argument");
    return GSB_ERR_INVALID;
  }
  if ((reinterpret_cast<uintptr_t>(a->grad_acc) & 15) || (reinterpret_cast<uintptr_t>(a->records) & 15) ||
      (!precomp && (reinterpret_cast<uintptr_t>(a->rotations) & 15))) {
    set_error("gsb_preprocess_bwd: grad_acc/records/rotations need 16-byte alignment");
    return GSB_ERR_INVALID;
  }
  cudaStream_t s = (cudaStream_t)stream;
  const bool sh16 = a->sh && a->sh_coeffs == 16 && !(reinterpret_cast<uintptr_t>(a->sh) & 15) &&
                    !(reinterpret_cast<uintptr_t>(a->grad_sh) & 15);
  if (sh16) {
    const int blocks = div_up(threads_needed, PB_SH16_THREADS);
    if (precomp)
      preprocess_bwd_kernel<true, SHM_16><<<blocks, PB_SH16_THREADS, 0, s>>>(*a);
    else
      preprocess_bwd_kernel<false, SHM_16><<<blocks, PB_SH16_THREADS, 0, s>>>(*a);
  } else if (a->sh) {
    const int blocks = div_up(threads_needed, PB_THREADS);
    if (precomp)
      preprocess_bwd_kernel<true, SHM_ANY><<<blocks, PB_THREADS, 0, s>>>(*a);
    else
      preprocess_bwd_kernel<false, SHM_ANY><<<blocks, PB_THREADS, 0, s>>>(*a);
  } else {
    const int blocks = div_up(threads_needed, PB_THREADS);
    if (precomp)
      preprocess_bwd_kernel<true, SHM_NONE><<<blocks, PB_THREADS, 0, s>>>(*a);
    else
      preprocess_bwd_kernel<false, SHM_NONE><<<blocks, PB_THREADS, 0, s>>>(*a);
  }
  return check_launch("preprocess_bwd_kernel");
}
