// preprocess.cu -- per-Gaussian projection, EWA covariance, radius, AccuTile
// tile count and SH colour, fused into one pass over the Gaussians.
//
// Restates gswarp's _fused_project_cov3d_cov2d_preprocess_sr_warp_kernel
// (preprocess_kernels.py:83-269), its cov3D_precomp variant
// (_project_preprocess_visible_points_cov_warp_kernel :630-672 +
// _cov2d_preprocess_masked_pack_warp_kernel :345-476) and
// _forward_rgb_from_sh_v3_warp_kernel (:272-342).  Built with -fmad=false:
// radii, tiles_touched and depth bits must match the CPU oracle bit for bit.
//
// B200 layout: one thread per Gaussian, 256-thread CTAs; view/proj matrices
// staged once per CTA in shared memory; the SH row (up to 192 B) is read with
// 16-byte vector loads only for Gaussians that survive culling; the render
// record (48 B, three float4) is written with vector stores so the render
// kernels gather one Gaussian with three 16-byte loads.
#include "gsb_common.cuh"
#include "gsb_geometry.cuh"
#include "gsb_shrows.cuh"

namespace gsb {
namespace {

__constant__ float SH_C0 = 0.28209479177387814f;
__constant__ float SH_C1 = 0.4886025119029199f;
__constant__ float SH_C2[5] = {1.0925484305920792f, -1.0925484305920792f, 0.31539156525252005f,
                               -1.0925484305920792f, 0.5462742152960396f};
__constant__ float SH_C3[7] = {-0.5900435899266435f, 2.890611442640554f, -0.4570457994644658f,
                               0.3731763325901154f,  -0.4570457994644658f, 1.445305721320277f,
                               -0.5900435899266435f};

// SH degree 0..3 colour (preprocess_kernels.py:272-342).  Coefficient c of
// channel ch lives at sp[c*3+ch].
__device__ __forceinline__ void eval_sh(const float (&sp)[48], int K, int degree, float x,
                                        float y, float z, float col[3]) {
  const float c0 = SH_C0;
#pragma unroll
  for (int ch = 0; ch < 3; ++ch) col[ch] = c0 * sp[ch];
  if (degree > 0 && K > 3) {
    const float c1 = SH_C1;
    float b1 = -c1 * y, b2 = c1 * z, b3 = -c1 * x;
#pragma unroll
    for (int ch = 0; ch < 3; ++ch) col[ch] = col[ch] + b1 * sp[3 + ch];
#pragma unroll
    for (int ch = 0; ch < 3; ++ch) col[ch] = col[ch] + b2 * sp[6 + ch];
#pragma unroll
    for (int ch = 0; ch < 3; ++ch) col[ch] = col[ch] + b3 * sp[9 + ch];
    if (degree > 1 && K > 8) {
      float xx = x * x, yy = y * y, zz = z * z, xy = x * y, yz = y * z, xz = x * z;
      float w[5];
      w[0] = SH_C2[0] * xy;
      w[1] = SH_C2[1] * yz;
      w[2] = SH_C2[2] * (2.0f * zz - xx - yy);
      w[3] = SH_C2[3] * xz;
      w[4] = SH_C2[4] * (xx - yy);
#pragma unroll
      for (int k = 0; k < 5; ++k)
#pragma unroll
        for (int ch = 0; ch < 3; ++ch) col[ch] = col[ch] + w[k] * sp[(4 + k) * 3 + ch];
      if (degree > 2 && K > 15) {
        float v[7];
        v[0] = SH_C3[0] * y * (3.0f * xx - yy);
        v[1] = SH_C3[1] * xy * z;
        v[2] = SH_C3[2] * y * (4.0f * zz - xx - yy);
        v[3] = SH_C3[3] * z * (2.0f * zz - 3.0f * xx - 3.0f * yy);
        v[4] = SH_C3[4] * x * (4.0f * zz - xx - yy);
        v[5] = SH_C3[5] * z * (xx - yy);
        v[6] = SH_C3[6] * x * (xx - 3.0f * yy);
#pragma unroll
        for (int k = 0; k < 7; ++k)
#pragma unroll
          for (int ch = 0; ch < 3; ++ch) col[ch] = col[ch] + v[k] * sp[(9 + k) * 3 + ch];
      }
    }
  }
}

// View-dependent colour of one SH row (zero-padded past K) seen from cam:
// max(SH colour + 0.5, 0), returning the clamp bits (bit ch = channel ch
// was clamped).  Every path that evaluates SH colours goes through here, so
// the per-view preprocess and the multi-view colour kernel agree bit for bit.
__device__ __forceinline__ unsigned sh_colour(const float (&shv)[48], int K, int degree, float p0, float p1,
                                              float p2, float c0, float c1, float c2, float col[3]) {
  const float dx = p0 - c0, dy = p1 - c1, dz = p2 - c2;
  const float len_sq = dx * dx + dy * dy + dz * dz;
  const float inv_len = 1.0f / sqrtf(fmx(len_sq, 1.0e-20f));
  eval_sh(shv, K, degree, dx * inv_len, dy * inv_len, dz * inv_len, col);
  unsigned clamp_bits = 0u;
#pragma unroll
  for (int ch = 0; ch < 3; ++ch) {
    col[ch] = col[ch] + 0.5f;
    if (col[ch] < 0.0f) {
      col[ch] = 0.0f;
      clamp_bits |= 1u << ch;
    }
  }
  return clamp_bits;
}

constexpr int PF_THREADS = launch::PREPROCESS;
constexpr int PF_SH16_THREADS = launch::PREPROCESS_SH16;
constexpr int SH_ROW_F4 = 13;  // staged SH row: 48 floats padded to 52

// SH16: (P,16,3) SH rows, 16-byte aligned.  Each warp then moves the SH rows
// of its 32 consecutive Gaussians (one contiguous 6 KB span) into shared
// memory with coalesced 16-byte loads -- only the rows of Gaussians that
// survive culling -- and each thread evaluates its row from there (rows
// padded to 52 floats: conflict-free 16-byte reads).  Every lane of the warp
// takes part, so threads past P stay in the kernel with nothing to do.
// SH handling, a template parameter so that each variant carries only the
// registers of its own colour path.
enum ShMode { SHM_NONE = 0, SHM_ANY = 1, SHM_16 = 2 };

__device__ __forceinline__ void prefetch_l1(const void* p) { asm volatile("prefetch.global.L1 [%0];" ::"l"(p)); }

template <int SHM>
__global__ void __launch_bounds__(SHM == SHM_16 ? PF_SH16_THREADS : PF_THREADS, SHM == SHM_16 ? 8 : 1)
    preprocess_fwd_kernel(const gsb_preprocess_args a) {
  constexpr bool SH16 = SHM == SHM_16;
  __shared__ float s_view[16], s_proj[16], s_cam[3];
  __shared__ float4 s_rows[SH16 ? PF_SH16_THREADS * SH_ROW_F4 : 1];
  if (threadIdx.x < 16) {
    s_view[threadIdx.x] = a.viewmatrix[threadIdx.x];
    s_proj[threadIdx.x] = a.projmatrix[threadIdx.x];
  } else if (threadIdx.x < 19) {
    s_cam[threadIdx.x - 16] = a.campos ? a.campos[threadIdx.x - 16] : 0.0f;
  }
  __syncthreads();
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  const bool live = idx < a.P;
  if (!SH16 && !live) return;
  const int li = live ? idx : 0;  // in-bounds index for the loads of lanes past P
  // The scale / rotation loads wait for the near-plane test and the colour
  // load for the whole projection and coverage count: their lines are
  // requested now, together with the mean's.
  if (live) {
    if (a.scales) prefetch_l1(a.scales + (size_t)idx * 3);
    if (a.rotations) prefetch_l1(a.rotations + (size_t)idx * 4);
    if (a.colors_precomp) prefetch_l1(a.colors_precomp + (size_t)idx * 3);
    // the warp stages SH rows only after the projection tells which survive
    if (SH16 && a.sh && !a.colors_precomp) {
      prefetch_l1(a.sh + (size_t)idx * 48);
      prefetch_l1(a.sh + (size_t)idx * 48 + 47);
    }
  }
  const float* v = s_view;
  const float* pr = s_proj;
  const int gx = (a.W + BLOCK_X - 1) / BLOCK_X;
  const int gy = (a.H + BLOCK_Y - 1) / BLOCK_Y;

  const float p0 = a.means[li * 3 + 0], p1 = a.means[li * 3 + 1], p2 = a.means[li * 3 + 2];
  const float opacity = a.opacities[li];

  int radius = 0, tiles = 0;
  float depth = 0.0f, px = 0.0f, py = 0.0f;
  float con0 = 0.0f, con1 = 0.0f, con2 = 0.0f;
  float cov_a = 0.0f, cov_b = 0.0f, cov_c = 0.0f;

  // lanes past P take the near-plane-culled path and store nothing
  const float p_view_z = live ? v[2] * p0 + v[6] * p1 + v[10] * p2 + v[14] : 0.0f;
  bool go = false;
  float ppx = 0.0f, ppy = 0.0f;
  bool strict_det = false;
  if (a.cov3d_precomp == nullptr) {
    if (live && a.cov3d_out && !(p_view_z > 0.2f)) {
      float* c3 = a.cov3d_out + (size_t)idx * 6;
      for (int k = 0; k < 6; ++k) c3[k] = 0.0f;  // near-culled: zero (preprocess_kernels.py:116-121)
    }
    if (p_view_z > 0.2f) {
      const float hom_x = pr[0] * p0 + pr[4] * p1 + pr[8] * p2 + pr[12];
      const float hom_y = pr[1] * p0 + pr[5] * p1 + pr[9] * p2 + pr[13];
      const float hom_w = pr[3] * p0 + pr[7] * p1 + pr[11] * p2 + pr[15];
      const float inv_w = 1.0f / (hom_w + 1.0e-7f);
      ppx = hom_x * inv_w;
      ppy = hom_y * inv_w;
      const float s0 = a.scales[idx * 3 + 0] * a.scale_modifier;
      const float s1 = a.scales[idx * 3 + 1] * a.scale_modifier;
      const float s2 = a.scales[idx * 3 + 2] * a.scale_modifier;
      const float4 q = reinterpret_cast<const float4*>(a.rotations)[idx];
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
      if (a.cov3d_out) {
        // preprocess_kernels.py:177-182 (cov3d = M^T M, upper triangle)
        float* c3 = a.cov3d_out + (size_t)idx * 6;
        c3[0] = m00 * m00 + m10 * m10 + m20 * m20;
        c3[1] = m00 * m01 + m10 * m11 + m20 * m21;
        c3[2] = m00 * m02 + m10 * m12 + m20 * m22;
        c3[3] = m01 * m01 + m11 * m11 + m21 * m21;
        c3[4] = m01 * m02 + m11 * m12 + m21 * m22;
        c3[5] = m02 * m02 + m12 * m12 + m22 * m22;
      }
      float vx = v[0] * p0 + v[4] * p1 + v[8] * p2 + v[12];
      float vy = v[1] * p0 + v[5] * p1 + v[9] * p2 + v[13];
      const float vz = p_view_z;
      const float limx = 1.3f * a.tanfovx, limy = 1.3f * a.tanfovy;
      const float txtz = vx / vz, tytz = vy / vz;
      vx = fclamp(txtz, -limx, limx) * vz;
      vy = fclamp(tytz, -limy, limy) * vz;
      const float a_j = a.focal_x / vz, b_j = a.focal_y / vz;
      const float c_j = -(a.focal_x * vx) / (vz * vz);
      const float d_j = -(a.focal_y * vy) / (vz * vz);
      const float t00 = v[0] * a_j + v[2] * c_j;
      const float t10 = v[4] * a_j + v[6] * c_j;
      const float t20 = v[8] * a_j + v[10] * c_j;
      const float t01 = v[1] * b_j + v[2] * d_j;
      const float t11 = v[5] * b_j + v[6] * d_j;
      const float t21 = v[9] * b_j + v[10] * d_j;
      const float a00 = m00 * t00 + m01 * t10 + m02 * t20;
      const float a10 = m10 * t00 + m11 * t10 + m12 * t20;
      const float a20 = m20 * t00 + m21 * t10 + m22 * t20;
      const float a01 = m00 * t01 + m01 * t11 + m02 * t21;
      const float a11 = m10 * t01 + m11 * t11 + m12 * t21;
      const float a21 = m20 * t01 + m21 * t11 + m22 * t21;
      cov_a = a00 * a00 + a10 * a10 + a20 * a20 + 0.3f;
      cov_b = a00 * a01 + a10 * a11 + a20 * a21;
      cov_c = a01 * a01 + a11 * a11 + a21 * a21 + 0.3f;
      go = true;
    }
  } else {
    const float* c3 = a.cov3d_precomp + (size_t)idx * 6;
    if (p_view_z > 0.2f) {
      const float hom_x = pr[0] * p0 + pr[4] * p1 + pr[8] * p2 + pr[12];
      const float hom_y = pr[1] * p0 + pr[5] * p1 + pr[9] * p2 + pr[13];
      const float hom_w = pr[3] * p0 + pr[7] * p1 + pr[11] * p2 + pr[15];
      const float inv_w = 1.0f / (hom_w + 1.0e-7f);
      ppx = hom_x * inv_w;
      ppy = hom_y * inv_w;
      // conservative visibility (math_kernels.py:104-134, 392-406)
      const float row0 = fabsf(c3[0]) + fabsf(c3[1]) + fabsf(c3[2]);
      const float row1 = fabsf(c3[1]) + fabsf(c3[3]) + fabsf(c3[4]);
      const float row2 = fabsf(c3[2]) + fabsf(c3[4]) + fabsf(c3[5]);
      const float lam = fmx(row0, fmx(row1, row2));
      const float limx = 1.3f * a.tanfovx, limy = 1.3f * a.tanfovy;
      const float fx = (float)a.W / (2.0f * a.tanfovx);
      const float fy = (float)a.H / (2.0f * a.tanfovy);
      const float row0n = (fx / p_view_z) * sqrtf(1.0f + limx * limx);
      const float row1n = (fy / p_view_z) * sqrtf(1.0f + limy * limy);
      const float jf = row0n * row0n + row1n * row1n;
      const float lu = lam * jf + 0.3f;
      const int radius_upper = f2i(ceilf(3.0f * sqrtf(fmx(lu, 0.0f))));
      const Rect rr = tile_rect(ndc2pix(ppx, a.W), ndc2pix(ppy, a.H), radius_upper, gx, gy);
      if ((rr.x1 - rr.x0) * (rr.y1 - rr.y0) != 0) {
        float x = v[0] * p0 + v[4] * p1 + v[8] * p2 + v[12];
        float y = v[1] * p0 + v[5] * p1 + v[9] * p2 + v[13];
        const float z = v[2] * p0 + v[6] * p1 + v[10] * p2 + v[14];
        const float txtz = x / z, tytz = y / z;
        x = fclamp(txtz, -limx, limx) * z;
        y = fclamp(tytz, -limy, limy) * z;
        const float ja = a.focal_x / z, jb = a.focal_y / z;
        const float jc = -(a.focal_x * x) / (z * z);
        const float jd = -(a.focal_y * y) / (z * z);
        const float t00 = v[0] * ja + v[2] * jc;
        const float t10 = v[4] * ja + v[6] * jc;
        const float t20 = v[8] * ja + v[10] * jc;
        const float t01 = v[1] * jb + v[2] * jd;
        const float t11 = v[5] * jb + v[6] * jd;
        const float t21 = v[9] * jb + v[10] * jd;
        const float v00 = c3[0], v01 = c3[1], v02 = c3[2], v11 = c3[3], v12 = c3[4], v22 = c3[5];
        const float vt0x = v00 * t00 + v01 * t10 + v02 * t20;
        const float vt0y = v01 * t00 + v11 * t10 + v12 * t20;
        const float vt0z = v02 * t00 + v12 * t10 + v22 * t20;
        const float vt1x = v00 * t01 + v01 * t11 + v02 * t21;
        const float vt1y = v01 * t01 + v11 * t11 + v12 * t21;
        const float vt1z = v02 * t01 + v12 * t11 + v22 * t21;
        cov_a = t00 * vt0x + t10 * vt0y + t20 * vt0z + 0.3f;
        cov_b = t00 * vt1x + t10 * vt1y + t20 * vt1z;
        cov_c = t01 * vt1x + t11 * vt1y + t21 * vt1z + 0.3f;
        go = true;
        strict_det = true;
      }
    }
  }

  if (go) {
    // preprocess_kernels.py:221-269 (and :439-476 with a strict det test)
    const float det = cov_a * cov_c - cov_b * cov_b;
    const bool degenerate = strict_det ? (fabsf(det) < DET_EPSILON) : (fabsf(det) <= DET_EPSILON);
    if (!degenerate) {
      const float det_inv = 1.0f / det;
      const float k0 = cov_c * det_inv, k1 = -cov_b * det_inv, k2 = cov_a * det_inv;
      const float mid = 0.5f * (cov_a + cov_c);
      const float root = sqrtf(fmx(0.1f, mid * mid - det));
      const float l1 = mid + root, l2 = mid - root;
      const int rad = f2i(ceilf(3.0f * sqrtf(fmx(l1, l2))));
      const float qx = ndc2pix(ppx, a.W);
      const float qy = ndc2pix(ppy, a.H);
      const Rect cr = tile_rect(qx, qy, rad, gx, gy);
      if ((cr.x1 - cr.x0) * (cr.y1 - cr.y0) != 0) {
        radius = rad;
        depth = p_view_z;
        px = qx;
        py = qy;
        con0 = k0;
        con1 = k1;
        con2 = k2;
        Rect br;
        float bt;
        coverage_setup(px, py, cov_a, cov_c, opacity, radius, gx, gy, br, bt);
        unsigned brec[8];
        tiles = coverage_record(px, py, con0, con1, con2, bt, br, a.coverage_mode, brec);
        if (a.bin_records && tiles > 0) {
          uint4* d = reinterpret_cast<uint4*>(a.bin_records) + (size_t)idx * 2;
          d[0] = make_uint4(brec[0], brec[1], brec[2], brec[3]);
          d[1] = make_uint4(brec[4], brec[5], brec[6], brec[7]);
        }
      } else {
        cov_a = cov_b = cov_c = 0.0f;
      }
    } else {
      cov_a = cov_b = cov_c = 0.0f;
    }
  } else {
    cov_a = cov_b = cov_c = 0.0f;
  }

  // Colour: only Gaussians that can be rendered need it; the SH backward
  // only reads the clamp flags where the render gradient is non-zero.
  float col[3] = {0.0f, 0.0f, 0.0f};
  unsigned clamp_bits = 0u;
  if (SH16) {
    const bool need = radius > 0 && a.colors_precomp == nullptr;
    const unsigned need_mask = __ballot_sync(0xffffffffu, need);
    float4* rows = s_rows + (threadIdx.x & ~31) * SH_ROW_F4;
    const int lane = threadIdx.x & 31;
    if (need_mask) {
      const float4* src = reinterpret_cast<const float4*>(a.sh) + (size_t)(idx & ~31) * 12;
#pragma unroll 4
      for (int j = lane; j < 32 * 12; j += 32) {
        const int r = j / 12;
        if ((need_mask >> r) & 1u) rows[r * SH_ROW_F4 + (j - r * 12)] = __ldg(src + j);
      }
    }
    __syncwarp();
    if (need) {
      float shv[48];
      const float4* row = rows + lane * SH_ROW_F4;
#pragma unroll
      for (int q = 0; q < 12; ++q) {
        const float4 t = row[q];
        shv[q * 4 + 0] = t.x;
        shv[q * 4 + 1] = t.y;
        shv[q * 4 + 2] = t.z;
        shv[q * 4 + 3] = t.w;
      }
      clamp_bits = sh_colour(shv, 16, a.sh_degree, p0, p1, p2, s_cam[0], s_cam[1], s_cam[2], col);
    }
    if (!live) return;
  } else if (radius > 0) {
    if (a.colors_precomp) {
      col[0] = a.colors_precomp[idx * 3 + 0];
      col[1] = a.colors_precomp[idx * 3 + 1];
      col[2] = a.colors_precomp[idx * 3 + 2];
      if (a.colors_clamp_signed) {
        // multi-view SH colours: -0.0 marks a clamped channel
#pragma unroll
        for (int ch = 0; ch < 3; ++ch)
          if (signbit(col[ch])) {
            col[ch] = 0.0f;
            clamp_bits |= 1u << ch;
          }
      }
    } else if (SHM == SHM_ANY && a.sh) {
      const float* sp = a.sh + (size_t)idx * a.sh_coeffs * 3;
      // The first 16 coefficients of the row, with 16-byte loads when the row
      // is an aligned 48-float record (SH degree 3).
      float shv[48];
      if (a.sh_coeffs == 16 && (reinterpret_cast<uintptr_t>(sp) & 15) == 0) {
        const float4* s4p = reinterpret_cast<const float4*>(sp);
#pragma unroll
        for (int q = 0; q < 12; ++q) {
          const float4 v = __ldg(s4p + q);
          shv[q * 4 + 0] = v.x;
          shv[q * 4 + 1] = v.y;
          shv[q * 4 + 2] = v.z;
          shv[q * 4 + 3] = v.w;
        }
      } else {
        const int nsh = (a.sh_coeffs < 16 ? a.sh_coeffs : 16) * 3;
#pragma unroll
        for (int k = 0; k < 48; ++k) shv[k] = k < nsh ? __ldg(sp + k) : 0.0f;
      }
      clamp_bits = sh_colour(shv, a.sh_coeffs, a.sh_degree, p0, p1, p2, s_cam[0], s_cam[1], s_cam[2], col);
    }
  }

  a.radii[idx] = radius;
  a.depths[idx] = depth;
  a.tiles_touched[idx] = tiles;
  if (a.proj_2d) reinterpret_cast<float2*>(a.proj_2d)[idx] = make_float2(px, py);
  if (a.conic_2d) {
    a.conic_2d[idx * 3 + 0] = con0;
    a.conic_2d[idx * 3 + 1] = con1;
    a.conic_2d[idx * 3 + 2] = con2;
  }
  if (a.conic_2d_inv) {
    a.conic_2d_inv[idx * 3 + 0] = cov_a;
    a.conic_2d_inv[idx * 3 + 1] = cov_b;
    a.conic_2d_inv[idx * 3 + 2] = cov_c;
  }
  if (radius > 0 || !a.sparse_records) {
    float4* rec = reinterpret_cast<float4*>(a.records) + (size_t)idx * 3;
    const float op_rec = radius > 0 ? opacity : 0.0f;
    rec[0] = make_float4(px, py, con0, con1);
    rec[1] = make_float4(con2, op_rec, depth, __uint_as_float(clamp_bits));
    rec[2] = make_float4(col[0], col[1], col[2], 0.0f);
  }
}

// Multi-view SH colours: one thread per Gaussian, 128-thread CTAs.  Each
// warp stages the SH rows of its 32 consecutive Gaussians (one contiguous
// span of 32*K*3 floats) in shared memory with coalesced loads, each thread
// copies its row to registers once and evaluates it from every camera.
constexpr int SHV_THREADS = launch::SH_COLORS_VIEWS;
constexpr int SHV_ROW_F = 49;  // 48 floats padded: per-thread scalar reads hit 32 banks

__global__ void __launch_bounds__(SHV_THREADS) sh_colors_views_kernel(const gsb_sh_views_args a) {
  __shared__ float s_rows[SHV_THREADS * SHV_ROW_F];
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  const int lane = threadIdx.x & 31;
  const int base = idx - lane;
  if (base >= a.P) return;  // whole warp past P
  const int K = a.sh_coeffs, RF = K * 3;
  float* rows = s_rows + (threadIdx.x & ~31) * SHV_ROW_F;
  sh_rows_load<SHV_ROW_F>(rows, a.sh + (size_t)base * RF, RF, min(32, a.P - base), 0xffffffffu, lane);
  __syncwarp();
  if (idx >= a.P) return;
  float shv[48];
  const float* row = rows + lane * SHV_ROW_F;
#pragma unroll
  for (int e = 0; e < 48; ++e) shv[e] = e < RF ? row[e] : 0.0f;
  const float p0 = a.means[idx * 3 + 0], p1 = a.means[idx * 3 + 1], p2 = a.means[idx * 3 + 2];
  for (int v = 0; v < a.num_views; ++v) {
    const float* cam = a.campos + v * 3;
    float col[3];
    const unsigned clamp_bits = sh_colour(shv, K, a.sh_degree, p0, p1, p2, __ldg(cam), __ldg(cam + 1),
                                          __ldg(cam + 2), col);
    float* out = a.colors + ((size_t)v * a.P + idx) * 3;
#pragma unroll
    for (int ch = 0; ch < 3; ++ch) out[ch] = ((clamp_bits >> ch) & 1u) ? -0.0f : col[ch];
  }
}

__global__ void mark_visible_kernel(int P, const float* __restrict__ means,
                                    const float* __restrict__ view, uint8_t* out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= P) return;
  const float z = view[2] * means[i * 3] + view[6] * means[i * 3 + 1] +
                  view[10] * means[i * 3 + 2] + view[14];
  out[i] = z > 0.2f ? 1 : 0;
}

__global__ void threshold_log_kernel(const float* in, float* out, long long n) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = crlogf(in[i]);
}

}  // namespace
}  // namespace gsb

using namespace gsb;

GSB_EXPORT int gsb_preprocess_fwd(const gsb_preprocess_args* a, void* stream) {
  if (!a || a->P < 0 || a->W <= 0 || a->H <= 0) {
    set_error("gsb_preprocess_fwd: invalid sizes");
    return GSB_ERR_INVALID;
  }
  if (a->P == 0) return GSB_OK;
  const bool sr = a->scales && a->rotations;
  if (sr == (a->cov3d_precomp != nullptr)) {
    set_error("gsb_preprocess_fwd: provide exactly one of scales/rotations or cov3d_precomp");
    return GSB_ERR_INVALID;
  }
  if (!a->means || !a->opacities || !a->viewmatrix || !a->projmatrix || !a->radii ||
      !a->depths || !a->tiles_touched || !a->records) {
    set_error("gsb_preprocess_fwd: null pointer argument");
    return GSB_ERR_INVALID;
  }
  if (a->sh && (a->sh_coeffs <= 0 || !a->campos)) {
    set_error("gsb_preprocess_fwd: SH colours need sh_coeffs > 0 and campos");
    return GSB_ERR_INVALID;
  }
  if ((reinterpret_cast<uintptr_t>(a->records) & 15) ||
      (a->rotations && (reinterpret_cast<uintptr_t>(a->rotations) & 15)) ||
      (reinterpret_cast<uintptr_t>(a->proj_2d) & 7)) {
    set_error("gsb_preprocess_fwd: records/rotations need 16-byte and proj_2d 8-byte alignment");
    return GSB_ERR_INVALID;
  }
  if (a->bin_records && ((reinterpret_cast<uintptr_t>(a->bin_records) & 15) ||
                         div_up(a->W, BLOCK_X) > 65535 || div_up(a->H, BLOCK_Y) > 65535)) {
    set_error("gsb_preprocess_fwd: bin_records needs 16-byte alignment and tile grids below 65536");
    return GSB_ERR_INVALID;
  }
  const bool sh16 = a->sh && !a->colors_precomp && a->sh_coeffs == 16 &&
                    !(reinterpret_cast<uintptr_t>(a->sh) & 15);
  cudaStream_t s = (cudaStream_t)stream;
  if (sh16)
    preprocess_fwd_kernel<SHM_16><<<div_up(a->P, PF_SH16_THREADS), PF_SH16_THREADS, 0, s>>>(*a);
  else if (a->sh && !a->colors_precomp)
    preprocess_fwd_kernel<SHM_ANY><<<div_up(a->P, PF_THREADS), PF_THREADS, 0, s>>>(*a);
  else
    preprocess_fwd_kernel<SHM_NONE><<<div_up(a->P, PF_THREADS), PF_THREADS, 0, s>>>(*a);
  return check_launch("preprocess_fwd_kernel");
}

GSB_EXPORT int gsb_sh_colors_views(const gsb_sh_views_args* a, void* stream) {
  if (!a || a->P < 0 || a->num_views < 0 || a->sh_coeffs < 1 || a->sh_coeffs > 16 || a->sh_degree < 0 ||
      a->sh_degree > 3) {
    set_error("gsb_sh_colors_views: invalid sizes (P, num_views >= 0; 1 <= sh_coeffs <= 16; degree 0..3)");
    return GSB_ERR_INVALID;
  }
  if (a->P == 0 || a->num_views == 0) return GSB_OK;
  if (!a->means || !a->sh || !a->campos || !a->colors) {
    set_error("gsb_sh_colors_views: null pointer argument");
    return GSB_ERR_INVALID;
  }
  sh_colors_views_kernel<<<div_up(a->P, SHV_THREADS), SHV_THREADS, 0, (cudaStream_t)stream>>>(*a);
  return check_launch("sh_colors_views_kernel");
}

GSB_EXPORT int gsb_mark_visible(int P, const float* means, const float* viewmatrix, uint8_t* out,
                                void* stream) {
  if (P < 0 || (P > 0 && (!means || !viewmatrix || !out))) {
    set_error("gsb_mark_visible: invalid arguments");
    return GSB_ERR_INVALID;
  }
  if (P == 0) return GSB_OK;
  mark_visible_kernel<<<div_up(P, 256), 256, 0, (cudaStream_t)stream>>>(P, means, viewmatrix, out);
  return check_launch("mark_visible_kernel");
}

GSB_EXPORT int gsb_selftest_threshold_log(const float* in, float* out, long long n, void* stream) {
  if (n < 0 || (n > 0 && (!in || !out))) {
    set_error("gsb_selftest_threshold_log: invalid arguments");
    return GSB_ERR_INVALID;
  }
  if (n == 0) return GSB_OK;
  threshold_log_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(in, out, n);
  return check_launch("threshold_log_kernel");
}
